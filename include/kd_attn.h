/*
 * kd_attn.h -- C ABI of libkd_attn, the B200 (sm_100a) attention library
 * behind kandinsky.cpp's CrossDiT attention.
 *
 * Drop-in boundary.  kandinsky.cpp routes both CrossDiT attention call sites
 * through ops::attention (src/core/ops.hpp:107-207):
 *   - DiTSelfAttention::forward  (src/models/crossdit.hpp:117-154; call at :150)
 *   - DiTCrossAttention::forward (src/models/crossdit.hpp:174-200; call at :198)
 * whose flash branch builds ggml_flash_attn_ext(q, k, v, mask, scale, 0, 0)
 * (ops.hpp:176) with Q f32, K/V cast to f16 (ops.hpp:167-169), an optional f16
 * mask, precision F32 (ops.hpp:177).  The entry points below replace that
 * operator and the RMSNorm / RoPE graph ops in front of it.
 *
 * Conventions (mirroring include/kandinsky.h of the reference):
 *   - every call returns a kd_attn_status; 0 is success, negative is an error
 *     (kandinsky.h returns -1 / NULL on error, kandinsky.h:77-89);
 *   - the caller owns every buffer passed in; the library never frees them;
 *   - device pointers only in kd_tensor.data (except where noted), work is
 *     enqueued on the given cudaStream_t (passed as void*), nothing blocks;
 *   - a context may be used from one host thread at a time, and its calls share
 *     the context's device scratch: issue them on one stream, or order calls on
 *     different streams with events (the host-buffer call orders its own copy
 *     streams after the given stream);
 *   - there is no CPU fallback: shapes the kernels do not cover return
 *     KD_ATTN_ERR_UNSUPPORTED and the caller keeps its own path;
 *   - kd_tensor mirrors ggml_tensor's {type, ne[4], nb[4], data}, sizes in
 *     elements with dim 0 fastest and strides in bytes, so a ggml tensor maps
 *     onto it field by field.
 */
#ifndef KD_ATTN_H
#define KD_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KD_ATTN_VERSION_MAJOR 0
#define KD_ATTN_VERSION_MINOR 2

typedef enum {
    KD_ATTN_OK = 0,
    KD_ATTN_ERR_INVALID_ARGUMENT = -1, /* null pointer, inconsistent shapes or strides */
    KD_ATTN_ERR_UNSUPPORTED = -2,      /* valid for ggml but not covered here (e.g. head_dim 96) */
    KD_ATTN_ERR_CUDA = -3,             /* a CUDA runtime call failed; see kd_attn_last_error */
    KD_ATTN_ERR_OUT_OF_MEMORY = -4,    /* context scratch could not grow */
    KD_ATTN_ERR_DEVICE_TIMEOUT = -5,   /* a bounded device-side wait expired (kd_attn_device_status) */
    KD_ATTN_ERR_NCCL = -6,             /* the head all-gather failed */
} kd_attn_status;

/* Same values and callback shape as kandinsky.h:12-19 (kd_log_level_t / kd_log_cb_t),
 * so the host application's logger can be passed through unchanged. */
typedef enum {
    KD_ATTN_LOG_DEBUG = 0,
    KD_ATTN_LOG_INFO = 1,
    KD_ATTN_LOG_WARN = 2,
    KD_ATTN_LOG_ERROR = 3,
} kd_attn_log_level;
typedef void (*kd_attn_log_cb)(kd_attn_log_level level, const char* text, void* user_data);

/* ggml type ids (ggml.h: GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1, GGML_TYPE_BF16 = 30) */
typedef enum {
    KD_ATTN_TYPE_F32 = 0,
    KD_ATTN_TYPE_F16 = 1,
    KD_ATTN_TYPE_BF16 = 30,
} kd_attn_type;

typedef struct {
    void* data;     /* device pointer */
    int32_t type;   /* kd_attn_type */
    int64_t ne[4];  /* sizes, dim 0 fastest (ggml ne) */
    size_t nb[4];   /* strides in bytes (ggml nb) */
} kd_tensor;

/* 3D (t, h, w) rotary embedding of the visual tokens, computed on the fly
 * (replaces rope::compute_visual_rope, src/rope.hpp:56-102, and the table
 * upload at crossdit.hpp:562-565,601-602).  Token l of a sequence sits at
 * t = l / (grid[1]*grid[2]), h = (l / grid[2]) % grid[1], w = l % grid[2]
 * (rope.hpp:74).  Axis a rotates the pairs of its axes_dim[a] block with
 * angle = pos_a * theta^(-i/(axes_dim[a]/2)) / scale_factor[a]. */
typedef struct {
    int32_t axes_dim[3];    /* {32, 48, 48} for Kandinsky 5 (crossdit.hpp:73) */
    int32_t grid[3];        /* token grid (frames, height, width) after patching */
    float scale_factor[3];  /* {1, 2, 2} in the Pro configs (crossdit.hpp:73) */
    float theta;            /* 10000 (rope.hpp:60) */
} kd_rope3d;

typedef struct kd_attn_ctx kd_attn_ctx;

typedef struct {
    int32_t device;              /* CUDA device ordinal */
    int32_t n_ranks;             /* head-sharding group size (1 = single GPU) */
    int32_t rank;                /* this process's rank in the group */
    const void* nccl_unique_id;  /* n_ranks > 1: the 128-byte ncclUniqueId every rank of the group
                                    received from rank 0's kd_attn_nccl_unique_id; the context then
                                    owns an NCCL communicator (kd_attn_create is collective) */
    kd_attn_log_cb log_cb;       /* NULL: messages go to stderr at WARN and above */
    void* log_user_data;
} kd_attn_init;

/* Fills out[128] with a fresh ncclUniqueId (rank 0 calls it and shares the
 * bytes with the group out of band).  NCCL is loaded on demand (libnccl.so.2,
 * or the path in $KD_ATTN_NCCL_LIB). */
kd_attn_status kd_attn_nccl_unique_id(void* out128);

/* Replaces: nothing in the reference holds attention state; ggml's backend and
 * gallocr (src/core/executor.hpp:99-259) play this role.  Creates the per-device
 * context that owns the operand scratch, the device error word and (for
 * n_ranks > 1) the NCCL communicator.
 * Returns KD_ATTN_OK and *out, or an error and *out = NULL. */
kd_attn_status kd_attn_create(const kd_attn_init* init, kd_attn_ctx** out);
void kd_attn_destroy(kd_attn_ctx* ctx);

/* Process-wide log callback (kandinsky.h:19 kd_log_cb_t shape): used by contexts
 * created with log_cb = NULL and by kd_attn_flash_ext_noalloc; NULL restores
 * the default (WARN and above to stderr).  Thread-safe. */
void kd_attn_set_log_callback(kd_attn_log_cb cb, void* user_data);

/* Text of the last error raised on this context ("" when none). */
const char* kd_attn_last_error(const kd_attn_ctx* ctx);

/* Synchronises `stream`, then reads and clears the device error word that the
 * kernels' bounded waits set; KD_ATTN_ERR_DEVICE_TIMEOUT if any wait expired. */
kd_attn_status kd_attn_device_status(kd_attn_ctx* ctx, void* stream);

/* Device counters of the flash kernel, accumulated over every launch on this
 * context since the last reset: out[0] = K/V tiles (128 keys) loaded, out[1] =
 * (Q tile of 128 rows) x (K/V tile) products computed.  Fully masked tiles are
 * neither loaded nor computed, so with a block-sparse mask these equal the
 * counts of kept tiles that the mask implies.  Synchronises `stream`; reset != 0
 * zeroes the counters after reading.  No reference counterpart. */
kd_attn_status kd_attn_tile_stats(kd_attn_ctx* ctx, void* stream, uint64_t out[2], int32_t reset);

/* Self-test of failure detection: launches one bounded device wait that nothing
 * releases (the wait the kernels use, on a barrier nobody arrives on).  After
 * wait_ms (1..10000) it gives up and sets the context's error word, so the next
 * kd_attn_device_status returns KD_ATTN_ERR_DEVICE_TIMEOUT (and clears it); the
 * context stays usable.  Nothing faults, traps or spins without a bound. */
kd_attn_status kd_attn_selftest_wait(kd_attn_ctx* ctx, uint32_t wait_ms, void* stream);

/* ---------------------------------------------------------------------------
 * Prologue: RMSNorm per head + 3D RoPE + cast + permute, one HBM pass.
 * Replaces, per projection x (crossdit.hpp:132-141, :188-193):
 *   ggml_reshape_4d(x, d, H, L, N)                          crossdit.hpp:132-133
 *   RMSNorm::forward = ggml_rms_norm(eps) * weight          module.hpp:177, ops.hpp:76-81
 *   rope::apply(x, table)                                   rope.hpp:109-155
 *   ggml_cont(ggml_permute(.., 0,2,1,3)) + ggml_cast(F16)   ops.hpp:122-131,167-169
 * x : [H*d, L, N] f32 (ggml [C, L, N] from to_query/to_key/to_value)
 * y : [d, L, H, N] of type f16, bf16 or f32 (the flash operand layout)
 * norm: 0 = no RMSNorm (V), 1 = RMSNorm with `gain` (device [d], NULL = unit gain)
 * rope: NULL = no rotation (cross-attention, V).  With rope, axes_dim must sum
 *       to d and grid must multiply to L.
 * d = x.ne[0] / n_head is 128 (CrossDiT pro_video, lite_image) or 64 (lite_video:
 * 28 heads of 1792 channels, axes {16, 24, 24}, crossdit.hpp:36,48-56). */
kd_attn_status kd_attn_prologue(kd_attn_ctx* ctx, const kd_tensor* x, int32_t n_head, int32_t norm,
                                const float* gain, float eps, const kd_rope3d* rope, kd_tensor* y,
                                void* stream);

/* The prologue of one attention call in ONE launch: Q and K RMS-normalised
 * (q_gain / k_gain, NULL = unit gain) and, when `rope` is given, rotated; V only
 * permuted and cast (crossdit.hpp:132-141 for self-attention, :188-193 for
 * cross-attention, + ops.hpp:122-131,167-169).  Tensors of equal length are
 * processed row by row together (one sin/cos per token).  Any of the three
 * pairs may be NULL.  n_head comes from the outputs' ne[2]; all outputs have
 * type `out_dtype` (f16, bf16 or f32). */
kd_attn_status kd_attn_qk_prologue(kd_attn_ctx* ctx, const kd_tensor* q_in, const kd_tensor* k_in,
                                   const kd_tensor* v_in, const float* q_gain, const float* k_gain, float eps,
                                   const kd_rope3d* rope, int32_t out_dtype, kd_tensor* q_out,
                                   kd_tensor* k_out, kd_tensor* v_out, void* stream);

/* ---------------------------------------------------------------------------
 * QKV projection with the prologue as its epilogue.
 * Replaces, for one attention block, the three Linear layers and everything up to
 * the flash operands:
 *   q, k, v = to_query/to_key/to_value(x)       crossdit.hpp:123-125 (ops::linear, ops.hpp:27-42:
 *                                               ggml_mul_mat(w, x) + bias)
 *   + the prologue of kd_attn_qk_prologue        crossdit.hpp:132-141, ops.hpp:122-131,167-169
 * as one tensor-core GEMM whose epilogue adds the bias, RMS-normalises Q and K
 * per head (q_gain / k_gain, NULL = unit gain), applies the 3D RoPE when `rope`
 * is given, casts, and stores [d, L, H, N] operands: the f32 projections are
 * never written to memory.  The GEMM runs in bf16 with fp32 accumulation; quantized
 * weights are expanded to bf16 first (q8_0: value d*q; q4_0: value d*(q-8), element
 * j in the low nibble and j+16 in the high one -- ggml's block formats, as
 * scripts/convert_to_gguf.py:90-146 writes them).
 * x     : [K, L, N] f32, rows 16-byte aligned; K a multiple of 32
 * wq/wk/wv : weights in ggml layout [K, C] (row r = output feature r); any of the
 *         three may be NULL together with its output (e.g. the Q projection of
 *         cross-attention alone, or its K/V projection of the text states)
 * q_out/k_out/v_out : [d, L, H, N] f16 or bf16 (= out_dtype), d = 128 or 64 (the
 *         lite video model; rope axes then sum to 64), H*d = C a multiple of 256,
 *         rows 16-byte aligned.  Q and K are normalised (and
 *         rotated), V only cast. */
#define KD_ATTN_TYPE_Q4_0 2 /* ggml.h GGML_TYPE_Q4_0: 18-byte blocks of 32 (f16 scale, 16 bytes of nibbles) */
#define KD_ATTN_TYPE_Q8_0 8 /* ggml.h GGML_TYPE_Q8_0: 34-byte blocks of 32 (f16 scale, 32 int8) */
typedef struct {
    const void* data;   /* device pointer to C rows of K elements of `type` */
    int32_t type;       /* KD_ATTN_TYPE_F32 / F16 / BF16 / Q4_0 / Q8_0 */
    int64_t ne[2];      /* {K, C} (ggml ne of the weight tensor) */
    size_t nb1;         /* bytes between rows (ggml nb[1]) */
    const float* bias;  /* device f32 [C] or NULL */
} kd_linear;

kd_attn_status kd_attn_qkv_projection(kd_attn_ctx* ctx, const kd_tensor* x, const kd_linear* wq,
                                      const kd_linear* wk, const kd_linear* wv, const float* q_gain,
                                      const float* k_gain, float eps, const kd_rope3d* rope, int32_t out_dtype,
                                      kd_tensor* q_out, kd_tensor* k_out, kd_tensor* v_out, void* stream);

/* Replaces ops::linear (ops.hpp:27-42): y = x W^T + b, the same GEMM as the projection with a plain
 * bias epilogue -- the out-projection of the attention blocks (crossdit.hpp:153).
 * x : [K, L, N] f32 (rounded to bf16 rows inside the call) or bf16 (read in place: K a multiple of
 *     128, rows evenly spaced and 16-byte aligned)
 * w : [K, C] (C a multiple of 256), types as for kd_attn_qkv_projection
 * y : [C, L, N] f32, bf16 or f16, rows contiguous and 16-byte aligned */
kd_attn_status kd_attn_linear(kd_attn_ctx* ctx, const kd_tensor* x, const kd_linear* w, kd_tensor* y, void* stream);

/* Replaces DiTSelfAttention::forward (crossdit.hpp:117-154) from the hidden states to the block output:
 * kd_attn_qkv_projection (bf16 operands), the flash kernel (scale 1/sqrt(d), no mask) and the
 * out-projection, with the intermediate tensors in the context's scratch.
 * x : [C, L, N] f32; wq/wk/wv : [C, C]; wo : [C, C_out]; n_head : the module's num_heads, head dim
 * d = C / n_head = 128 (pro_video, lite_image) or 64 (lite_video); q_gain/k_gain : RMSNorm weights
 * [d] (NULL = unit); rope : NULL = no rotation, else axes summing to d; y : [C_out, L, N] f32 (or
 * bf16/f16). */
kd_attn_status kd_attn_self_attention_block(kd_attn_ctx* ctx, const kd_tensor* x, const kd_linear* wq,
                                            const kd_linear* wk, const kd_linear* wv, const kd_linear* wo,
                                            int32_t n_head, const float* q_gain, const float* k_gain, float eps,
                                            const kd_rope3d* rope, kd_tensor* y, void* stream);

/* Replaces DiTCrossAttention::forward (crossdit.hpp:174-200): visual queries from x_query [C, Lq, N] f32,
 * keys and values from the text states x_kv [C, Lk, N] f32 (RMSNorm on Q and K, no RoPE), flash
 * attention with the text's valid lengths -- kv_len (device int32 [N]) and/or an f16 mask as for
 * kd_attn_flash_ext, either may be NULL -- and the out-projection; y : [C_out, Lq, N].  n_head as
 * for kd_attn_self_attention_block. */
kd_attn_status kd_attn_cross_attention_block(kd_attn_ctx* ctx, const kd_tensor* x_query, const kd_tensor* x_kv,
                                             const kd_linear* wq, const kd_linear* wk, const kd_linear* wv,
                                             const kd_linear* wo, int32_t n_head, const float* q_gain,
                                             const float* k_gain, float eps, const kd_tensor* mask,
                                             const int32_t* kv_len, kd_tensor* y, void* stream);

/* ---------------------------------------------------------------------------
 * ggml_flash_attn_ext semantics (called at ops.hpp:176):
 *   out[:, h, i, n] = softmax_j(scale * q[:, i, h, n] . k[:, j, hk, nk] + mask[j, i, h%mh, n%mn]) v[:, j, hk, nk]
 * q    : [D, Lq, H, N]      f32 | f16 | bf16 (f32 is rounded to K's type first,
 *                           as ggml's CPU op rounds Q to the dot type)
 * k, v : [D, Lk, Hkv, Nkv]  f16 | bf16, same type; H % Hkv == 0 and N % Nkv == 0
 *                           (GQA broadcast as in ggml)
 * mask : NULL or f16 [>=Lk, >=Lq, mh, mn], additive, -inf marks a masked key;
 *        H % mh == 0, N % mn == 0.  Tiles that are entirely -inf are skipped.
 * kv_len: NULL or device int32 [N]: keys j >= kv_len[n] are masked (the
 *        variable text length of cross-attention without a dense mask).
 * tile_mask: NULL or a device bitmap of 64 x 64 (query x key) tiles shared by
 *        every head and sequence: tile (qb, kb) is bit (kb % 8) of byte
 *        tile_mask[qb * ceil(Lk/64 / 8) + kb / 8], qb < ceil(Lq/64),
 *        kb < ceil(Lk/64).  A clear bit means every pair in the tile is masked:
 *        the tile is skipped and its mask elements are never read.  Without a
 *        dense mask a set bit means the whole tile is kept (a block-sparse mask
 *        in 1/8192 of the dense mask's bytes); with one, set tiles take their
 *        values from the mask.  No ggml counterpart.
 * out  : [D, H, Lq, N] f32 | bf16 | f16 (ggml's dst permutation; with
 *        contiguous strides this is [H*D, Lq, N], the ops::attention result)
 * lse  : NULL or device f32 [N, H, Lq], natural-log softmax denominator
 *        (ln sum_j exp(scale*q.k_j + mask_j)); -inf for fully masked rows.
 * max_bias and logit_softcap must be 0 (the only values ops.hpp:176 passes).
 * Rows whose keys are all masked produce 0.  D is 128, 64 (the lite video model's
 * heads, crossdit.hpp:36,48-56: same kernel, one 64-column box per tile), or 512 -- one
 * head of a VAE mid block (src/models/vae.hpp:89) -- with no mask, kv_len or tile_mask
 * and at least one key. */
kd_attn_status kd_attn_flash_ext(kd_attn_ctx* ctx, const kd_tensor* q, const kd_tensor* k,
                                 const kd_tensor* v, const kd_tensor* mask, float scale,
                                 float max_bias, float logit_softcap, const int32_t* kv_len,
                                 const uint8_t* tile_mask, kd_tensor* out, float* lse, void* stream);

/* ---------------------------------------------------------------------------
 * Allocation-free variant of kd_attn_flash_ext.  It has no counterpart in the
 * reference.  It is for callers that may not allocate device memory: embedders
 * whose device memory belongs to another allocator (a ggml backend buffer, a
 * serving runtime's arena) and who may not call cudaMalloc behind its back, or
 * code that runs where the CUDA runtime forbids allocation.  It needs no
 * kd_attn_ctx (whose creation allocates) and calls no cudaMalloc, cudaFree or
 * allocating library routine.
 *
 * Same arguments and semantics as kd_attn_flash_ext; it runs on the calling
 * thread's current CUDA device, and every buffer it is given must be device
 * memory of that device (else KD_ATTN_ERR_INVALID_ARGUMENT).  Its scratch (Q
 * rounded to the operand type when Q is f32 or strided, plus the mask's tile
 * classes) lives in one statically sized device array of
 * KD_ATTN_NOALLOC_SCRATCH_BYTES that belongs to the library's device code: it
 * is allocated on a device when that code is loaded there -- under CUDA's
 * default lazy module loading at this entry point's first call on the device,
 * with CUDA_MODULE_LOADING=EAGER as soon as the library's kernels are loaded,
 * whichever entry point is used -- and it is held until the process exits.
 * Problems that need more scratch than that are rejected with
 * KD_ATTN_ERR_UNSUPPORTED before anything is launched (Q already in K's type
 * with 16-byte-aligned rows needs none).
 *   - The first call on a device looks up that array's device address; make
 *     that first call before any stream capture begins.
 *   - Every call on a device shares the one array: calls that may overlap on
 *     the GPU (different streams without ordering) race and must not be issued.
 *   - A device-side wait that runs out (bounded as in the context path) sets
 *     a sticky error word beside the array; kd_attn_noalloc_status reads it. */
#define KD_ATTN_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
kd_attn_status kd_attn_flash_ext_noalloc(const kd_tensor* q, const kd_tensor* k, const kd_tensor* v,
                                         const kd_tensor* mask, float scale, float max_bias,
                                         float logit_softcap, const int32_t* kv_len,
                                         const uint8_t* tile_mask, kd_tensor* out, float* lse,
                                         void* stream);

/* The allocation-free path's kd_attn_device_status (no reference counterpart):
 * synchronises `stream`, then reads and clears the current device's sticky
 * error word of kd_attn_flash_ext_noalloc.  KD_ATTN_ERR_DEVICE_TIMEOUT means a
 * call since the last check gave up on a wait and its output is incomplete. */
kd_attn_status kd_attn_noalloc_status(void* stream);

/* Failure-detection self-test of the allocation-free path (no reference
 * counterpart): one bounded device wait that nothing releases, on the current
 * device, reporting through the same error word; after wait_ms (1..10000) it
 * gives up, and the next kd_attn_noalloc_status returns
 * KD_ATTN_ERR_DEVICE_TIMEOUT.  Nothing faults, traps or spins without a bound. */
kd_attn_status kd_attn_noalloc_selftest_wait(uint32_t wait_ms, void* stream);

/* ---------------------------------------------------------------------------
 * The two CrossDiT call sites end to end (prologue + flash), operands staged
 * in the context's scratch.
 * Self-attention: DiTSelfAttention::forward between the QKV Linears and the
 *   out-projection (crossdit.hpp:132-150 + ops.hpp:107-206).
 * Cross-attention: DiTCrossAttention::forward (crossdit.hpp:186-198 +
 *   ops.hpp:107-206), no RoPE, optional mask / kv_len.
 * q_in, k_in, v_in : [C = n_head*d, L, N] f32, head dim d = 128 or 64 (as ops::attention
 *                    derives it, q.ne[0] / n_head, ops.hpp:116); rope axes sum to d
 * op_type          : operand type, KD_ATTN_TYPE_F16 (ggml semantics) or BF16
 * out              : [C, Lq, N] f32 | bf16 */
/* ops::attention's flash branch as it stands (ops.hpp:107-185,204-206), for
 * callers that apply no RMSNorm / RoPE first: q_in [n_head*d, Lq, N], k_in and
 * v_in [n_kv_head*d, Lk, N] (f32, d = 128 or 64, n_head % n_kv_head == 0: the GQA
 * expansion of ops.hpp:135-157 is done by indexing, not by copies); Q, K and V are
 * permuted and rounded to op_type (ops.hpp:122-131,167-169, f16 in ggml), then flash
 * attention with scale 1/sqrt(d).  mask: NULL or f16 in ggml's flash orientation
 * [>=Lk, >=Lq, mh, mn] (ops.hpp:171-174 transposes an [N, Lq, Lk] mask first; that
 * branch is never reached by the CrossDiT call sites).  out [n_head*d, Lq, N].
 * n_head = 1 with 512 channels (packed rows, no mask) is the VAE mid-block call (vae.hpp:89):
 * head_dim 512, scale 1/sqrt(512). */
kd_attn_status kd_attn_attention(kd_attn_ctx* ctx, const kd_tensor* q_in, const kd_tensor* k_in,
                                 const kd_tensor* v_in, int32_t n_head, const kd_tensor* mask,
                                 int32_t op_type, kd_tensor* out, float* lse, void* stream);

kd_attn_status kd_attn_self_attention(kd_attn_ctx* ctx, const kd_tensor* q_in, const kd_tensor* k_in,
                                      const kd_tensor* v_in, int32_t n_head, const float* q_gain,
                                      const float* k_gain, float eps, const kd_rope3d* rope,
                                      int32_t op_type, kd_tensor* out, float* lse, void* stream);

/* Self-attention on HOST buffers: the executor's upload -> graph compute ->
 * download sequence (src/core/executor.hpp:235, :241, :253) for this one op,
 * pipelined by head groups.  The heads are split into >= 4 equal groups; the
 * host->device copy of group g+1 and the device->host copy of group g-1 run on
 * two context-owned copy streams while group g computes on `stream`.  When
 * `stream` has drained, `out` holds the result (the caller's stream waits on
 * the last device->host copy).  Host buffers should be page-locked
 * (cudaMallocHost / cudaHostRegister); pageable memory is correct but does not
 * overlap.  Arguments as kd_attn_self_attention, with q_in/k_in/v_in/out in host
 * memory (f32 inputs; out f32 or op_type), rows of each sequence evenly spaced
 * or not, no lse.  Results are bit-identical to kd_attn_self_attention. */
kd_attn_status kd_attn_self_attention_host(kd_attn_ctx* ctx, const kd_tensor* q_in, const kd_tensor* k_in,
                                           const kd_tensor* v_in, int32_t n_head, const float* q_gain,
                                           const float* k_gain, float eps, const kd_rope3d* rope,
                                           int32_t op_type, kd_tensor* out, void* stream);

kd_attn_status kd_attn_cross_attention(kd_attn_ctx* ctx, const kd_tensor* q_in, const kd_tensor* k_in,
                                       const kd_tensor* v_in, int32_t n_head, const float* q_gain,
                                       const float* k_gain, float eps, const kd_tensor* mask,
                                       const int32_t* kv_len, int32_t op_type, kd_tensor* out,
                                       float* lse, void* stream);

/* ---------------------------------------------------------------------------
 * Head sharding.  No reference counterpart (the reference runs on device 0
 * only, src/pipeline.cpp:214).  Rank r of n owns heads [r*H/n, (r+1)*H/n) and
 * produces shard = [D, H/n, Lq, N]; this gathers every rank's shard into
 * full = [D, H, Lq, N] (= [C, Lq, N]) ahead of the out-projection
 * (crossdit.hpp:153) with one ncclAllGather into scratch plus a permute. */
kd_attn_status kd_attn_allgather_heads(kd_attn_ctx* ctx, const kd_tensor* shard, kd_tensor* full,
                                       void* stream);

/* Symmetric buffers for the fused head exchange.  Collective over the
 * context's group: every rank calls it with the same size, in the same order.
 * Each rank gets `bytes` of its own device memory (*out) and maps every other
 * rank's copy (CUDA IPC over NVLink); a kernel can then store into all copies.
 * kd_attn_symmetric_free is collective too (it waits for every rank, on
 * `stream`, before unmapping); kd_attn_destroy releases what is left. */
kd_attn_status kd_attn_symmetric_alloc(kd_attn_ctx* ctx, size_t bytes, void** out);
kd_attn_status kd_attn_symmetric_free(kd_attn_ctx* ctx, void* ptr, void* stream);

/* Head-sharded self-attention with the all-gather fused into the flash
 * kernel: the reference runs the whole of DiTSelfAttention::forward's
 * attention (crossdit.hpp:132-150) on one device; here rank r of n computes
 * heads [r*n_head_local, (r+1)*n_head_local) from its column shard of the
 * projections (q_in, k_in, v_in: [n_head_local*d, L, N] f32, d = 128 or 64) and its
 * flash-kernel epilogue stores every output row both into its own copy of
 * out_full and, over NVLink, into every other rank's copy, at the rank's
 * columns, so the exchange overlaps the attention math instead of following it.
 * out_full: [n_head_local*n_ranks*d, L, N] (f32 or op_type) inside a
 * kd_attn_symmetric_alloc buffer, at the same offset on every rank.
 * Collective: two barriers on the communicator, one before the kernels (no rank
 * still reads the previous contents of its copy) and one after (every row has
 * landed in every copy).  When `stream` has drained, each rank's out_full holds
 * all heads -- the input of the out-projection (crossdit.hpp:153).  With one
 * rank this is kd_attn_self_attention into out_full. */
kd_attn_status kd_attn_self_attention_sharded(kd_attn_ctx* ctx, const kd_tensor* q_in, const kd_tensor* k_in,
                                              const kd_tensor* v_in, int32_t n_head_local, const float* q_gain,
                                              const float* k_gain, float eps, const kd_rope3d* rope,
                                              int32_t op_type, kd_tensor* out_full, void* stream);

/* DiTSelfAttention::forward (crossdit.hpp:117-154) with heads sharded over the group: rank r passes the
 * replicated hidden states x [C, L, N] f32, ITS column shard of the Q/K/V weights (wq/wk/wv: [C, C_local],
 * the output features of heads [r*n_head_local, (r+1)*n_head_local), C_local a multiple of 256) and the
 * full out_layer weight wo [n_ranks*C_local, C_out]; n_head_local = C_local / d.  The projection and
 * attention of its heads run locally, the flash epilogue stores its heads into every rank's attn_full (bf16
 * [n_ranks*C_local, L, N], contiguous, inside a kd_attn_symmetric_alloc buffer), and after the closing
 * barrier out_layer runs on the gathered output: y [C_out, L, N] on every rank.  When y is contiguous
 * and inside a kd_attn_symmetric_alloc buffer, rank r computes token rows [r*M/n, (r+1)*M/n) of y
 * (M = L*N) and copies them into every other rank's y (a third barrier closes the call); otherwise
 * every rank computes all rows.  Collective (two or three barriers on the communicator). */
kd_attn_status kd_attn_self_attention_block_sharded(kd_attn_ctx* ctx, const kd_tensor* x, const kd_linear* wq,
                                                    const kd_linear* wk, const kd_linear* wv, const kd_linear* wo,
                                                    int32_t n_head_local, const float* q_gain, const float* k_gain,
                                                    float eps, const kd_rope3d* rope, kd_tensor* attn_full,
                                                    kd_tensor* y, void* stream);

/* The same for DiTCrossAttention::forward (crossdit.hpp:186-198): this rank's heads of the
 * visual queries against the text keys/values (column shards of k_in/v_in), no RoPE, the
 * optional mask / kv_len of kd_attn_cross_attention, every row exchanged in the flash epilogue. */
kd_attn_status kd_attn_cross_attention_sharded(kd_attn_ctx* ctx, const kd_tensor* q_in, const kd_tensor* k_in,
                                               const kd_tensor* v_in, int32_t n_head_local, const float* q_gain,
                                               const float* k_gain, float eps, const kd_tensor* mask,
                                               const int32_t* kv_len, int32_t op_type, kd_tensor* out_full,
                                               void* stream);

/* ---------------------------------------------------------------------------
 * Seeded N(0,1) fill on the device: Philox4x32-10 + Box-Muller with the
 * counter layout of PhiloxRNG::randn (src/rng.hpp:51-69): element i of a call
 * at counter offset `offset` uses counter (offset, 0, i, 0) and key = seed.
 * dst: device f32 [n].  Used to build the synthetic benchmark inputs. */
kd_attn_status kd_attn_fill_randn(kd_attn_ctx* ctx, float* dst, uint64_t n, uint64_t seed,
                                  uint32_t offset, void* stream);

/* Library version as (major << 16) | minor. */
int32_t kd_attn_version(void);

#ifdef __cplusplus
}
#endif

#endif /* KD_ATTN_H */
