/*
 * kd_oracle.h -- CPU restatement of kandinsky.cpp's CrossDiT attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library (libkd_attn) links,
 * loads or calls this code; it is the checker that the tests, the smoke entry
 * and the bench's CPU-baseline leg compare the CUDA path against.
 *
 * What it restates (reference = AkaneTendo25/kandinsky.cpp):
 *   - PhiloxRNG::randn              src/rng.hpp:42-131  (Philox4x32-10 + Box-Muller)
 *   - rope::get_freqs               src/rope.hpp:23-29
 *   - rope::compute_text_rope       src/rope.hpp:36-49
 *   - rope::compute_visual_rope     src/rope.hpp:56-102
 *   - rope::apply                   src/rope.hpp:109-155
 *   - RMSNorm::forward / ops::rms_norm  src/core/module.hpp:163-180, src/core/ops.hpp:76-81
 *   - ops::attention (flash branch) src/core/ops.hpp:107-185,204-206
 *   - ggml_flash_attn_ext (CPU), called at src/core/ops.hpp:176.  ggml is an
 *     external, un-vendored, unpinned dependency (CMakeLists.txt:8-15,43;
 *     README.md:17-20) that is absent from this machine, so its published CPU
 *     algorithm (online-softmax flash attention, Rabe & Staats 2021, with the
 *     f16 value accumulator of ggml-cpu's one-chunk kernel) is restated here.
 *
 * Parity status: the RoPE tables and the Philox generator are pinned to the
 * reference's own source (compiled from its headers by oracle/ref_pin, golden
 * vectors under tests/golden).  flash_attn_ext itself is UNPINNED: no ggml
 * build and no ggml golden vectors exist here.
 */
#ifndef KD_ORACLE_H
#define KD_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (ggml.h: GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1, GGML_TYPE_BF16 = 30) */
enum { KDO_F32 = 0, KDO_F16 = 1, KDO_BF16 = 30 };

/* ggml-style tensor view: ne = sizes, nb = byte strides, dim 0 fastest. */
typedef struct {
    const void* data;
    int32_t type;
    int64_t ne[4];
    int64_t nb[4];
} kdo_tensor;

enum { KDO_MODE_EXACT = 0, KDO_MODE_GGML = 1 };

/* ---- scalar conversions (round to nearest even) ---- */
uint16_t kdo_f32_to_f16(float f);
float kdo_f16_to_f32(uint16_t h);
uint16_t kdo_f32_to_bf16(float f);
float kdo_bf16_to_f32(uint16_t h);
void kdo_convert(const float* src, int64_t n, int32_t dst_type, void* dst);
void kdo_to_f32(const void* src, int32_t src_type, int64_t n, float* dst);

/* ---- seeded inputs: src/rng.hpp:51-69 (one randn(n) call at counter offset) ---- */
void kdo_philox_randn(uint64_t seed, uint32_t offset, uint64_t n, float* out, int nthreads);

/* ---- RoPE tables ---- */
void kdo_rope_freqs(int dim, float theta, float* out);
void kdo_text_rope_table(int seq_len, int head_dim, float theta, float* out);
void kdo_visual_rope_table(int n_frames, int height, int width, const int axes_dims[3],
                           const float scale_factor[3], float theta, float* out);

/* ---- prologue pieces on [C = n_head*head_dim, L, N] f32 activations ---- */
void kdo_rms_norm_heads(const float* x, int64_t n_rows, int head_dim, const float* gain, float eps,
                        float* y, int nthreads);
void kdo_rope_apply(float* x, int64_t n_tokens, int64_t n_seq, int n_head, int head_dim,
                    const float* table, int nthreads);

/* ---- ggml_flash_attn_ext restatement ----
 * q: [DK, Lq, H, N]; k: [DK, Lk, Hkv, Nkv]; v: [DV, Lk, Hkv, Nkv];
 * mask (nullable): f16 [>=Lk, >=Lq, mh, mn] broadcast over heads/sequences;
 * kv_len (nullable): per-sequence valid key count (keys >= kv_len[n] are masked);
 * out: f32 [DV, H, Lq, N] contiguous (the ggml dst permutation);
 * lse (nullable): f32 [N, H, Lq], natural log of sum_j exp(scale*q.k_j + mask_j), fp64.
 * Returns 0 on success, negative on a shape error. */
int kdo_flash_attn_ext(const kdo_tensor* q, const kdo_tensor* k, const kdo_tensor* v,
                       const kdo_tensor* mask, float scale, const int32_t* kv_len, int mode,
                       float* out, float* lse, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
