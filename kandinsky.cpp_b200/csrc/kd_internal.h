// kd_internal.h -- declarations shared between the host API (kd_api.cu) and
// the kernel translation units.  Not part of the public ABI.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace kd {

// Tile classes of the additive mask, per 64 x 64 (query x key) tile.
enum : uint8_t { kTileSkip = 0, kTileFull = 1, kTileMixed = 2 };

// Flash-attention forward geometry (sm_100a kernel in kd_fmha.cu).
constexpr int kHeadDim = 128;
constexpr int kHeadDim64 = 64;    // the lite video model's head (axes 16 + 24 + 24): kd_fmha.cu at D = 64
constexpr int kHeadDim512 = 512;  // the VAE mid-block head (kd_fmha512.cu)
constexpr int kBlockM = 128;   // query rows per Q tile = one M=128 tcgen05 MMA
constexpr int kQTiles = 2;     // Q tiles per CTA, one softmax warpgroup each
constexpr int kRowsPerCta = kBlockM * kQTiles;
constexpr int kBlockN = 128;   // keys per K/V tile
constexpr int kMaxKvTiles = 2048;  // per-unit kept-tile list capacity (Lk <= 262144)
constexpr int kMaxPeers = 7;       // other ranks an output row is also written to (8 GPUs)
// Unmasked calls with at most this many keys (padded length) run the short-key instantiation:
// double-buffered Q, units published two ahead, Q loads issued by the scheduler warp, and (16-bit
// outputs, no peer exchange) the O tiles written with TMA stores from shared memory.
#ifndef KD_FMHA_Q2_MAX_KEYS
#define KD_FMHA_Q2_MAX_KEYS 1024
#endif
constexpr int kQ2MaxKeys = KD_FMHA_Q2_MAX_KEYS;

struct FmhaParams {
    int D;                   // head dim: 128, or 64 (the lite models' heads)
    int Lq, Lk, H, N;        // query rows, keys, heads, sequences
    int rk2, rk3;            // H / Hkv, N / Nkv (ggml broadcast ratios)
    float scale_log2;        // scale * log2(e)
    float inv_scale;         // 1 / scale (mask values are folded into raw scores)
    void* out;               // [D, H, Lq, N]
    long long o_nb1, o_nb2, o_nb3;  // byte strides of out (head, row, sequence)
    float* lse;              // [N, H, Lq] or null
    const uint8_t* tile_cls; // [mn][mh][n_qb][n_kb] or null
    int n_qb, n_kb;
    const uint16_t* mask;    // f16 bits [.., Lk] rows, or null
    long long m_nb1, m_nb2, m_nb3;
    int mh, mn;
    const int32_t* kv_len;   // [N] or null
    unsigned* err;           // sticky device error word
    unsigned* abort_flag;    // per-launch abort flag (cleared by the host before each launch)
    unsigned* work_counter;  // next unit to hand out (cleared by the host before each launch)
    int num_ctas;            // persistent grid size (number of SMs)
    unsigned long long wait_ns;
    unsigned long long* tile_stats;  // [2] or null: K/V tiles loaded, (Q tile, K/V tile) pairs computed
    // Head-sharded output exchange: every output row is also stored at the same byte offset from
    // each of these bases (other GPUs' copies of the output, mapped into this process).
    char* peer_out[kMaxPeers];
    int n_peer_out;
    int out_v8;              // 1: out rows are 32-byte aligned (256-bit stores in the epilogue)
    int head_pairs;          // masked kernel: units of 128 rows x heads (2hp, 2hp+1) -- needs one mask
                             // plane for all heads (mh == 1), an even head count and no peers
    int tma_out;             // short-key kernel: tmO describes `out` (16-bit, no peers); O tiles go out by TMA
};

enum class OpType { F16, BF16 };
enum class OutType { F32, F16, BF16 };

// Launches the tcgen05 flash-attention forward.  tmQ/tmK/tmV are 4-D tiled
// tensor maps over [D, L, heads, seqs] with a {64, 128, 1, 1} box and
// 128-byte swizzle; tmO (read only when p.tma_out) maps `out` as [D, H, Lq, N]
// with a {64, 1, 128, 1} box (the same 128 rows of 128 bytes in shared memory) and swizzle.
cudaError_t launch_fmha(OpType op, OutType ot, const CUtensorMap& tmQ, const CUtensorMap& tmK,
                        const CUtensorMap& tmV, const CUtensorMap& tmO, const FmhaParams& p, cudaStream_t st);
int fmha_smem_bytes();
// head_dim 512, no mask (kd_fmha512.cu): tmQ over [512, Lq, H, N] with a {64, 128, 1, 1} box,
// tmK/tmV over [512, Lk, Hkv, Nkv] with a {64, 64, 1, 1} box, all 128-byte swizzled.
cudaError_t launch_fmha512(OpType op, OutType ot, const CUtensorMap& tmQ, const CUtensorMap& tmK,
                           const CUtensorMap& tmV, const FmhaParams& p, cudaStream_t st);

// ---------------------------------------------------------------- prologue
struct RopeTab {
    float freq[64];          // per rotary pair (D/2 of them): theta^(-i/half_axis), computed like rope.hpp:23-29
    float div[64];           // scale_factor of the pair's axis
    unsigned char axis[64];  // 0 = t, 1 = h, 2 = w
    int grid_h, grid_w;      // token -> (t,h,w): t = l/(gh*gw), h = (l/gw)%gh, w = l%gw
};

// One projection handled by the prologue: x [C = H*D, L, N] f32 -> y [D, L, H, N].
struct PrologueJob {
    const float* x;          // dim 0 contiguous
    long long x_nb1, x_nb2;  // byte strides of x (token, sequence)
    void* y;
    long long y_nb1, y_nb2, y_nb3;  // byte strides of y (row, head, sequence)
    const float* gain;       // [D] or null (unit gain); used when norm
    int norm;                // 1: RMSNorm
    int rope;                // 1: apply RoPE with the shared table
    int L, N, H;
};

// Up to three projections in one launch (blockIdx.y = projection).
constexpr int kPrologueMaxJobs = 3;
constexpr int kPrologueHeads = 8;  // heads per warp item (8 row loads in flight per lane)
struct PrologueParams {
    PrologueJob job[kPrologueMaxJobs];
    int njobs;
    int D;                   // head dim of every job: 128, or 64 (two heads per 128-element warp row)
    float eps;
    RopeTab tab;             // shared by every projection with rope = 1
};
cudaError_t launch_prologue(OutType yt, const PrologueParams& p, int num_sms, cudaStream_t st);

// Rounds a strided [D, L, H, N] f32/f16/bf16 tensor to the operand type, contiguous.
struct ConvertParams {
    const void* src; int src_type;   // kd_attn_type id
    long long nb1, nb2, nb3;
    void* dst;                       // contiguous [D, L, H, N]
    int L, H, N;
    int D;                           // row width: 64, 128 or 512
};
cudaError_t launch_convert_q(OpType dt, const ConvertParams& p, int num_sms, cudaStream_t st);

// Classifies each 64x64 tile of an f16 additive mask as skip / full / mixed.
// With a tile bitmap, tiles whose bit is clear are skip without reading the
// mask; without a mask, set bits are full tiles.
struct MaskClassParams {
    const uint16_t* mask;            // or null (bitmap only, one plane)
    const uint8_t* bits;             // or null: bit kb of row qb (rows of bits_row_bytes bytes)
    int bits_row_bytes;
    int vec16;                       // 1: mask base and row stride are 16-byte aligned (vector loads)
    long long nb1, nb2, nb3;         // byte strides (query row, head plane, sequence plane)
    int Lq, Lk, mh, mn;
    uint8_t* cls;                    // [mn][mh][n_qb][n_kb]
    int n_qb, n_kb;
};
cudaError_t launch_mask_classify(const MaskClassParams& p, cudaStream_t st);

// ---------------------------------------------------------------- QKV projection (kd_gemm.cu)
// One projection of the fused GEMM: C output features = C/D heads, written as [D, L, H, N].
struct QkvSlot {
    void* out;
    long long o_nb1, o_nb2, o_nb3;  // byte strides of out (row, head, sequence)
    const float* bias;              // [C] or null
    const float* gain;              // [128] or null (unit gain); read when norm
    int norm;                       // 1: RMSNorm per head
    int rope;                       // 1: rotate with QkvParams::rope_cs
};
struct QkvParams {
    QkvSlot slot[3];
    int D;                   // head dim of the normalised/rotated slots: 128, or 64 (a warpgroup's 64 columns
                             // are one whole head: no exchange of RMSNorm sums); 128 for plain linears
    int nslots;              // projections concatenated along the B operand's rows (slot s = rows [s*C, (s+1)*C))
    int C;                   // output features per projection, a multiple of 256
    int K;                   // input features
    int M;                   // tokens = L * N
    int L;                   // tokens per sequence (token m is l = m % L of sequence n = m / L)
    float eps;
    const float2* rope_cs;   // [L][D/2] (cos, sin) or null
    unsigned* err;
    unsigned* abort_flag;
    unsigned long long wait_ns;
};
// Rows of one TMA box of each GEMM operand: each CTA of a pair stages 128 token rows of A and 128 feature
// rows of B per K step (the kernel's shared-memory slots are sized from these).
constexpr int kGemmBoxRowsA = 128;
constexpr int kGemmBoxRowsB = 128;
// K per stage, and the 64-wide K slices one TMA copy brings; the operands' rows are zero-padded to a
// multiple of kGemmKChunk (Kp).
constexpr int kGemmBoxChunks = 2;
constexpr int kGemmKChunk = 64 * kGemmBoxChunks;
// tmX: bf16 [Kp, M] viewed as {64, M, Kp/64} with a {64, kGemmBoxRowsA, kGemmBoxChunks} box; tmW: bf16
// [Kp, nslots*C] viewed as {64, nslots*C, Kp/64} with a {64, kGemmBoxRowsB, kGemmBoxChunks} box; both
// 128-byte swizzled.
cudaError_t launch_qkv_gemm(OutType ot, const CUtensorMap& tmX, const CUtensorMap& tmW, const QkvParams& p, int num_sms,
                            cudaStream_t st);
// ggml weight rows [rows][row_bytes] of type f32 (0), f16 (1), q4_0 (2), q8_0 (8), bf16 (30) -> bf16 rows
// row0 .. row0+rows-1 of dst [*, Kp], columns K .. Kp-1 zero; K and Kp multiples of 32.
cudaError_t launch_expand_weights(const void* w, int type, long long row_bytes, int K, int Kp, int rows, int row0,
                                  __nv_bfloat16* dst, int num_sms, cudaStream_t st);
// f32 x [K, L, N] (byte strides nb1, nb2; K a multiple of 32, rows 16-byte aligned) -> bf16 [M = L*N][Kp],
// columns K .. Kp-1 zero.
cudaError_t launch_to_bf16_rows(const void* x, long long nb1, long long nb2, int K, int Kp, int L, long long M,
                                __nv_bfloat16* dst, int num_sms, cudaStream_t st);
// (cos, sin) of every token and rotary pair of the 3D RoPE table: cs[l * pairs + i], pairs = D/2.
cudaError_t launch_rope_table(const RopeTab& tab, int L, int pairs, float2* cs, int num_sms, cudaStream_t st);

// One bounded wait that nothing releases (sets the self-test error bit after wait_ns).
cudaError_t launch_wait_selftest(unsigned* err, unsigned* abort_flag, unsigned long long wait_ns, cudaStream_t st);

cudaError_t launch_randn(float* dst, unsigned long long n, unsigned long long seed, unsigned offset, int num_sms,
                         cudaStream_t st);

// Rank-major gathered shards [R][N*Lq][Hs*128] -> [N*Lq][R*Hs*128] (elt bytes 2 or 4).
cudaError_t launch_unshard_heads(const void* src, void* dst, long long rows, int ranks, long long shard_row_bytes,
                                 int num_sms, cudaStream_t st);

}  // namespace kd
