// kd_gemm.cu -- the QKV projection of DiTSelfAttention::forward with the attention prologue fused
// into its epilogue, on sm_100a (B200).
//
// The reference computes q, k, v = Linear(x) (src/models/crossdit.hpp:123-125: ggml_mul_mat on
// q4_0 / q8_0 / f16 weights plus a bias, ops::linear), writes them as f32 [C, L, N], then the
// graph reads them back for the per-head RMSNorm (crossdit.hpp:135-136), rope::apply (:140-141)
// and the permute + cast to the flash operands (ops.hpp:122-131,167-169).  Here one GEMM produces
// the three projections and its epilogue applies bias, RMSNorm, RoPE and the cast and stores the
// flash-attention operands [128, L, H, N] directly: the f32 projections never reach HBM.
//
//   expand_weights_kernel  ggml weight [C_in, C_out] (q8_0: 34-byte blocks of an f16 scale and 32
//                          int8, value d*q; q4_0: 18-byte blocks of an f16 scale and 16 bytes,
//                          element j in the low nibble and j+16 in the high one, value d*(q-8) --
//                          the layout scripts/convert_to_gguf.py:90-146 writes; f16 / bf16 / f32)
//                          -> bf16 rows of the concatenated [Kp, 3*C_out] B operand (Kp: C_in rounded
//                          up to the 128-wide K step, zero-padded)
//   to_bf16_rows_kernel    x f32 [C_in, L, N] -> bf16 [Kp, L*N] (the A operand, token rows)
//   rope_table_kernel      cos/sin of every (token, rotary pair), the prologue's angle formula
//   qkv_gemm_kernel        persistent tcgen05 GEMM on CTA pairs, 256 tokens x 256 output features
//                          per tile (two heads of one projection), K in steps of 128 through a
//                          3-stage TMA ring, fp32 accumulators double-buffered in TMEM so one tile's
//                          epilogue (16 warps) overlaps the next tile's MMAs
//
// Every wait is bounded (kd_common.cuh: mbar_wait).
#include "kd_common.cuh"
#include "kd_internal.h"

namespace kd {
namespace {

// Tiles of 256 tokens x 256 output features are computed by a CTA pair (a cluster of 2 on neighbouring
// SMs) with tcgen05.mma.cta_group::2: each CTA stages its 128 token rows of A and its 128 feature rows of B,
// the MMA (M = 256, N = 256, issued by the pair's rank-0 CTA) reads both CTAs' halves, and each CTA's TMEM
// receives the 128 x 256 accumulator of its own token rows.  Per SM that is 16 KB of A and 16 KB of B per
// 64-wide K step -- two thirds of the shared-memory traffic of a one-CTA 128 x 256 tile, whose TMA writes
// plus MMA operand reads exceed the SM's shared-memory bandwidth (measured: tensor pipe 56 % active).
constexpr int kBM = kGemmBoxRowsA;       // token rows per CTA (the pair covers 256)
constexpr int kPairM = 2 * kBM;
constexpr int kBN = 256;                 // output features per tile (MMA N): two heads
constexpr int kHalfN = kGemmBoxRowsB;    // B rows staged by each CTA
static_assert(kBM == 128 && 2 * kHalfN == kBN, "pair tile geometry");
// K per stage: kGemmBoxChunks 64-wide slices (one 128-byte swizzled row each), brought by ONE 3-D TMA copy
// per operand.  Measured with the MMAs switched off, a CTA pair streams its operands at the same rate with
// 18, 37 or 74 pairs running -- a per-SM limit, not L2's -- and 16 KB copies delivered ~37 B/clk per SM;
// fewer, larger copies move more bytes per SM.
constexpr int kBK = kGemmKChunk;
constexpr int kABytes = kBM * kBK * 2;     // 32 KB
constexpr int kBBytes = kHalfN * kBK * 2;  // 32 KB
constexpr int kSubBytes = kBM * 64 * 2;    // one 64-wide K slice of 128 rows: 16 KB
static_assert(kBM == kHalfN && kBK == 64 * kGemmBoxChunks, "stage geometry");
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kGStages = 3;
constexpr int kGSmemBar = kGStages * kStageBytes;
// full[S], empty[S], acc_full[2], acc_empty[2], exch[2 tile parities][2 heads]
constexpr int kGNumBars = 2 * kGStages + 8;
constexpr int kGSmemSlot = kGSmemBar + kGNumBars * 8;
// RMSNorm partial sums exchanged between the two warpgroups of a head: [tile parity][warpgroup][row] float2
constexpr int kGSmemPart = kGSmemSlot + 16;
constexpr int kGSmemAlloc = kGSmemPart + 2 * 4 * 128 * 8 + 1024;
static_assert(kGSmemAlloc <= 232448, "shared memory budget");
// Warps 0-15: epilogue, four warpgroups, warpgroup g on head (g >> 1) of the tile, columns 64 * (g & 1) ..
// +63 (a warp reads the TMEM lanes of its index mod 4, i.e. 32 token rows); warp 16: TMA producer; warp 17:
// TMEM allocation and (rank 0) MMA issue.  Sixteen epilogue warps, four per SM sub-partition, hide the
// latency of the TMEM, RoPE-table and store traffic that one warp per sub-partition left exposed: measured,
// that epilogue took ~71K cycles per tile against ~33K of MMA.
constexpr int kEpiWarps = 16;
constexpr int kWarpProducer = 16;
constexpr int kWarpMma = 17;
constexpr int kGThreads = 32 * (kEpiWarps + 2);
constexpr int kGroupM = 8;  // 256-row m-tiles per raster band: the pairs in flight share 8 A blocks and ~9 B blocks

// Tile t of the persistent loop -> (m-tile, n-tile).  Bands of kGroupM m-tiles are swept n-tile by n-tile,
// m fastest, so the pairs running at one time read a few MB of A and B that stay in L2.
__device__ __forceinline__ void tile_coords(long long t, int m_tiles, int n_tiles_n, int& mt, int& nt) {
    const long long band = t / ((long long)kGroupM * n_tiles_n);
    const int first = (int)band * kGroupM;
    const int gm = min(kGroupM, m_tiles - first);
    const int within = (int)(t - band * kGroupM * n_tiles_n);
    mt = first + within % gm;
    nt = within / gm;
}

// ------------------------------------------------------------------ CTA-pair primitives
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// The shared::cluster address of the variable at shared::cta address `saddr` in the pair's CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Tile load into this CTA's shared memory whose completion is counted on an mbarrier of either CTA of
// the pair (here always rank 0's): .cta_group::2, no multicast.  The maps are 3-D, {64, rows, K / 64}: one
// copy brings kGemmBoxChunks 64-wide K slices of its rows, slice j at j * kSubBytes.
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster, int c1,
                                                 int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(0), "r"(c1), "r"(c2)
        : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem of both CTAs] (+)= A[smem of both CTAs] * B[smem of both CTAs], issued by one lane of rank 0.
__device__ __forceinline__ void mma_pair_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive once on the mbarrier at the same offset in both CTAs when the pair's MMAs issued so far complete.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}\n" ::"r"(
            smem_u32(bar)),
        "h"((unsigned short)0x3)
        : "memory");
}

// (hi, lo) += v with hi + lo kept exact to ~2^-48 relative: TwoSum of hi and v, its error added to lo.
__device__ __forceinline__ void two_sum_acc(float& hi, float& lo, float v) {
    const float s = __fadd_rn(hi, v);
    const float bv = __fsub_rn(s, hi);
    const float err = __fadd_rn(__fsub_rn(hi, __fsub_rn(s, bv)), __fsub_rn(v, bv));
    hi = s;
    lo = __fadd_rn(lo, err);
}

template <typename TO>
__device__ __forceinline__ void store_chunk(TO* dst, const float* v) {  // 32 values, 64 bytes
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i)
        d[i] = make_uint4(Pack2<TO>::pack(v[8 * i], v[8 * i + 1]), Pack2<TO>::pack(v[8 * i + 2], v[8 * i + 3]),
                          Pack2<TO>::pack(v[8 * i + 4], v[8 * i + 5]), Pack2<TO>::pack(v[8 * i + 6], v[8 * i + 7]));
}
template <>
__device__ __forceinline__ void store_chunk<float>(float* dst, const float* v) {  // 32 values, 128 bytes
    float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int i = 0; i < 8; ++i) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

// Launched as clusters of 2 (blockIdx.x = 2 * pair + rank); both CTAs run the producer and the epilogue
// warps, rank 0 also issues the MMAs.
template <typename TO, int kD>
__global__ void __launch_bounds__(kGThreads, 1)
    qkv_gemm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                    const __grid_constant__ QkvParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const long long pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const DevCtl ctl{p.err, p.abort_flag, p.wait_ns};
    const int n_tiles_n = p.nslots * p.C / kBN;
    const int m_tiles = (p.M + kPairM - 1) / kPairM;
    const long long n_tiles = (long long)m_tiles * n_tiles_n;
    const int k_steps = (p.K + kBK - 1) / kBK;  // the operands' rows are zero-padded to k_steps * kBK

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kGSmemBar);
    uint64_t* full = bars;              // rank 0's count both CTAs' bytes of a stage
    uint64_t* empty = bars + kGStages;  // each CTA's: its stage may be refilled
    uint64_t* acc_full = bars + 2 * kGStages;
    uint64_t* acc_empty = acc_full + 2;  // rank 0's: both CTAs' epilogues have read the accumulator
    uint64_t* exch = acc_empty + 2;      // the two warpgroups of a head have posted their RMSNorm partial sums
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kGSmemSlot);
    if (threadIdx.x == 0) {
        for (int s = 0; s < kGStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 2 * 32 * kEpiWarps);
        }
        for (int i = 0; i < 4; ++i) mbar_init(&exch[i], 256);
        fence_mbar_init();
    }
    if (warp == kWarpMma) {
        tmem_alloc_pair(tmem_slot, 512);
        tmem_relinquish_pair();
    }
    // both CTAs' barriers exist before either CTA's copies or MMAs can signal them
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t full0 = map_to_rank(smem_u32(full), 0);
    const uint32_t acc_empty0 = map_to_rank(smem_u32(acc_empty), 0);

    if (warp == kWarpProducer) {
        // ------------------------------------------------------------ TMA producer (both CTAs)
        if (lane == 0) {
            tma_prefetch_desc(&tmX);
            tma_prefetch_desc(&tmW);
        }
        const uint32_t base = smem_u32(smem);
        uint32_t it = 0;
        bool ok = true;
        for (long long t = pair; t < n_tiles && ok; t += npairs) {
            int mt, nt;
            tile_coords(t, m_tiles, n_tiles_n, mt, nt);
            for (int kb = 0; kb < k_steps; ++kb) {
                const int s = it % kGStages;
                if (!(ok = __all_sync(0xffffffffu,
                                      mbar_wait(&empty[s], ((it / kGStages) & 1u) ^ 1u, ctl, kErrTimeoutKVEmpty))))
                    break;
                if (lane == 0) {
                    if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * kStageBytes);
                    const uint32_t st = base + s * kStageBytes;
                    tma_load_3d_pair(st, &tmX, full0 + 8u * s, mt * kPairM + (int)rank * kBM, kb * kGemmBoxChunks);
                    tma_load_3d_pair(st + kABytes, &tmW, full0 + 8u * s, nt * kBN + (int)rank * kHalfN,
                                     kb * kGemmBoxChunks);
                }
                __syncwarp();
                ++it;
            }
        }
        // Producer tail: the MMA's releases of the last stages arrive on this CTA's barriers from the pair's
        // commits; wait for them so that nothing is still addressed to this CTA when it leaves.
        if (ok)
            for (uint32_t k = (it > (uint32_t)kGStages ? it - kGStages : 0u); k < it; ++k)
                if (!__all_sync(0xffffffffu, mbar_wait(&empty[k % kGStages], (k / kGStages) & 1u, ctl, kErrTimeoutDrain)))
                    break;
    } else if (warp == kWarpMma && rank == 0) {
        // ------------------------------------------------------------ MMA issuer (rank 0 of the pair)
        constexpr uint32_t idesc = idesc_f16_f32acc(true, kPairM, kBN, false);
        constexpr uint32_t dhi = sw128_desc_hi(1024);
        const uint32_t base = smem_u32(smem);
        uint32_t it = 0, tc = 0;
        bool ok = true, issued = false;
        for (long long t = pair; t < n_tiles && ok; t += npairs, ++tc) {
            const uint32_t ab = tc & 1u;
            if (tc >= 2 &&
                !(ok = __all_sync(0xffffffffu, mbar_wait(&acc_empty[ab], ((tc >> 1) - 1) & 1u, ctl, kErrTimeoutO))))
                break;
            tc_fence_after();
            for (int kb = 0; kb < k_steps; ++kb) {
                const int s = it % kGStages;
                if (!(ok = __all_sync(0xffffffffu, mbar_wait(&full[s], (it / kGStages) & 1u, ctl, kErrTimeoutKVFull))))
                    break;
                ++it;
                tc_fence_after();
                const uint32_t alo = sw128_desc_lo(base + s * kStageBytes, 16);
                const uint32_t blo = sw128_desc_lo(base + s * kStageBytes + kABytes, 16);
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {
                    const uint32_t off = (uint32_t)((kk >> 2) * kSubBytes + (kk & 3) * 32) >> 4;
                    mma_pair_ss(tmem + ab * kBN, desc_join(alo + off, dhi), desc_join(blo + off, dhi), idesc,
                                (kb | kk) ? 1u : 0u);
                }
                tc_commit_pair(&empty[s]);
                issued = true;
            }
            if (ok) tc_commit_pair(&acc_full[ab]);
        }
        if (!ok && issued) {
            // gave up mid-way: a further arrival once every MMA issued so far has retired
            tc_commit_pair(&acc_full[tc & 1u]);
            mbar_wait(&acc_full[tc & 1u], (tc >> 1) & 1u, ctl, kErrTimeoutDrain, false);
        }
        // (otherwise both epilogues have waited for the last tile's accumulator, which retires every MMA)
    } else if (warp < kEpiWarps) {
        // ------------------------------------------------------------ epilogue: bias, RMSNorm, RoPE, cast
        const int r = ((warp & 3) << 5) + lane;  // token row of this CTA's 128
        const int wg = warp >> 2, hh = wg >> 1, half = wg & 1;
        const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
        float2* part = reinterpret_cast<float2*>(smem + kGSmemPart);
        uint32_t tc = 0;
        for (long long t = pair; t < n_tiles; t += npairs, ++tc) {
            const uint32_t ab = tc & 1u;
            int mt, nt;
            tile_coords(t, m_tiles, n_tiles_n, mt, nt);
            if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[ab], (tc >> 1) & 1u, ctl, kErrTimeoutO))) break;
            tc_fence_after();
            const long long m = (long long)mt * kPairM + (long long)rank * kBM + r;
            const bool valid = m < p.M;
            const int l = valid ? (int)(m % p.L) : 0, n = valid ? (int)(m / p.L) : 0;
            const int col0 = nt * kBN + hh * 128;
            const QkvSlot& S = p.slot[col0 / p.C];
            const int fcol = col0 % p.C + half * 64;        // this warpgroup's first feature of the slot
            const int h = fcol / kD, c0 = fcol % kD;        // its head and first column within the head
            // this thread's 64 accumulator columns, then the buffer is released at once: the MMAs of a later
            // tile may overwrite it while the values are processed from registers
            uint32_t xr[64];
            tmem_ld64_sync(tmem + lane_addr + ab * kBN + hh * 128 + half * 64, xr);
            tc_fence_before();
            mbar_arrive_remote(acc_empty0 + 8u * ab);
            float x[64];
#pragma unroll
            for (int d = 0; d < 64; ++d) x[d] = __uint_as_float(xr[d]);
            if (S.bias) {  // 16-byte aligned (checked by the host)
                const float4* b4 = reinterpret_cast<const float4*>(S.bias + fcol);
#pragma unroll
                for (int q = 0; q < 16; ++q) {
                    const float4 b = __ldg(b4 + q);
                    x[4 * q] = __fadd_rn(x[4 * q], b.x);
                    x[4 * q + 1] = __fadd_rn(x[4 * q + 1], b.y);
                    x[4 * q + 2] = __fadd_rn(x[4 * q + 2], b.z);
                    x[4 * q + 3] = __fadd_rn(x[4 * q + 3], b.w);
                }
            }
            // ggml's CPU rms_norm sums the float squares in double, rounds the mean to float and scales by
            // 1/sqrt(mean + eps).  FP64 arithmetic is slow on this part (measured ~350 cycles per element
            // here), so the sum is carried as an unevaluated float pair (Knuth's TwoSum, ~48 significant bits):
            // its rounding to float equals that of the double sum except within ~2^-48 of a rounding tie.
            // Each warpgroup sums its half of the row; the halves are swapped through shared memory on every
            // tile (so the exchange barriers' phases follow the tile count) and combined in a fixed order.  A
            // 64-wide head is one warpgroup's whole row and ignores the other half's sum; the exchange runs
            // all the same (without it this instantiation's epilogue spilled 812 bytes).
            float hi = 0.0f, lo = 0.0f;
#pragma unroll
            for (int d = 0; d < 64; ++d) two_sum_acc(hi, lo, __fmul_rn(x[d], x[d]));
            float2* pp = part + (size_t)(tc & 1u) * 4 * 128;
            pp[wg * 128 + r] = make_float2(hi, lo);
            uint64_t* xb = &exch[(tc & 1u) * 2 + hh];
            mbar_arrive(xb);
            if (!__all_sync(0xffffffffu, mbar_wait(xb, (tc >> 1) & 1u, ctl, kErrTimeoutO))) break;
            const float2 other = kD == 128 ? pp[(wg ^ 1) * 128 + r] : make_float2(0.0f, 0.0f);
            float scale = 1.0f;
            if (S.norm) {
                float thi = half == 0 ? hi : other.x, tlo = half == 0 ? lo : other.y;
                two_sum_acc(thi, tlo, half == 0 ? other.x : hi);  // (+0: the sum unchanged for 64-wide heads)
                tlo = __fadd_rn(tlo, half == 0 ? other.y : lo);
                // exact scaling by 2^-7 or 2^-6
                const float mean = __fmul_rn(__fadd_rn(thi, tlo), 1.0f / kD);
                scale = __frcp_rn(__fsqrt_rn(__fadd_rn(mean, p.eps)));
#pragma unroll
                for (int d = 0; d < 64; ++d) x[d] = __fmul_rn(x[d], scale);
                if (S.gain) {  // 16-byte aligned (checked by the host)
                    const float4* g4 = reinterpret_cast<const float4*>(S.gain + c0);
#pragma unroll
                    for (int q = 0; q < 16; ++q) {
                        const float4 g = __ldg(g4 + q);
                        x[4 * q] = __fmul_rn(x[4 * q], g.x);
                        x[4 * q + 1] = __fmul_rn(x[4 * q + 1], g.y);
                        x[4 * q + 2] = __fmul_rn(x[4 * q + 2], g.z);
                        x[4 * q + 3] = __fmul_rn(x[4 * q + 3], g.w);
                    }
                }
            }
            TO* dst = reinterpret_cast<TO*>(static_cast<char*>(S.out) + (long long)n * S.o_nb3 +
                                            (long long)h * S.o_nb2 + (long long)l * S.o_nb1) + c0;
            const float2* cs = S.rope ? p.rope_cs + (long long)l * (kD / 2) + c0 / 2 : nullptr;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                if (cs) {
                    // rope::apply (rope.hpp:140-141): (x0 c - x1 s, x0 s + x1 c), products rounded apart
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float2 a = __ldg(cs + c * 16 + i);  // (cos, sin)
                        const float x0 = x[c * 32 + 2 * i], x1 = x[c * 32 + 2 * i + 1];
                        x[c * 32 + 2 * i] = __fsub_rn(__fmul_rn(x0, a.x), __fmul_rn(x1, a.y));
                        x[c * 32 + 2 * i + 1] = __fadd_rn(__fmul_rn(x0, a.y), __fmul_rn(x1, a.x));
                    }
                }
                if (valid) store_chunk<TO>(dst + c * 32, x + c * 32);
            }
        }
    }

    // After a bounded wait gave up, copies this CTA issued may still be landing: give them time before the
    // pair's shared memory is released.  (Without an abort every copy was consumed by an MMA.)
    if (threadIdx.x == 0 && *reinterpret_cast<volatile unsigned*>(p.abort_flag)) {
        const unsigned long long t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 50000ull) {
        }
    }
    tc_fence_before();
    cluster_sync_all();  // no CTA leaves while its partner may still signal its barriers
    if (warp == kWarpMma) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 512);
    }
}

// One thread per 32-element block of one output-feature row: ggml weight -> bf16 row of B.
__global__ void expand_weights_kernel(const uint8_t* w, int type, long long row_bytes, int K, int Kp, int rows,
                                      int row0, __nv_bfloat16* dst) {
    const long long blocks_per_row = Kp / 32;  // blocks at or past K are the zero padding
    const long long total = blocks_per_row * rows;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int o = (int)(i / blocks_per_row), b = (int)(i % blocks_per_row);
        const uint8_t* src = w + (long long)o * row_bytes;
        float v[32];
        if (b >= K / 32) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.0f;
        } else if (type == 8) {  // q8_0: f16 d, int8 q[32]
            const uint8_t* blk = src + (long long)b * 34;
            const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = d * (float)(int8_t)blk[2 + j];
        } else if (type == 2) {  // q4_0: f16 d, 16 bytes; element j low nibble, j+16 high nibble, value d*(q-8)
            const uint8_t* blk = src + (long long)b * 18;
            const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                v[j] = d * (float)((int)(blk[2 + j] & 0x0F) - 8);
                v[j + 16] = d * (float)((int)(blk[2 + j] >> 4) - 8);
            }
        } else if (type == 0) {
            const float* f = reinterpret_cast<const float*>(src) + b * 32;
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = f[j];
        } else {
            const unsigned short* u = reinterpret_cast<const unsigned short*>(src) + b * 32;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                v[j] = type == 1 ? __half2float(__ushort_as_half(u[j])) : __bfloat162float(__ushort_as_bfloat16(u[j]));
        }
        uint4* d = reinterpret_cast<uint4*>(dst + (long long)(row0 + o) * Kp + b * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q)
            d[q] = make_uint4(Pack2<__nv_bfloat16>::pack(v[8 * q], v[8 * q + 1]),
                              Pack2<__nv_bfloat16>::pack(v[8 * q + 2], v[8 * q + 3]),
                              Pack2<__nv_bfloat16>::pack(v[8 * q + 4], v[8 * q + 5]),
                              Pack2<__nv_bfloat16>::pack(v[8 * q + 6], v[8 * q + 7]));
    }
}

// x f32 [K, L, N] (rows 16-byte aligned) -> bf16 [Kp, L*N] contiguous, columns K .. Kp-1 zero; 8 elements
// per thread.
__global__ void to_bf16_rows_kernel(const char* x, long long nb1, long long nb2, int K, int Kp, int L, long long M,
                                    __nv_bfloat16* dst) {
    const long long per_row = Kp / 8;
    const long long total = per_row * M;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long m = i / per_row;
        const int c = (int)(i % per_row) * 8;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
        if (c < K) {  // K is a multiple of 32: a group of 8 is wholly inside or wholly padding
            const float4* s = reinterpret_cast<const float4*>(x + (m / L) * nb2 + (m % L) * nb1 + (long long)c * 4);
            a = s[0];
            b = s[1];
        }
        *reinterpret_cast<uint4*>(dst + m * Kp + c) =
            make_uint4(Pack2<__nv_bfloat16>::pack(a.x, a.y), Pack2<__nv_bfloat16>::pack(a.z, a.w),
                       Pack2<__nv_bfloat16>::pack(b.x, b.y), Pack2<__nv_bfloat16>::pack(b.z, b.w));
    }
}

// (cos, sin) of every (token l, rotary pair i): angle = pos_axis(l) * freq_i / scale_axis, the
// prologue's formula (rope.hpp:78-95 order of operations, correctly rounded float ops).
__global__ void rope_table_kernel(const RopeTab tab, int L, int pairs, float2* cs) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < (long long)L * pairs;
         i += (long long)gridDim.x * blockDim.x) {
        const int l = (int)(i / pairs), pi = (int)(i % pairs);
        const int w = l % tab.grid_w, hh = (l / tab.grid_w) % tab.grid_h, t = l / (tab.grid_w * tab.grid_h);
        const int ax = tab.axis[pi];
        const float pos = (float)(ax == 0 ? t : (ax == 1 ? hh : w));
        float s, c;
        sincosf(__fdiv_rn(__fmul_rn(pos, tab.freq[pi]), tab.div[pi]), &s, &c);
        cs[i] = make_float2(c, s);
    }
}

int grid_1d(long long work, int num_sms) {
    long long b = (work + 255) / 256;
    const long long cap = (long long)num_sms * 8;
    if (b > cap) b = cap;
    return (int)(b < 1 ? 1 : b);
}

}  // namespace

cudaError_t launch_expand_weights(const void* w, int type, long long row_bytes, int K, int Kp, int rows, int row0,
                                  __nv_bfloat16* dst, int num_sms, cudaStream_t st) {
    const long long total = (long long)(Kp / 32) * rows;
    if (total == 0) return cudaSuccess;
    expand_weights_kernel<<<grid_1d(total, num_sms), 256, 0, st>>>(static_cast<const uint8_t*>(w), type, row_bytes, K,
                                                                    Kp, rows, row0, dst);
    return cudaGetLastError();
}

cudaError_t launch_to_bf16_rows(const void* x, long long nb1, long long nb2, int K, int Kp, int L, long long M,
                                __nv_bfloat16* dst, int num_sms, cudaStream_t st) {
    if (M == 0) return cudaSuccess;
    to_bf16_rows_kernel<<<grid_1d(M * (Kp / 8), num_sms), 256, 0, st>>>(static_cast<const char*>(x), nb1, nb2, K, Kp,
                                                                        L, M, dst);
    return cudaGetLastError();
}

cudaError_t launch_rope_table(const RopeTab& tab, int L, int pairs, float2* cs, int num_sms, cudaStream_t st) {
    if (L == 0) return cudaSuccess;
    rope_table_kernel<<<grid_1d((long long)L * pairs, num_sms), 256, 0, st>>>(tab, L, pairs, cs);
    return cudaGetLastError();
}

cudaError_t launch_qkv_gemm(OutType ot, const CUtensorMap& tmX, const CUtensorMap& tmW, const QkvParams& p, int num_sms,
                            cudaStream_t st) {
    // head dim 64 (the lite model's normalised/rotated slots) or 128 (also every plain linear)
    auto kern = p.D == 64 ? (ot == OutType::BF16 ? qkv_gemm_kernel<__nv_bfloat16, 64>
                                                 : (ot == OutType::F16 ? qkv_gemm_kernel<__half, 64>
                                                                       : qkv_gemm_kernel<float, 64>))
                          : (ot == OutType::BF16 ? qkv_gemm_kernel<__nv_bfloat16, 128>
                                                 : (ot == OutType::F16 ? qkv_gemm_kernel<__half, 128>
                                                                       : qkv_gemm_kernel<float, 128>));
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kGSmemAlloc);
    if (e != cudaSuccess) return e;
    const long long tiles = (long long)((p.M + kPairM - 1) / kPairM) * (p.nslots * p.C / kBN);
    if (tiles <= 0) return cudaSuccess;
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kGThreads);
    cfg.dynamicSmemBytes = kGSmemAlloc;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // one persistent CTA pair per pair of SMs that can hold one at the same time
    cfg.gridDim = dim3((unsigned)(2 * ((num_sms + 1) / 2)));
    int pairs = 0;
    e = cudaOccupancyMaxActiveClusters(&pairs, kern, &cfg);
    if (e != cudaSuccess) return e;
    if (pairs <= 0) return cudaErrorInvalidConfiguration;
    if (pairs > tiles) pairs = (int)tiles;
    cfg.gridDim = dim3((unsigned)(2 * pairs));
    return cudaLaunchKernelEx(&cfg, kern, tmX, tmW, p);
}

}  // namespace kd
