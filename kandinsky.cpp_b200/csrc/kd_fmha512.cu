// kd_fmha512.cu -- flash-attention forward for head_dim 512 on sm_100a (B200).
//
// ggml_flash_attn_ext for the one call site of the reference whose head is not 128 wide: the
// VAE mid-block attention, VAEAttnBlock::forward (src/models/vae.hpp:89), which attends over the
// H*W latent positions with ONE head of the full channel count (512) through ops::attention's
// flash branch (src/core/ops.hpp:164-185).  O = softmax(scale * Q K^T) V, fp32 accumulation,
// f16 or bf16 operands; no mask (the call passes none).
//
// One CTA per 128 query rows of one (head, sequence); its Q tile (128 x 512, 128 KB) stays in
// shared memory.  K/V stream through a 6-stage TMA ring in stages of 64 keys x 128 columns.
//
//   warp 0      TMA producer: Q once, then per pass and per 64-key tile K chunks 0-3 and the
//               pass's two V chunks
//   warp 1      MMA issuer: S = sum_c Q_c K_c^T (M=128, N=64, 32 K-steps) into TMEM, then
//               O_half += P V_c for the pass's two 128-column V chunks (P from TMEM)
//   warps 4-7   softmax + epilogue, one query row per thread (TMEM lane = row)
//
// TMEM: S [0, 64) (P, 16-bit pairs, over its first 32 columns), O [64, 320): 256 columns, one
// half of the 512 output columns.  The output is therefore made in two passes over the keys:
// pass 0 computes the online softmax (running max m, row sum l, lazy rescaling of O when m grows
// by more than 8 in log2 units) and the first 256 output columns; pass 1 recomputes S, takes the
// exponentials against pass 0's final m (so no rescaling) and makes the other 256 columns.  The
// tensor core does S twice -- 1.5x the attention's MMA work -- which this once-per-image call
// affords; it keeps every output column in fp32 TMEM until it is normalised.
//
// Every wait is bounded (kd_common.cuh: mbar_wait); on expiry the CTA records an error bit,
// stops issuing work, drains what it has in flight and frees TMEM.
#include <type_traits>

#include "kd_common.cuh"
#include "kd_internal.h"

namespace kd {
namespace {

constexpr int kD = kHeadDim512;
constexpr int kM = 128;                      // query rows per CTA
constexpr int kN = 64;                       // keys per tile
constexpr int kQBox = kM * 128;              // 16 KB: 128 rows x 64 columns (16-bit)
constexpr int kQBytes = kD / 64 * kQBox;     // 128 KB
constexpr int kKVBox = kN * 128;             // 8 KB: 64 rows x 64 columns
constexpr int kStageBytes = 2 * kKVBox;      // 16 KB: 64 keys x 128 columns
constexpr int kStages = 6;
constexpr int kSmemKV = kQBytes;
constexpr int kSmemBar = kSmemKV + kStages * kStageBytes;
// q_full, kv_full[S], kv_empty[S], s_full, p_full, o_full, o_free, drain
constexpr int kNumBars = 1 + 2 * kStages + 5;
constexpr int kSmemSlot = kSmemBar + kNumBars * 8;
constexpr int kSmemAlloc = kSmemSlot + 16 + 1024;
static_assert(kSmemAlloc <= 232448, "shared memory budget");
constexpr int kThreads = 256;
constexpr uint32_t kTmemCols = 512;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;

template <typename TO>
__device__ __forceinline__ void store32(TO* dst, const float (&v)[32]) {
    if constexpr (std::is_same<TO, float>::value) {
        float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
        for (int i = 0; i < 8; ++i) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
        uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
        for (int i = 0; i < 4; ++i)
            d[i] = make_uint4(Pack2<TO>::pack(v[8 * i], v[8 * i + 1]), Pack2<TO>::pack(v[8 * i + 2], v[8 * i + 3]),
                              Pack2<TO>::pack(v[8 * i + 4], v[8 * i + 5]), Pack2<TO>::pack(v[8 * i + 6], v[8 * i + 7]));
    }
}

template <typename T, typename TO>
__global__ void __launch_bounds__(kThreads, 1)
    fmha512_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const FmhaParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const DevCtl ctl{p.err, p.abort_flag, p.wait_ns};
    const int n_qblk = (p.Lq + kM - 1) / kM;
    const int qblk = blockIdx.x % n_qblk;
    const int h = (blockIdx.x / n_qblk) % p.H;
    const int n = blockIdx.x / (n_qblk * p.H);
    const int row0 = qblk * kM;
    const int nk = n / p.rk3, hk = h / p.rk2;
    const int nt = (p.Lk + kN - 1) / kN;  // key tiles (the tail beyond Lk is zero-filled and masked)

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemBar);
    uint64_t* q_full = bars;
    uint64_t* kv_full = bars + 1;
    uint64_t* kv_empty = kv_full + kStages;
    uint64_t* s_full = kv_empty + kStages;
    uint64_t* p_full = s_full + 1;
    uint64_t* o_full = s_full + 2;
    uint64_t* o_free = s_full + 3;
    uint64_t* drain = s_full + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSmemSlot);

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(p_full, kM);
        mbar_init(o_full, 1);
        mbar_init(o_free, kM);
        mbar_init(drain, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            mbar_arrive_expect_tx(q_full, kQBytes);
#pragma unroll 1
            for (int b = 0; b < kD / 64; ++b) tma_load_4d(smem + b * kQBox, &tmQ, q_full, b * 64, row0, h, n);
        }
        __syncwarp();
        uint32_t it = 0;
        bool ok = true;
        // one ring position: wait for the stage, load 64 keys x 128 columns (chunk c) of K or V
        auto push = [&](const CUtensorMap* map, int c, int j) -> bool {
            const int s = it % kStages;
            if (!__all_sync(0xffffffffu, mbar_wait(&kv_empty[s], ((it / kStages) & 1u) ^ 1u, ctl, kErrTimeoutKVEmpty)))
                return false;
            if (lane == 0) {
                mbar_arrive_expect_tx(&kv_full[s], kStageBytes);
#pragma unroll
                for (int b = 0; b < 2; ++b)
                    tma_load_4d(smem + kSmemKV + s * kStageBytes + b * kKVBox, map, &kv_full[s], c * 128 + b * 64,
                                j * kN, hk, nk);
            }
            __syncwarp();
            ++it;
            return true;
        };
        for (int pass = 0; pass < 2 && ok; ++pass)
            for (int j = 0; j < nt && ok; ++j) {
                for (int c = 0; c < kD / 128 && ok; ++c) ok = push(&tmK, c, j);
                for (int c = 0; c < 2 && ok; ++c) ok = push(&tmV, 2 * pass + c, j);
            }
        if (!ok) {  // abort: let every copy this warp issued land before the CTA exits
            mbar_wait(q_full, 0, ctl, kErrTimeoutDrain, false);
            for (uint32_t k = (it > (uint32_t)kStages ? it - kStages : 0u); k < it; ++k)
                mbar_wait(&kv_full[k % kStages], (k / kStages) & 1u, ctl, kErrTimeoutDrain, false);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        const uint32_t qa = smem_u32(smem);
        const uint32_t kva = smem_u32(smem + kSmemKV);
        constexpr uint32_t idS = idesc_f16_f32acc(kBf16, kM, kN, false);
        constexpr uint32_t idPV = idesc_f16_f32acc(kBf16, kM, 128, true);
        constexpr uint32_t dhi = sw128_desc_hi(1024);
        uint32_t it = 0, g = 0;
        bool ok = __all_sync(0xffffffffu, mbar_wait(q_full, 0, ctl, kErrTimeoutQ));
        auto stage = [&](int& s) -> bool {
            s = it % kStages;
            const uint32_t ph = (it / kStages) & 1u;
            ++it;
            return __all_sync(0xffffffffu, mbar_wait(&kv_full[s], ph, ctl, kErrTimeoutKVFull));
        };
        bool issued = false;
        for (int pass = 0; pass < 2 && ok; ++pass) {
            for (int j = 0; j < nt && ok; ++j) {
                // S = sum over the four 128-column chunks of Q_c K_c^T (K-major SW128 on both sides)
                for (int c = 0; c < kD / 128; ++c) {
                    int s = 0;
                    if (!(ok = stage(s))) break;
                    tc_fence_after();
                    const uint32_t blo = sw128_desc_lo(kva + s * kStageBytes, 16);
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint32_t qo = ((2 * c + (kk >> 2)) * kQBox + (kk & 3) * 32) >> 4;
                        const uint32_t ko = ((kk >> 2) * kKVBox + (kk & 3) * 32) >> 4;
                        mma_ss(tmem, desc_join(sw128_desc_lo(qa, 16) + qo, dhi), desc_join(blo + ko, dhi), idS,
                               (c | kk) ? 1u : 0u);
                    }
                    tc_commit(&kv_empty[s]);
                    issued = true;
                }
                if (!ok) break;
                tc_commit(s_full);
                // O_half += P V_c for the pass's two V chunks (V MN-major: keys are rows of 128 bytes,
                // the chunk's two 64-column boxes 8 KB apart)
                if (!(ok = __all_sync(0xffffffffu, mbar_wait(p_full, g & 1, ctl, kErrTimeoutP)))) break;
                ++g;
                if (pass == 1 && j == 0 &&
                    !(ok = __all_sync(0xffffffffu, mbar_wait(o_free, 0, ctl, kErrTimeoutO))))
                    break;
                tc_fence_after();
                for (int c = 0; c < 2; ++c) {
                    int s = 0;
                    if (!(ok = stage(s))) break;
                    tc_fence_after();
                    const uint32_t vlo = sw128_desc_lo(kva + s * kStageBytes, kKVBox);
#pragma unroll
                    for (int kk = 0; kk < kN / 16; ++kk)
                        mma_ts(tmem + 64 + c * 128, tmem + kk * 8, desc_join(vlo + ((kk * 16 * 128) >> 4), dhi), idPV,
                               (j > 0 || kk > 0) ? 1u : 0u);
                    tc_commit(&kv_empty[s]);
                }
            }
            if (ok) tc_commit(o_full);
        }
        if (issued) {
            tc_commit(drain);
            mbar_wait(drain, 0, ctl, kErrTimeoutDrain, false);
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------ softmax + epilogue
        const int r = ((warp & 3) << 5) + lane;
        const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tS = tmem + lane_addr;
        const uint32_t tO = tmem + lane_addr + 64;
        const int qrow = row0 + r;
        const bool row_valid = qrow < p.Lq;
        const float sl2 = p.scale_log2;
        float m = -INFINITY, l = 0.f;
        uint32_t g = 0;
        bool ok = true;
        for (int pass = 0; pass < 2 && ok; ++pass) {
            float lp = 0.f;  // pass 1: row sum against pass 0's final m
            for (int j = 0; j < nt; ++j) {
                if (!(ok = __all_sync(0xffffffffu, mbar_wait(s_full, g & 1, ctl, kErrTimeoutS)))) break;
                ++g;
                tc_fence_after();
                uint32_t su[64];
                tmem_ld64_sync(tS, su);
                const int lim = p.Lk - j * kN;  // keys past Lk are -inf
                if (lim < kN) {
#pragma unroll
                    for (int c = 0; c < kN; ++c)
                        if (c >= lim) su[c] = __float_as_uint(-INFINITY);
                }
                if (pass == 0) {
                    float mx = -INFINITY;
#pragma unroll
                    for (int c = 0; c < kN; c += 2) mx = fmax3(mx, __uint_as_float(su[c]), __uint_as_float(su[c + 1]));
                    const float m_new = fmaxf(m, mx * sl2);
                    const bool resc = m_new > m + kRescaleThreshold;
                    float alpha = 1.f;
                    if (resc) {
                        alpha = ex2_approx(m - m_new);
                        l *= alpha;
                        m = m_new;
                    }
                    // rescale this pass's O (PV of the previous tile is complete: its issue preceded S's)
                    if (__any_sync(0xffffffffu, resc) && j > 0) {
#pragma unroll 1
                        for (int c = 0; c < 8; ++c) {
                            uint32_t o[32];
                            tmem_ld32_sync(tO + c * 32, o);
#pragma unroll
                            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                            tmem_st32(tO + c * 32, o);
                        }
                    }
                }
                const float neg_mu = (m == -INFINITY) ? 0.f : -m;
                float rs = 0.f;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t pk[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float a = ex2_approx(fmaf(__uint_as_float(su[32 * c + 2 * i]), sl2, neg_mu));
                        const float b = ex2_approx(fmaf(__uint_as_float(su[32 * c + 2 * i + 1]), sl2, neg_mu));
                        rs += a + b;
                        pk[i] = Pack2<T>::pack(a, b);
                    }
                    tmem_st16(tS + c * 16, pk);
                }
                if (pass == 0)
                    l += rs;
                else
                    lp += rs;
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(p_full);
            }
            if (!ok) break;
            // epilogue of the pass: O_half / (row sum) -> output columns [256 pass, 256 pass + 256)
            if (!(ok = __all_sync(0xffffffffu, mbar_wait(o_full, pass & 1, ctl, kErrTimeoutO)))) break;
            tc_fence_after();
            const float sum = pass == 0 ? l : lp;
            const float inv = sum > 0.f ? 1.0f / sum : 0.f;
            TO* orow = row_valid ? reinterpret_cast<TO*>(reinterpret_cast<char*>(p.out) + (long long)n * p.o_nb3 +
                                                         (long long)qrow * p.o_nb2 + (long long)h * p.o_nb1) +
                                       pass * 256
                                 : nullptr;
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {
                uint32_t o[32];
                tmem_ld32_sync(tO + c * 32, o);
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(o[i]) * inv;
                if (orow) store32<TO>(orow + c * 32, v);
            }
            tc_fence_before();
            mbar_arrive(o_free);  // pass 1's first PV may overwrite O now
            if (pass == 0 && row_valid && p.lse)
                p.lse[((long long)n * p.H + h) * p.Lq + qrow] = (l > 0.f) ? (m + log2f(l)) * kLn2 : -INFINITY;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

template <typename T, typename TO>
cudaError_t launch512_t(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV, const FmhaParams& p,
                        cudaStream_t st) {
    auto kern = fmha512_kernel<T, TO>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAlloc);
    if (e != cudaSuccess) return e;
    const long long grid = (long long)((p.Lq + kM - 1) / kM) * p.H * p.N;
    if (grid <= 0) return cudaSuccess;
    if (grid > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    kern<<<(unsigned)grid, kThreads, kSmemAlloc, st>>>(tmQ, tmK, tmV, p);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_fmha512(OpType op, OutType ot, const CUtensorMap& tmQ, const CUtensorMap& tmK,
                           const CUtensorMap& tmV, const FmhaParams& p, cudaStream_t st) {
    if (op == OpType::BF16) {
        if (ot == OutType::F32) return launch512_t<__nv_bfloat16, float>(tmQ, tmK, tmV, p, st);
        if (ot == OutType::BF16) return launch512_t<__nv_bfloat16, __nv_bfloat16>(tmQ, tmK, tmV, p, st);
        return launch512_t<__nv_bfloat16, __half>(tmQ, tmK, tmV, p, st);
    }
    if (ot == OutType::F32) return launch512_t<__half, float>(tmQ, tmK, tmV, p, st);
    if (ot == OutType::BF16) return launch512_t<__half, __nv_bfloat16>(tmQ, tmK, tmV, p, st);
    return launch512_t<__half, __half>(tmQ, tmK, tmV, p, st);
}

}  // namespace kd
