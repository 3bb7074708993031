// kd_kernels.cu -- the HBM-bound kernels around the attention core:
//   - prologue: RMSNorm per head + 3D RoPE + cast + permute in one pass
//     (replaces crossdit.hpp:132-141 and ops.hpp:122-131,167-169);
//   - Q rounding to the operand type (ggml rounds f32 Q to K's dot type);
//   - classification of an f16 additive mask into 64 x 64 skip/full/mixed tiles;
//   - Philox4x32-10 + Box-Muller fill (src/rng.hpp:51-69 counter layout);
//   - the permute that follows the head all-gather.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kd_common.cuh"
#include "kd_internal.h"

namespace kd {

namespace {

template <typename TO>
__device__ __forceinline__ void store4(void* dst, float a, float b, float c, float d);
template <>
__device__ __forceinline__ void store4<float>(void* dst, float a, float b, float c, float d) {
    *reinterpret_cast<float4*>(dst) = make_float4(a, b, c, d);
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(void* dst, float a, float b, float c, float d) {
    *reinterpret_cast<uint2*>(dst) = make_uint2(Pack2<__nv_bfloat16>::pack(a, b), Pack2<__nv_bfloat16>::pack(c, d));
}
template <>
__device__ __forceinline__ void store4<__half>(void* dst, float a, float b, float c, float d) {
    *reinterpret_cast<uint2*>(dst) = make_uint2(Pack2<__half>::pack(a, b), Pack2<__half>::pack(c, d));
}

__device__ __forceinline__ float pick_pos(int axis, int t, int h, int w) { return (float)(axis == 0 ? t : (axis == 1 ? h : w)); }

// RMSNorm over one head row of D elements held as one float4 per lane in D/4 consecutive lanes (all
// 32 lanes call it), following ggml's CPU rms_norm: squares formed in float, summed in double, mean
// rounded to float, scale = 1/sqrtf(mean + eps), y = x*scale*g.
template <int D>
__device__ __forceinline__ float4 rms_norm_row(float4 x, float4 g, float eps) {
    double ss = (double)__fmul_rn(x.x, x.x) + (double)__fmul_rn(x.y, x.y) + (double)__fmul_rn(x.z, x.z) +
                (double)__fmul_rn(x.w, x.w);
#pragma unroll
    for (int o = D / 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float mean = (float)(ss * (1.0 / D));  // 1/D is exact: D is a power of two
    const float scale = __frcp_rn(__fsqrt_rn(__fadd_rn(mean, eps)));
    return make_float4(__fmul_rn(__fmul_rn(x.x, scale), g.x), __fmul_rn(__fmul_rn(x.y, scale), g.y),
                       __fmul_rn(__fmul_rn(x.z, scale), g.z), __fmul_rn(__fmul_rn(x.w, scale), g.w));
}

// RoPE of rotary pairs (x, y) and (z, w) as rope::apply does it (rope.hpp:140-141):
// x0' = x0*c - x1*s, x1' = x0*s + x1*c, each product rounded separately (no contraction).
__device__ __forceinline__ float4 rope_row(float4 x, float s0, float c0, float s1, float c1) {
    return make_float4(__fsub_rn(__fmul_rn(x.x, c0), __fmul_rn(x.y, s0)), __fadd_rn(__fmul_rn(x.x, s0), __fmul_rn(x.y, c0)),
                       __fsub_rn(__fmul_rn(x.z, c1), __fmul_rn(x.w, s1)), __fadd_rn(__fmul_rn(x.z, s1), __fmul_rn(x.w, c1)));
}

// blockIdx.y selects the projection (its parameters stay in registers for the
// whole loop); one warp per (sequence n, token l, group of kPrologueHeads
// warp rows) of it, all of the group's row loads issued before any arithmetic.
// A warp row is 128 consecutive elements of x: one head of 128, or two heads of
// 64 (lanes 0-15 and 16-31).  A lane owns elements 4*hl .. 4*hl+3 of its head
// (hl = lane within the head), i.e. rotary pairs 2*hl and 2*hl+1, whose angle
// depends only on the token: sin/cos are computed once per token and reused
// for the group's heads.  The angle is pos * freq / scale_factor as
// rope.hpp:78-95 computes it.
// (Q, K and V of one token in one item, sharing sin/cos between Q and K, was
// measured slower: 12 rows per item needs 104 registers and halves occupancy.)
template <typename TO, int D>
__global__ void __launch_bounds__(256) prologue_kernel(const __grid_constant__ PrologueParams p) {
    const int lane = threadIdx.x & 31;
    constexpr int lph = D / 4;           // lanes per head: 32 or 16
    constexpr int hpr = 128 / D;         // heads per warp row: 1 or 2
    const int hl = lane & (lph - 1);     // lane within its head
    const int sub = lane / lph;          // head within the warp row
    // per-lane RoPE constants, read from the parameter bank once (not per row)
    const float fr0 = p.tab.freq[2 * hl], fr1 = p.tab.freq[2 * hl + 1];
    const float dv0 = p.tab.div[2 * hl], dv1 = p.tab.div[2 * hl + 1];
    const int ax0 = p.tab.axis[2 * hl], ax1 = p.tab.axis[2 * hl + 1];
    const PrologueJob& T = p.job[blockIdx.y];
    float4 g = make_float4(1.f, 1.f, 1.f, 1.f);
    if (T.norm && T.gain) g = __ldg(reinterpret_cast<const float4*>(T.gain) + hl);
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    const int wrows = (T.H + hpr - 1) / hpr;  // warp rows per token
    const int hgroups = (wrows + kPrologueHeads - 1) / kPrologueHeads;
    const long long items = (long long)T.N * T.L * hgroups;
    for (long long it = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); it < items; it += warps) {
        const int hg = (int)(it % hgroups);
        const long long nl = it / hgroups;
        const int l = (int)(nl % T.L);
        const int n = (int)(nl / T.L);
        const int r0 = hg * kPrologueHeads;               // first warp row of the item
        const int nr = min(kPrologueHeads, wrows - r0);
        const int h0 = r0 * hpr + sub;                    // this lane's head in warp row 0
        const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<const char*>(T.x) +
                                                            (long long)n * T.x_nb2 + (long long)l * T.x_nb1) +
                            r0 * 32 + lane;
        // head of warp row j present (with two heads per row, an odd head count leaves the second
        // half of the last row empty: zeros, normalised beside the others, never stored)
        auto present = [&](int j) { return hpr == 1 || h0 + j * hpr < T.H; };
        float4 v[kPrologueHeads];
#pragma unroll
        for (int j = 0; j < kPrologueHeads; ++j) {
            if (hpr > 1) v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (j < nr && present(j)) v[j] = __ldcs(src + j * 32);
        }
        float s0 = 0.f, c0 = 1.f, s1 = 0.f, c1 = 1.f;
        if (T.rope) {
            const int hw = p.tab.grid_h * p.tab.grid_w;
            const int t = l / hw, hh = (l / p.tab.grid_w) % p.tab.grid_h, w = l % p.tab.grid_w;
            sincosf(__fdiv_rn(__fmul_rn(pick_pos(ax0, t, hh, w), fr0), dv0), &s0, &c0);
            sincosf(__fdiv_rn(__fmul_rn(pick_pos(ax1, t, hh, w), fr1), dv1), &s1, &c1);
        }
        char* dst = reinterpret_cast<char*>(T.y) + (long long)n * T.y_nb3 + (long long)h0 * T.y_nb2 +
                    (long long)l * T.y_nb1 + (long long)hl * 4 * sizeof(TO);
#pragma unroll
        for (int j = 0; j < kPrologueHeads; ++j) {
            if (j >= nr) break;
            float4 x = v[j];
            if (T.norm) x = rms_norm_row<D>(x, g, p.eps);
            if (T.rope) x = rope_row(x, s0, c0, s1, c1);
            if (present(j)) store4<TO>(dst + (long long)j * hpr * T.y_nb2, x.x, x.y, x.z, x.w);
        }
    }
}

__device__ __forceinline__ float load_elt(const void* base, long long idx, int type) {
    if (type == 0) return __ldg(reinterpret_cast<const float*>(base) + idx);
    const unsigned short b = __ldg(reinterpret_cast<const unsigned short*>(base) + idx);
    if (type == 1) return __half2float(__ushort_as_half(b));
    return __bfloat162float(__ushort_as_bfloat16(b));
}

// One warp per piece of a row -- the whole row for D = 64 or 128 (4 elements per lane), 128 elements
// for D = 512; the source row is contiguous (nb0 = element size), so piece j starts 128 * j elements
// into it.
template <typename TD>
__global__ void __launch_bounds__(256) convert_q_kernel(const ConvertParams p) {
    const int lane = threadIdx.x & 31;
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    const int width = p.D < kHeadDim ? p.D : kHeadDim;  // elements per piece
    const int sub = p.D / width;                        // pieces per row
    const long long lsub = (long long)p.L * sub;
    const long long rows = (long long)p.N * p.H * lsub;
    const int esz = p.src_type == 0 ? 4 : 2;
    if (4 * lane >= width) return;  // (64-wide rows: lanes 16-31 have nothing to do)
    for (long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows;
         row += warps) {
        const long long lj = row % lsub;
        const int l = (int)(lj / sub), j = (int)(lj % sub);
        const long long nh = row / lsub;
        const int h = (int)(nh % p.H);
        const int n = (int)(nh / p.H);
        const char* src = reinterpret_cast<const char*>(p.src) + (long long)n * p.nb3 + (long long)h * p.nb2 +
                          (long long)l * p.nb1 + (long long)j * width * esz;
        float a = load_elt(src, 4 * lane + 0, p.src_type), b = load_elt(src, 4 * lane + 1, p.src_type);
        float c = load_elt(src, 4 * lane + 2, p.src_type), d = load_elt(src, 4 * lane + 3, p.src_type);
        char* dst = reinterpret_cast<char*>(p.dst) + (row * width + 4 * lane) * (long long)sizeof(TD);
        store4<TD>(dst, a, b, c, d);
    }
}

// One warp per 64 x 64 (query x key) tile, grid-strided over all tiles of all
// mask planes: lane l reads keys 2l, 2l+1 of the tile's 64 rows, 8 rows in
// flight at a time, and the warp votes whether every in-range element is -inf
// (skip) or +-0 (full); anything else is mixed.  Elements outside
// [0,Lq) x [0,Lk) are ignored; a tile with no in-range element is a skip tile.
// A tile whose bit in the optional bitmap is clear is skip and its mask
// elements are never read; without a mask, a set bit means full.
__global__ void __launch_bounds__(256) mask_classify_kernel(const MaskClassParams p) {
    const int lane = threadIdx.x & 31;
    const long long tiles_per_plane = (long long)p.n_qb * p.n_kb;
    const long long tiles = tiles_per_plane * p.mh * p.mn;
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    for (long long t = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < tiles; t += warps) {
        const int plane = (int)(t / tiles_per_plane);
        const long long r = t % tiles_per_plane;
        const int qb = (int)(r / p.n_kb), kb = (int)(r % p.n_kb);
        if (p.bits || !p.mask) {
            const bool bit = !p.bits || ((p.bits[(long long)qb * p.bits_row_bytes + (kb >> 3)] >> (kb & 7)) & 1u);
            if (!bit || !p.mask) {
                if (lane == 0) p.cls[t] = bit ? kTileFull : kTileSkip;
                continue;
            }
        }
        const int mhi = plane % p.mh, mni = plane / p.mh;
        const char* base = reinterpret_cast<const char*>(p.mask) + (long long)mni * p.nb3 + (long long)mhi * p.nb2;
        if (p.vec16 && (qb + 1) * 64 <= p.Lq && (kb + 1) * 64 <= p.Lk) {
            // Interior tile, 16-byte aligned rows: lane reads 8 values (16 B) of a row, 4 rows per
            // warp load, and folds them into a running OR and AND of the 32-bit words.  All -inf
            // <=> AND == OR == 0xFC00FC00; all +-0 <=> (OR & 0x7FFF7FFF) == 0.
            const int rsub = lane >> 3, c16 = lane & 7;
            const char* t0 = base + (long long)(qb * 64 + rsub) * p.nb1 + (long long)kb * 128 + c16 * 16;
            uint32_t vor = 0u, vand = 0xFFFFFFFFu;
#pragma unroll 8
            for (int r0 = 0; r0 < 64; r0 += 4) {
                const uint4 w = __ldg(reinterpret_cast<const uint4*>(t0 + (long long)r0 * p.nb1));
                vor |= w.x | w.y | w.z | w.w;
                vand &= w.x & w.y & w.z & w.w;
            }
            vor = __reduce_or_sync(0xffffffffu, vor);
            vand = __reduce_and_sync(0xffffffffu, vand);
            if (lane == 0)
                p.cls[t] = (vand == 0xFC00FC00u && vor == 0xFC00FC00u)
                               ? kTileSkip
                               : ((vor & 0x7FFF7FFFu) == 0u ? kTileFull : kTileMixed);
            continue;
        }
        const int key = kb * 64 + 2 * lane;
        const int rows = min(64, p.Lq - qb * 64);
        bool all_inf = true, all_zero = true;
        for (int r0 = 0; r0 < rows; r0 += 8) {
            uint16_t v[8][2];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint16_t* row = reinterpret_cast<const uint16_t*>(base + (long long)(qb * 64 + r0 + i) * p.nb1);
                const bool in_row = r0 + i < rows;
                v[i][0] = (in_row && key < p.Lk) ? __ldg(row + key) : (uint16_t)0xFC00u;
                v[i][1] = (in_row && key + 1 < p.Lk) ? __ldg(row + key + 1) : (uint16_t)0xFC00u;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const bool in = r0 + i < rows && key + e < p.Lk;
                    if (in) {
                        all_inf &= (v[i][e] == 0xFC00u);
                        all_zero &= ((v[i][e] & 0x7FFFu) == 0u);
                    }
                }
        }
        const bool wi = __all_sync(0xffffffffu, all_inf);
        const bool wz = __all_sync(0xffffffffu, all_zero);
        if (lane == 0) p.cls[t] = wi ? kTileSkip : (wz ? kTileFull : kTileMixed);
    }
}

// Philox4x32-10 (Salmon et al. 2011) with the counter/key layout of
// PhiloxRNG::randn (rng.hpp:51-69) and Box-Muller (rng.hpp:130-134).
__global__ void randn_kernel(float* dst, unsigned long long n, unsigned long long seed, unsigned offset) {
    const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
    for (unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        unsigned c0 = offset, c1 = 0, c2 = (unsigned)i, c3 = 0;
        unsigned k0 = (unsigned)(seed & 0xffffffffull), k1 = (unsigned)(seed >> 32);
#pragma unroll
        for (int r = 0; r < 10; ++r) {
            const unsigned long long p0 = (unsigned long long)c0 * 0xD2511F53ull;
            const unsigned long long p1 = (unsigned long long)c2 * 0xCD9E8D57ull;
            const unsigned n0 = (unsigned)(p1 >> 32) ^ c1 ^ k0;
            const unsigned n1 = (unsigned)p1;
            const unsigned n2 = (unsigned)(p0 >> 32) ^ c3 ^ k1;
            const unsigned n3 = (unsigned)p0;
            c0 = n0; c1 = n1; c2 = n2; c3 = n3;
            if (r < 9) { k0 += 0x9E3779B9u; k1 += 0xBB67AE85u; }
        }
        const float inv32 = 2.3283064e-10f;
        const float inv32_2pi = 2.3283064e-10f * 6.2831855f;
        const float u = __fadd_rn(__fmul_rn((float)c0, inv32), inv32 / 2);
        const float v = __fadd_rn(__fmul_rn((float)c1, inv32_2pi), inv32_2pi / 2);
        dst[i] = __fmul_rn(sqrtf(-2.0f * logf(u)), sinf(v));
    }
}

// dst row r = concat over ranks k of src[k][r] (each shard_row_bytes long, 16-byte multiple).
__global__ void unshard_kernel(const uint4* src, uint4* dst, long long rows, int ranks, long long shard_u4) {
    const long long total = rows * ranks * shard_u4;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        const long long w = i % shard_u4;
        const long long rk = i / shard_u4;
        const int k = (int)(rk % ranks);
        const long long r = rk / ranks;
        dst[i] = src[((long long)k * rows + r) * shard_u4 + w];
    }
}

// Self-test of the bounded-wait path: one thread waits on a shared-memory mbarrier that nothing
// arrives on, with the same mbar_wait the flash kernel uses.  After ctl.wait_ns the wait gives
// up, sets kErrSelfTest in the error word and the abort flag, and the kernel returns.
__global__ void wait_selftest_kernel(DevCtl ctl) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        mbar_wait(&bar, 0, ctl, kErrSelfTest, /*honor_abort=*/false, /*sleep_ns=*/1000);
    }
}

int grid_for(long long warps_needed, int num_sms) {
    long long blocks = (warps_needed + 7) / 8;
    long long cap = (long long)num_sms * 16;
    if (blocks > cap) blocks = cap;
    return (int)(blocks < 1 ? 1 : blocks);
}

}  // namespace

cudaError_t launch_prologue(OutType yt, const PrologueParams& p, int num_sms, cudaStream_t st) {
    long long items = 0;
    for (int j = 0; j < p.njobs; ++j) {
        const PrologueJob& J = p.job[j];
        const int wrows = (J.H + 128 / p.D - 1) / (128 / p.D);
        const long long n = (long long)J.N * J.L * ((wrows + kPrologueHeads - 1) / kPrologueHeads);
        items = items > n ? items : n;
    }
    if (items == 0 || p.njobs <= 0) return cudaSuccess;
    const dim3 grid(grid_for(items, num_sms), p.njobs);
    if (p.D == kHeadDim64) {
        if (yt == OutType::BF16)
            prologue_kernel<__nv_bfloat16, kHeadDim64><<<grid, 256, 0, st>>>(p);
        else if (yt == OutType::F16)
            prologue_kernel<__half, kHeadDim64><<<grid, 256, 0, st>>>(p);
        else
            prologue_kernel<float, kHeadDim64><<<grid, 256, 0, st>>>(p);
    } else {
        if (yt == OutType::BF16)
            prologue_kernel<__nv_bfloat16, kHeadDim><<<grid, 256, 0, st>>>(p);
        else if (yt == OutType::F16)
            prologue_kernel<__half, kHeadDim><<<grid, 256, 0, st>>>(p);
        else
            prologue_kernel<float, kHeadDim><<<grid, 256, 0, st>>>(p);
    }
    return cudaGetLastError();
}

cudaError_t launch_wait_selftest(unsigned* err, unsigned* abort_flag, unsigned long long wait_ns, cudaStream_t st) {
    wait_selftest_kernel<<<1, 32, 0, st>>>(DevCtl{err, abort_flag, wait_ns});
    return cudaGetLastError();
}

cudaError_t launch_convert_q(OpType dt, const ConvertParams& p, int num_sms, cudaStream_t st) {
    const long long rows = (long long)p.N * p.H * p.L * (p.D > kHeadDim ? p.D / kHeadDim : 1);
    if (rows == 0) return cudaSuccess;
    const int grid = grid_for(rows, num_sms);
    if (dt == OpType::BF16)
        convert_q_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(p);
    else
        convert_q_kernel<__half><<<grid, 256, 0, st>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_mask_classify(const MaskClassParams& p, cudaStream_t st) {
    if (p.n_qb == 0 || p.n_kb == 0) return cudaSuccess;
    const long long tiles = (long long)p.n_qb * p.n_kb * p.mh * p.mn;
    long long blocks = (tiles + 7) / 8;
    if (blocks > 148LL * 64) blocks = 148LL * 64;
    mask_classify_kernel<<<(int)blocks, 256, 0, st>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_randn(float* dst, unsigned long long n, unsigned long long seed, unsigned offset, int num_sms,
                         cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    long long blocks = (long long)((n + 255) / 256);
    if (blocks > (long long)num_sms * 32) blocks = (long long)num_sms * 32;
    randn_kernel<<<(int)blocks, 256, 0, st>>>(dst, n, seed, offset);
    return cudaGetLastError();
}

cudaError_t launch_unshard_heads(const void* src, void* dst, long long rows, int ranks, long long shard_row_bytes,
                                 int num_sms, cudaStream_t st) {
    const long long shard_u4 = shard_row_bytes / 16;
    const long long total = rows * ranks * shard_u4;
    if (total == 0) return cudaSuccess;
    long long blocks = (total + 255) / 256;
    if (blocks > (long long)num_sms * 32) blocks = (long long)num_sms * 32;
    unshard_kernel<<<(int)blocks, 256, 0, st>>>(reinterpret_cast<const uint4*>(src), reinterpret_cast<uint4*>(dst),
                                                rows, ranks, shard_u4);
    return cudaGetLastError();
}

}  // namespace kd
