// kd_fmha.cu -- flash-attention forward for sm_100a (B200).
//
// Computes ggml_flash_attn_ext (called at src/core/ops.hpp:176 of the
// reference) for head_dim 128:  O = softmax(scale * Q K^T + mask) V per
// (head, sequence), fp32 accumulation, f16 or bf16 operands.
//
// Persistent: one CTA per SM takes "units" -- 2 x 128 query rows of one
// (head, sequence) -- from a global counter in increasing order and streams
// the K/V tiles of each unit's head through a shared-memory ring (5 stages of one
// 128 x 128 tile in the dense kernel, 4 plus the kept-tile lists in the masked one):
//
//   warp 0      TMA producer: Q0, Q1 per unit (as soon as the previous unit's
//               last S MMA frees the Q buffer), then K_j, V_j (128 x 128 tiles,
//               two 64-column boxes with 128-byte swizzle each)
//   warp 1      MMA issuer (one thread): S_i = Q_i K_j^T into TMEM (SS MMA,
//               both operands K-major), O_i += P_i V_j (TS MMA, P from TMEM,
//               V MN-major); owns the 512-column TMEM allocation
//   warp 2      scheduler: takes the next unit and publishes it with the list
//               of K/V tiles it must visit (tiles whose mask is entirely -inf
//               for all 256 rows are never loaded), one unit ahead
//   warp 3      head-sharded runs only: copies each finished unit's output rows
//               (already stored locally, read back from L2) into every peer
//               GPU's copy of the output, one coalesced row per instruction
//   warps 4-7   softmax + correction + epilogue for Q tile 0 (TMEM lanes 0-127)
//   warps 8-11  the same for Q tile 1
//
// A unit's epilogue (O out of TMEM, normalise, store) overlaps the next
// unit's Q load and first S MMAs; the next unit's first PV_i waits only for
// the epilogue to have read O_i (o_free).
//
// TMEM columns: S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512); P_i (16-bit,
// two per column) overwrites the first 64 columns of S_i once S_i has been read.
//
// MMA issue order per K/V tile j (FA4-style ping-pong, so one softmax
// warpgroup works while the tensor core runs the other tile's MMAs):
//   PV0(j), S0(j+1), PV1(j), S1(j+1)
// S_i(j+1) is issued after PV_i(j), so the commit that publishes S_i(j+1)
// also certifies that PV_i(j) finished: the softmax may rescale O_i right
// after it sees S_i(j+1) without another barrier.
//
// Softmax keeps a running max m (log2 domain) and only rescales O and the row
// sum when the max grows by more than 8 (P values stay <= 256); the final
// normalisation divides by the row sum, and LSE = (m + log2 l) * ln 2.
//
// Every wait is bounded (kd_common.cuh: mbar_wait); on expiry the CTA records
// an error bit, stops issuing work, drains what it has in flight and frees TMEM.
#include <type_traits>

#include "kd_common.cuh"
#include "kd_internal.h"

namespace kd {

namespace {

constexpr int kTileBytes = kBlockN * kHeadDim * 2;  // 32 KB: one 128 x 128 16-bit tile
constexpr int kBoxBytes = kTileBytes / 2;           // one 128-row x 64-column box
constexpr int kThreads = 384;
constexpr int kOutSlots = 4;  // units published to the copy-out warp and not yet copied

// Shared-memory layout of one instantiation.  The K/V ring gets every byte the 227 KB allow: the
// masked kernel keeps two kept-tile lists (16 KB) and 4 stages; the dense kernel visits every tile
// in order, needs no lists, and gets a 5th stage (its measured bottleneck was waiting for K/V
// tiles to land with only 2 tiles of lookahead per Q tile pair).  The short-key instantiation
// (kQ2: unmasked, a few K/V tiles per unit, as in cross-attention against text states) trades two
// ring stages for a second Q buffer and publishes units two ahead instead of one, so the next
// unit's Q streams in from HBM while this unit computes rather than after its last S MMA.
template <bool kSparse, bool kQ2 = false>
struct Layout {
    static constexpr int kQBufs = kQ2 ? 2 : 1;
    static constexpr int kListBufs = kQ2 ? 3 : 2;   // unit descriptors in flight
    static constexpr int kStages = kSparse ? 4 : (kQ2 ? 3 : 5);
    static constexpr int kSmemQ = 0;
    static constexpr int kSmemKV = kSmemQ + kQBufs * kQTiles * kTileBytes;
    static constexpr int kSmemBar = kSmemKV + kStages * kTileBytes;
    // q_full[2], q_empty[2], kv_full[S], kv_empty[S], then 2 each of s_full, p_full, p_half, o_full,
    // o_free, then drain, kOutSlots each of out_full, out_empty, then 3 each of list_full, list_empty
    static constexpr int kNumBars = 4 + 2 * kStages + 10 + 1 + 2 * kOutSlots + 6;
    static constexpr int kSmemTmemSlot = kSmemBar + kNumBars * 8;
    // unit, n_kept, lk_eff per list buffer (3 each), last0/last1 per list buffer (6), then the
    // copy-out ring's unit per slot
    static constexpr int kSmemUnit = kSmemTmemSlot + 16;
    static constexpr int kSmemList = (kSmemUnit + (15 + kOutSlots) * 4 + 15) & ~15;  // 2 lists (masked only)
    static constexpr int kSmemTotal = kSmemList + (kSparse ? 2 * kMaxKvTiles * 4 : 0);
    static constexpr int kSmemAlloc = kSmemTotal + 1024;  // slack to align the tiles to 1024 bytes
    static_assert(kSmemAlloc <= 232448, "shared memory budget");
};
// threads that release a list buffer: producer warp, MMA warp, both softmax warpgroups
constexpr int kListConsumers = 32 + 32 + 2 * kBlockM;

constexpr uint32_t kTmemCols = 512;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;      // log2 units: P <= 2^8 between rescales
// The short-key instantiation rescales whenever the running maximum grows: a unit there sees one or two
// K/V tiles, and a P taken against a stale maximum leaves the row's largest weight > 1 and rounded to
// the operand type instead of exactly 1 -- on peaked rows (a few dominant keys, as against text states)
// that rounding is most of the output error.
constexpr float kRescaleThresholdQ2 = 0.0f;
// Tuning knobs (compile-time):
//   KD_FMHA_POLY_PAIRS: bit i set = score pair i of each 32-key chunk takes exp2 from the
//                       FMA pipe (exp2_poly) instead of MUFU ex2 (0 = all MUFU).
//   KD_FMHA_SPLIT_P:    1 = hand P to the MMA in two 64-key halves (PV starts on the first
//                       half while the second is exponentiated), 0 = one hand-off.
//   KD_FMHA_MAX3:       1 = three-input max.f32 for the row maximum.
#ifndef KD_FMHA_POLY_PAIRS
#define KD_FMHA_POLY_PAIRS 0x0000u
#endif
#ifndef KD_FMHA_POLY_PAIRS_D64  // the same for the head_dim-64 kernels, whose exponentials bound them
#define KD_FMHA_POLY_PAIRS_D64 0x1249u
#endif
#ifndef KD_FMHA_SPLIT_P
#define KD_FMHA_SPLIT_P 0
#endif
#ifndef KD_FMHA_MAX3
#define KD_FMHA_MAX3 1
#endif
constexpr uint32_t kPolyPairs = KD_FMHA_POLY_PAIRS;
constexpr uint32_t kPolyPairsD64 = KD_FMHA_POLY_PAIRS_D64;


// A list entry's class bits cover the unit's four 64-row groups, two per Q tile: Q tile i needs
// the K/V tile unless all four of its (row group, key half) classes are "skip".
__device__ __forceinline__ bool tile_needed(uint32_t entry, int i) { return ((entry >> (8 * i)) & 0xFFu) != 0; }
constexpr bool kSplitP = KD_FMHA_SPLIT_P != 0;


template <typename TO>
__device__ __forceinline__ void store_row32(TO* dst, const float (&v)[32]);

// 32 bytes per store instruction (st.global.v8.b32): a lane writes whole 32-byte sectors of its row.
// dst must be 32-byte aligned.
__device__ __forceinline__ void st_global_v8(void* dst, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t a4,
                                             uint32_t a5, uint32_t a6, uint32_t a7) {
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst), "r"(a0), "r"(a1), "r"(a2),
                 "r"(a3), "r"(a4), "r"(a5), "r"(a6), "r"(a7)
                 : "memory");
}
template <typename TO>
__device__ __forceinline__ void store_row32_v8(TO* dst, const float (&v)[32]);
template <>
__device__ __forceinline__ void store_row32_v8<float>(float* dst, const float (&v)[32]) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
        st_global_v8(dst + 8 * i, __float_as_uint(v[8 * i]), __float_as_uint(v[8 * i + 1]), __float_as_uint(v[8 * i + 2]),
                     __float_as_uint(v[8 * i + 3]), __float_as_uint(v[8 * i + 4]), __float_as_uint(v[8 * i + 5]),
                     __float_as_uint(v[8 * i + 6]), __float_as_uint(v[8 * i + 7]));
}
template <typename TO>
__device__ __forceinline__ void store_row32_v8(TO* dst, const float (&v)[32]) {  // 16-bit outputs
#pragma unroll
    for (int i = 0; i < 2; ++i)
        st_global_v8(dst + 16 * i, Pack2<TO>::pack(v[16 * i], v[16 * i + 1]), Pack2<TO>::pack(v[16 * i + 2], v[16 * i + 3]),
                     Pack2<TO>::pack(v[16 * i + 4], v[16 * i + 5]), Pack2<TO>::pack(v[16 * i + 6], v[16 * i + 7]),
                     Pack2<TO>::pack(v[16 * i + 8], v[16 * i + 9]), Pack2<TO>::pack(v[16 * i + 10], v[16 * i + 11]),
                     Pack2<TO>::pack(v[16 * i + 12], v[16 * i + 13]), Pack2<TO>::pack(v[16 * i + 14], v[16 * i + 15]));
}

template <>
__device__ __forceinline__ void store_row32<float>(float* dst, const float (&v)[32]) {
    float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int i = 0; i < 8; ++i) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}
template <>
__device__ __forceinline__ void store_row32<__nv_bfloat16>(__nv_bfloat16* dst, const float (&v)[32]) {
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i)
        d[i] = make_uint4(Pack2<__nv_bfloat16>::pack(v[8 * i], v[8 * i + 1]),
                          Pack2<__nv_bfloat16>::pack(v[8 * i + 2], v[8 * i + 3]),
                          Pack2<__nv_bfloat16>::pack(v[8 * i + 4], v[8 * i + 5]),
                          Pack2<__nv_bfloat16>::pack(v[8 * i + 6], v[8 * i + 7]));
}
template <>
__device__ __forceinline__ void store_row32<__half>(__half* dst, const float (&v)[32]) {
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i)
        d[i] = make_uint4(Pack2<__half>::pack(v[8 * i], v[8 * i + 1]), Pack2<__half>::pack(v[8 * i + 2], v[8 * i + 3]),
                          Pack2<__half>::pack(v[8 * i + 4], v[8 * i + 5]),
                          Pack2<__half>::pack(v[8 * i + 6], v[8 * i + 7]));
}

template <typename T, typename TO, bool kSparse, bool kPairs, bool kQ2, int kD>
__global__ void __launch_bounds__(kThreads, 1)
    fmha_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                    const FmhaParams p) {
    static_assert(!(kQ2 && (kSparse || kPairs)), "the double-buffered Q layout is a dense-list instantiation");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    using L = Layout<kSparse, kQ2>;
    constexpr int kStages = L::kStages;
    constexpr int kQBufs = L::kQBufs;
    constexpr int kLB = L::kListBufs;
    constexpr int kSmemQ = L::kSmemQ;
    constexpr int kSmemKV = L::kSmemKV;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const DevCtl ctl{p.err, p.abort_flag, p.wait_ns};
    // Head dim kD = 128, or 64: then only the first 64-column box of every Q/K/V tile is loaded, the S
    // MMAs take 4 K-steps, the PV MMAs N = 64 (O_i's first 64 TMEM columns) and rows are 64 wide.
    static_assert(kD == kHeadDim || kD == kHeadDim64, "head dim 128 or 64");
    constexpr int nbox = kD / 64;
    // Units: normally 256 query rows (Q tiles 0, 1) of one head; in head-pair mode (masked kernel,
    // one mask plane for all heads) the same 128 rows of heads 2hp and 2hp + 1, which need exactly
    // the same K/V tiles, so both Q tiles always have work at every listed tile.
    constexpr int kUnitRows = kPairs ? kBlockM : kRowsPerCta;
    const int n_qblk = (p.Lq + kUnitRows - 1) / kUnitRows;
    const int unit_heads = kPairs ? p.H / 2 : p.H;
    const int n_units = n_qblk * unit_heads * p.N;
    struct UnitGeo {
        int qblk, n;
        int row0[2], head[2];
    };
    auto geo = [&](int u) {
        UnitGeo g;
        g.qblk = u % n_qblk;
        const int hu = (u / n_qblk) % unit_heads;
        g.n = u / (n_qblk * unit_heads);
        for (int i = 0; i < 2; ++i) {
            g.row0[i] = kPairs ? g.qblk * kBlockM : g.qblk * kRowsPerCta + i * kBlockM;
            g.head[i] = kPairs ? 2 * hu + i : hu;
        }
        return g;
    };

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kSmemBar);
    uint64_t* q_full = bars + 0;             // [kQBufs] Q tiles of a unit landed
    uint64_t* q_empty = bars + 2;            // [kQBufs] the last S MMA of the unit using it completed
    uint64_t* kv_full = bars + 4;
    uint64_t* kv_empty = kv_full + kStages;
    uint64_t* s_full = kv_empty + kStages;   // [2]
    uint64_t* p_full = s_full + 2;           // [2]
    uint64_t* p_half = s_full + 4;           // [2] first 64 keys of P_i written (split hand-off only)
    uint64_t* o_full = s_full + 6;           // [2] last PV_i of a unit complete
    uint64_t* o_free = s_full + 8;           // [2] epilogue has read O_i out of TMEM
    uint64_t* drain = s_full + 10;
    uint64_t* out_full = s_full + 11;        // [kOutSlots] a unit's rows are stored locally (256 arrivals)
    uint64_t* out_empty = out_full + kOutSlots;  // [kOutSlots] the copy-out warp is done with the slot
    uint64_t* list_full = out_empty + kOutSlots;  // [kLB] unit descriptor + kept-tile list published
    uint64_t* list_empty = list_full + 3;         // [kLB] every consumer is done with that list buffer
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kSmemTmemSlot);
    int* s_unit = reinterpret_cast<int*>(smem + L::kSmemUnit);  // [kLB] unit index, -1 = no more work
    int* s_nkept = s_unit + 3;                                   // [kLB] kept K/V tiles of the unit
    int* s_lkeff = s_unit + 6;                                   // [kLB] valid keys of the unit's sequence
    int* s_last = s_unit + 9;                                    // [kLB][2] last list entry Q tile i needs, -1: none
    int* s_out_unit = s_unit + 15;                               // [kOutSlots] unit to copy out, -1 = finished
    // [2][kMaxKvTiles] kept-tile lists, masked kernel only; the dense kernel's entry j is tile j, all full
    uint32_t* lists = kSparse ? reinterpret_cast<uint32_t*>(smem + L::kSmemList) : nullptr;
    auto entry = [](const uint32_t* list, int j) -> uint32_t {
        return kSparse ? list[j] : (((uint32_t)j << 16) | 0x5555u);
    };

    if (threadIdx.x == 0) {
        // kQ2 with TMA output stores: a unit's Q buffer doubles as the staging area of its two O tiles,
        // so it is free again once the last S MMA has completed AND both warpgroups' stores have read it
        const uint32_t q_empty_count = (kQ2 && p.tma_out) ? 3u : 1u;
        for (int i = 0; i < 2; ++i) {
            mbar_init(&q_full[i], 1);
            mbar_init(&q_empty[i], q_empty_count);
        }
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], kBlockM);
            mbar_init(&p_half[i], kBlockM);
            mbar_init(&o_full[i], 1);
            mbar_init(&o_free[i], kBlockM);
        }
        for (int i = 0; i < 3; ++i) {
            mbar_init(&list_full[i], 32);
            mbar_init(&list_empty[i], kListConsumers);
        }
        mbar_init(drain, 1);
        for (int i = 0; i < kOutSlots; ++i) {
            mbar_init(&out_full[i], 2 * kBlockM);
            mbar_init(&out_empty[i], 1);
        }
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
    // Without a mask every listed K/V tile is needed by both Q tiles; the dense instantiation folds
    // the per-Q-tile skip tests away.
    auto need = [](uint32_t entry, int i) { return !kSparse || tile_needed(entry, i); };
    // Softmax threads: after storing their rows of the t-th unit (or -1 = no more units), wait for
    // the ring slot to be free and arrive on out_full; thread 128 writes the unit index first.
    auto publish_out = [&](int t, int u) -> bool {
        const int slot = t % kOutSlots;
        if (t >= kOutSlots &&
            !__all_sync(0xffffffffu, mbar_wait(&out_empty[slot], ((t / kOutSlots) - 1) & 1, ctl, kErrTimeoutOut)))
            return false;
        if (threadIdx.x == 128) s_out_unit[slot] = u;
        mbar_arrive(&out_full[slot]);
        return true;
    };


    // Loads a unit's two Q tiles into the next Q buffer, once the last S MMA of the unit that used that
    // buffer before has completed (q_uses counts the units whose Q was loaded so far).  The producer
    // warp does this; in the short-key instantiation the scheduler warp does it right after publishing
    // the unit, about one unit ahead of its use, so the HBM latency of Q overlaps a whole unit.
    auto load_q = [&](const UnitGeo& ug, uint32_t& q_uses) -> bool {
        const int qb = (int)(q_uses % kQBufs);
        if (q_uses >= (uint32_t)kQBufs &&
            !__all_sync(0xffffffffu, mbar_wait(&q_empty[qb], (q_uses / kQBufs - 1) & 1, ctl, kErrTimeoutQ)))
            return false;
        if (lane == 0) {
            mbar_arrive_expect_tx(&q_full[qb], kQTiles * nbox * kBoxBytes);
#pragma unroll
            for (int i = 0; i < kQTiles; ++i)
#pragma unroll
                for (int bx = 0; bx < 2; ++bx)
                    if (bx < nbox)
                        tma_load_4d(smem + kSmemQ + (qb * kQTiles + i) * kTileBytes + bx * kBoxBytes, &tmQ,
                                    &q_full[qb], bx * 64, ug.row0[i], ug.head[i], ug.n);
        }
        __syncwarp();
        ++q_uses;
        return true;
    };
    // Abort path: bounded wait (ignoring the abort flag) for the Q copies still in flight.
    auto drain_q = [&](uint32_t q_uses) {
        for (uint32_t k = (q_uses > (uint32_t)kQBufs ? q_uses - kQBufs : 0u); k < q_uses; ++k)
            mbar_wait(&q_full[k % kQBufs], (k / kQBufs) & 1u, ctl, kErrTimeoutDrain, false);
    };

    if (warp == 2) {
        // ------------------------------------------------------------ work scheduler + list builder
        // Takes units (256 query rows of one head and sequence) from the global counter in increasing
        // order, so CTAs working at the same time share heads and their K/V stay in L2.  For each unit
        // it publishes the list of K/V tiles to visit: entry = (tile << 16) | 2-bit class per
        // (64-row group g, 64-key half hh) at bit 4g + 2hh; without a mask every tile is FULL and the
        // kv_len / Lk tail is masked by index.  Double-buffered: unit t+1's list is built while unit t runs.
        uint32_t q_uses = 0;  // kQ2: units whose Q this warp loaded
        bool q_ok = true;
        for (int t = 0;; ++t) {
            const int b = t % kLB;
            // ahead of the consumers: poll slowly so the softmax warps keep the issue slots (faster
            // when this warp also issues the Q loads)
            if (t >= kLB && !__all_sync(0xffffffffu, mbar_wait(&list_empty[b], ((t / kLB) - 1) & 1, ctl,
                                                               kErrTimeoutList, true, kQ2 ? 200 : 2000)))
                break;
            int u = 0;
            if (lane == 0) u = (int)atomicAdd(p.work_counter, 1u);
            u = __shfl_sync(0xffffffffu, u, 0);
            if (u >= n_units || *reinterpret_cast<volatile unsigned*>(p.abort_flag)) {
                if (lane == 0) s_unit[b] = -1;
                __syncwarp();
                mbar_arrive(&list_full[b]);
                break;
            }
            const UnitGeo ug = geo(u);
            const int n = ug.n, h = ug.head[0];
            int lk_eff = p.Lk;
            if (p.kv_len) {
                const int kl = p.kv_len[n];
                lk_eff = kl < 0 ? 0 : (kl < p.Lk ? kl : p.Lk);
            }
            const int n_kv_tiles = (lk_eff + kBlockN - 1) / kBlockN;
            uint32_t* list = kSparse ? lists + b * kMaxKvTiles : nullptr;
            int count = 0;
            int last[2] = {-1, -1};
            const long long plane =
                p.tile_cls ? ((long long)(n % p.mn) * p.mh + (h % p.mh)) * (long long)p.n_qb * p.n_kb : 0;
            for (int base = 0; base < n_kv_tiles; base += 32) {
                const int kt = base + lane;
                uint32_t bits = 0;
                if (kt < n_kv_tiles) {
                    if (p.tile_cls) {
                        // class of each (64-row group g of the unit, 64-key half hh); head-pair units
                        // have 2 row groups shared by both Q tiles: their byte is copied for tile 1
#pragma unroll
                        for (int g = 0; g < (kPairs ? 2 : 4); ++g) {
                            const int qb = ug.row0[0] / 64 + g;
#pragma unroll
                            for (int hh = 0; hh < 2; ++hh) {
                                const int kb = 2 * kt + hh;
                                uint32_t c = kTileSkip;
                                if (qb < p.n_qb && kb < p.n_kb) c = p.tile_cls[plane + (long long)qb * p.n_kb + kb];
                                bits |= (c & 3u) << (4 * g + 2 * hh);
                            }
                        }
                        if (kPairs) bits |= bits << 8;
                    } else {
                        bits = 0x5555u;
                    }
                }
                const bool kept = bits != 0;
                const uint32_t ballot = __ballot_sync(0xffffffffu, kept);
                if (kSparse && kept) list[count + __popc(ballot & ((1u << lane) - 1u))] = ((uint32_t)kt << 16) | bits;
#pragma unroll
                for (int i = 0; i < 2; ++i) {  // position of the last entry Q tile i needs
                    const uint32_t bi = __ballot_sync(0xffffffffu, tile_needed(bits, i));
                    if (bi) last[i] = count + __popc(ballot & ((1u << (31 - __clz(bi))) - 1u));
                }
                count += __popc(ballot);
            }
            if (p.tile_stats) {
                // tiles this unit loads, and Q-tile x K/V-tile products it computes
                __syncwarp();  // other lanes' list entries are read below
                int pairs = 0;
                for (int j = lane; j < count; j += 32) pairs += (int)need(entry(list, j), 0) + (int)need(entry(list, j), 1);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) pairs += __shfl_xor_sync(0xffffffffu, pairs, o);
                if (lane == 0) {  // head-pair units load every listed tile for both heads
                    atomicAdd(p.tile_stats, (unsigned long long)(kPairs ? 2 * count : count));
                    atomicAdd(p.tile_stats + 1, (unsigned long long)pairs);
                }
            }
            if (lane == 0) {
                s_unit[b] = u;
                s_nkept[b] = count;
                s_lkeff[b] = lk_eff;
                s_last[2 * b] = last[0];
                s_last[2 * b + 1] = last[1];
            }
            __syncwarp();
            mbar_arrive(&list_full[b]);  // every lane: releases its own list writes
            if constexpr (kQ2) {
                if (count > 0 && !(q_ok = load_q(ug, q_uses))) break;
            }
        }
        if (!q_ok) drain_q(q_uses);
    } else if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
        }
        uint32_t it = 0;      // K/V ring position (continues across units)
        uint32_t q_uses = 0;  // units whose Q was loaded
        bool ok = true;
        for (int t = 0; ok; ++t) {
            const int b = t % kLB;
            if (!(ok = __all_sync(0xffffffffu, mbar_wait(&list_full[b], (t / kLB) & 1, ctl, kErrTimeoutList)))) break;
            const int u = s_unit[b];
            if (u < 0) break;
            const int n_iter = s_nkept[b];
            const UnitGeo ug = geo(u);
            const int n = ug.n, nk = n / p.rk3;
            const int hk0 = ug.head[0] / p.rk2, hk1 = ug.head[1] / p.rk2;
            const uint32_t* list = kSparse ? lists + b * kMaxKvTiles : nullptr;
            if (n_iter > 0) {
                if constexpr (!kQ2) {  // (the scheduler warp loads Q in the short-key instantiation)
                    if (!(ok = load_q(ug, q_uses))) break;
                }
                for (int j = 0; j < n_iter && ok; ++j) {
                    const int kt = (int)(entry(list, j) >> 16);
                    // ring order per entry: K, V -- or for head-pair units K(head 0), K(head 1),
                    // V(head 0), V(head 1), the order the MMA warp consumes them in
#pragma unroll 1
                    for (int w = 0; w < (kPairs ? 4 : 2); ++w) {
                        const bool is_v = kPairs ? (w >= 2) : (w == 1);
                        const int hk = (kPairs && (w & 1)) ? hk1 : hk0;
                        const int s = it % kStages;
                        const uint32_t ph = (it / kStages) & 1u;
                        ok = __all_sync(0xffffffffu, mbar_wait(&kv_empty[s], ph ^ 1u, ctl, kErrTimeoutKVEmpty));
                        if (!ok) break;
                        if (lane == 0) {
                            mbar_arrive_expect_tx(&kv_full[s], nbox * kBoxBytes);
                            const CUtensorMap* map = is_v ? &tmV : &tmK;
#pragma unroll
                            for (int bx = 0; bx < 2; ++bx)
                                if (bx < nbox)
                                    tma_load_4d(smem + kSmemKV + s * kTileBytes + bx * kBoxBytes, map, &kv_full[s],
                                                bx * 64, kt * kBlockN, hk, nk);
                        }
                        __syncwarp();
                        ++it;
                    }
                }
                if (!ok) break;
            }
            mbar_arrive(&list_empty[b]);
        }
        if (!ok) {
            // Abort path: wait (bounded, ignoring the abort flag) until every copy this warp issued has
            // landed, so no TMA write targets shared memory after the CTA exits.
            drain_q(q_uses);
            for (uint32_t k = (it > (uint32_t)kStages ? it - kStages : 0u); k < it; ++k)
                mbar_wait(&kv_full[k % kStages], (k / kStages) & 1u, ctl, kErrTimeoutDrain, false);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        const uint32_t qa = smem_u32(smem + kSmemQ);
        const uint32_t kva = smem_u32(smem + kSmemKV);
        constexpr uint32_t idS = idesc_f16_f32acc(kBf16, kBlockM, kBlockN, false);
        // PV's N is the head dim: O_i's first D columns
        constexpr uint32_t idPV = idesc_f16_f32acc(kBf16, kBlockM, kD, true);
        uint32_t it = 0;       // K/V ring position
        uint32_t units = 0;    // units with at least one tile: Q buffer units % kQBufs and its phase
        bool issued = false;

        auto next_stage = [&](int& s) -> bool {
            s = it % kStages;
            const uint32_t ph = (it / kStages) & 1u;
            ++it;
            return __all_sync(0xffffffffu, mbar_wait(&kv_full[s], ph, ctl, kErrTimeoutKVFull));
        };
        // The whole warp runs the issue code (one elected lane issues each instruction).
        // Descriptors: low words built once per tile, a constant added per K-step.
        constexpr uint32_t dhi = sw128_desc_hi(1024);
        uint32_t qbuf = 0;     // Q buffer of the current unit
        auto issue_s = [&](int i, int s, uint32_t qb) {
            const uint32_t alo = sw128_desc_lo(qa + (qb * kQTiles + i) * kTileBytes, 16),
                           blo = sw128_desc_lo(kva + s * kTileBytes, 16);
#pragma unroll
            for (int kk = 0; kk < kD / 16; ++kk) {
                const uint32_t o = ((kk >> 2) * kBoxBytes + (kk & 3) * 32) >> 4;
                mma_ss(tmem + i * 128, desc_join(alo + o, dhi), desc_join(blo + o, dhi), idS, kk > 0 ? 1u : 0u);
            }
        };
        // O_i += P_i V for keys [64*half, 64*half + 64): P columns 32*half.., V rows 64*half..
        auto issue_pv = [&](int i, int s, bool acc, int half) {
            const uint32_t vlo = sw128_desc_lo(kva + s * kTileBytes, kBoxBytes);
#pragma unroll
            for (int k4 = 0; k4 < kBlockN / 32; ++k4) {
                const int kk = half * (kBlockN / 32) + k4;
                mma_ts(tmem + 256 + i * 128, tmem + i * 128 + kk * 8, desc_join(vlo + ((kk * 16 * 128) >> 4), dhi),
                       idPV, (acc || kk > 0) ? 1u : 0u);
            }
        };
        auto commit = [&](uint64_t* bar) { tc_commit(bar); };
        // wait for P_i of its needed tile number gi (both halves, or each half with the split hand-off), issue PV_i
        auto pv = [&](int i, int s, bool acc, uint32_t gi) -> bool {
            if (kSplitP) {
                if (!__all_sync(0xffffffffu, mbar_wait(&p_half[i], gi & 1, ctl, kErrTimeoutP))) return false;
                tc_fence_after();
                issue_pv(i, s, acc, 0);
                if (!__all_sync(0xffffffffu, mbar_wait(&p_full[i], gi & 1, ctl, kErrTimeoutP))) return false;
                tc_fence_after();
                issue_pv(i, s, acc, 1);
                return true;
            }
            if (!__all_sync(0xffffffffu, mbar_wait(&p_full[i], gi & 1, ctl, kErrTimeoutP))) return false;
            tc_fence_after();
            issue_pv(i, s, acc, 0);
            issue_pv(i, s, acc, 1);
            return true;
        };

        // Per K/V tile j of the unit's list, in this order:  PV0(j), S0(j+1), PV1(j), S1(j+1), each
        // only for the Q tiles that need that K/V tile (the list holds tiles some Q tile needs).
        // S_i(next) is always issued after PV_i(now), so P_i's TMEM is read before S_i overwrites it.
        uint32_t gq0 = 0, gq1 = 0;   // needed tiles so far, per Q tile: phase of p_full[i]
        uint32_t uq0 = 0, uq1 = 0;   // units in which Q tile i had work: phase of o_free[i]
        bool pre = false;            // kQ2: S0(0) and S1(0) of this unit were issued by the previous unit
        bool ok = true;
        for (int t = 0; ok; ++t) {
            const int b = t % kLB;
            if (!(ok = __all_sync(0xffffffffu, mbar_wait(&list_full[b], (t / kLB) & 1, ctl, kErrTimeoutList)))) break;
            const int u = s_unit[b];
            if (u < 0) break;
            const int n_iter = s_nkept[b];
            const int last0 = s_last[2 * b], last1 = s_last[2 * b + 1];
            const uint32_t* list = kSparse ? lists + b * kMaxKvTiles : nullptr;
            if (n_iter == 0) {
                mbar_arrive(&list_empty[b]);
                continue;
            }
            qbuf = units % kQBufs;
            if (!(ok = __all_sync(0xffffffffu, mbar_wait(&q_full[qbuf], (units / kQBufs) & 1, ctl, kErrTimeoutQ))))
                break;
            bool first0 = true, first1 = true;
            // PV_i for K/V tile j when Q tile i needs it; the first one of a unit overwrites O_i, so
            // the previous unit's epilogue must have read O_i first (o_free)
            auto pv_tile = [&](int i, int j, bool& first, uint32_t& gi, uint32_t ui, int last, int sv) -> bool {
                if (first && ui > 0 &&
                    !__all_sync(0xffffffffu, mbar_wait(&o_free[i], (ui - 1) & 1, ctl, kErrTimeoutO)))
                    return false;
                if (!pv(i, sv, !first, gi)) return false;
                ++gi;
                first = false;
                if (j == last) commit(&o_full[i]);
                return true;
            };
            if constexpr (kPairs) {
                // head-pair unit: ring order per entry K(head 0), K(head 1), V(head 0), V(head 1);
                // same PV0(j), S0(j+1), PV1(j), S1(j+1) order, each Q tile on its own head's tiles
                int sK0 = 0, sK1 = 0;
                if (!(ok = next_stage(sK0)) || !(ok = next_stage(sK1))) break;
                tc_fence_after();
                issue_s(0, sK0, qbuf);
                commit(&s_full[0]);
                issue_s(1, sK1, qbuf);
                commit(&s_full[1]);
                commit(&kv_empty[sK0]);
                commit(&kv_empty[sK1]);
                if (n_iter == 1) commit(&q_empty[qbuf]);
                issued = true;
                for (int j = 0; j < n_iter; ++j) {
                    const bool more = j + 1 < n_iter;
                    int sV0 = 0, sV1 = 0, sK0n = 0, sK1n = 0;
                    if (!(ok = next_stage(sV0)) || !(ok = next_stage(sV1))) break;
                    if (!(ok = pv_tile(0, j, first0, gq0, uq0, last0, sV0))) break;
                    if (more) {
                        if (!(ok = next_stage(sK0n)) || !(ok = next_stage(sK1n))) break;
                        issue_s(0, sK0n, qbuf);
                        commit(&s_full[0]);
                    }
                    if (!(ok = pv_tile(1, j, first1, gq1, uq1, last1, sV1))) break;
                    commit(&kv_empty[sV0]);
                    commit(&kv_empty[sV1]);
                    if (more) {
                        issue_s(1, sK1n, qbuf);
                        commit(&s_full[1]);
                        commit(&kv_empty[sK0n]);
                        commit(&kv_empty[sK1n]);
                        if (j + 2 == n_iter) commit(&q_empty[qbuf]);
                    }
                }
            } else {
                int sK = 0, sV = 0;
                uint32_t e_next = entry(list, 0);
                if (!pre) {
                    if (!(ok = next_stage(sK))) break;
                    tc_fence_after();
                    if (need(e_next, 0)) {
                        issue_s(0, sK, qbuf);
                        commit(&s_full[0]);
                    }
                    if (need(e_next, 1)) {
                        issue_s(1, sK, qbuf);
                        commit(&s_full[1]);
                    }
                    commit(&kv_empty[sK]);
                    if (n_iter == 1) commit(&q_empty[qbuf]);  // the unit's last S MMA is issued: Q may be replaced
                }
                pre = false;
                issued = true;
                for (int j = 0; j < n_iter; ++j) {
                    const uint32_t e = e_next;
                    const bool more = j + 1 < n_iter;
                    if (more) e_next = entry(list, j + 1);
                    if (!(ok = next_stage(sV))) break;
                    int sK2 = -1;
                    bool early0 = false, early1 = false;
                    // Masked lists: a Q tile with no PV at this K/V tile has nothing to wait for, so its
                    // next S is issued before the other Q tile's PV (which waits on that tile's softmax)
                    // and the tensor core keeps working.  Its previous PV is already queued ahead of it.
                    if (kSparse && more) {
                        early0 = !need(e, 0) && need(e_next, 0);
                        early1 = !need(e, 1) && need(e_next, 1);
                        if (early0 || early1) {
                            if (!(ok = next_stage(sK2))) break;
                            if (early0) {
                                issue_s(0, sK2, qbuf);
                                commit(&s_full[0]);
                            }
                            if (early1) {
                                issue_s(1, sK2, qbuf);
                                commit(&s_full[1]);
                            }
                        }
                    }
                    if (need(e, 0) && !(ok = pv_tile(0, j, first0, gq0, uq0, last0, sV))) break;
                    if (more) {
                        if (sK2 < 0 && !(ok = next_stage(sK2))) break;
                        if (!early0 && need(e_next, 0)) {
                            issue_s(0, sK2, qbuf);
                            commit(&s_full[0]);
                        }
                    }
                    // Short-key instantiation, last tile of the unit: the next unit's Q is already
                    // loading (the scheduler warp issued it a unit ahead), so its S0(0) goes out right
                    // after PV0(last) -- softmax warpgroup 0 then starts the next unit as soon as its
                    // epilogue ends instead of waiting for warpgroup 1's last P.  S1(0) follows PV1(last).
                    int sKn = -1;
                    uint32_t qbn = 0;
                    int nn = 0;
                    if (kQ2 && !more) {
                        const int bn = (t + 1) % kLB;
                        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&list_full[bn], ((t + 1) / kLB) & 1, ctl,
                                                                     kErrTimeoutList))))
                            break;
                        nn = s_unit[bn] >= 0 ? s_nkept[bn] : 0;
                        if (nn > 0) {
                            qbn = (units + 1) % kQBufs;
                            if (!(ok = __all_sync(0xffffffffu, mbar_wait(&q_full[qbn], ((units + 1) / kQBufs) & 1,
                                                                         ctl, kErrTimeoutQ))))
                                break;
                            if (!(ok = next_stage(sKn))) break;
                            tc_fence_after();
                            issue_s(0, sKn, qbn);
                            commit(&s_full[0]);
                        }
                    }
                    if (need(e, 1) && !(ok = pv_tile(1, j, first1, gq1, uq1, last1, sV))) break;
                    commit(&kv_empty[sV]);
                    if (sKn >= 0) {
                        issue_s(1, sKn, qbn);
                        commit(&s_full[1]);
                        commit(&kv_empty[sKn]);
                        if (nn == 1) commit(&q_empty[qbn]);
                        pre = true;
                    }
                    if (more) {
                        if (!early1 && need(e_next, 1)) {
                            issue_s(1, sK2, qbuf);
                            commit(&s_full[1]);
                        }
                        commit(&kv_empty[sK2]);
                        if (j + 2 == n_iter) commit(&q_empty[qbuf]);
                    }
                }
            }
            mbar_arrive(&list_empty[b]);
            if (!first0) ++uq0;
            if (!first1) ++uq1;
            ++units;
        }
        if (issued) {
            // every MMA issued above must retire before the TMEM is released
            commit(drain);
            mbar_wait(drain, 0, ctl, kErrTimeoutDrain, false);
        }
    } else if (warp == 3) {
        // ------------------------------------------------------------ head-sharded copy-out
        // Each finished unit's rows (256 rows of 128 outputs of one head) are read back from this
        // GPU's output (L2-resident: just written) and stored into every peer GPU's copy at the same
        // offset.  A row is 256 or 512 bytes; 16 bytes per lane, so one instruction moves one (f32)
        // or two (16-bit) whole rows: NVLink sees full contiguous rows, and the softmax warps never
        // wait on remote memory.
        if (p.n_peer_out) {
            constexpr int kChunks = kD * (int)sizeof(TO) / 16;  // 16-byte chunks per row (8 to 32)
            constexpr int kRowsPerInstr = 32 / kChunks;
            constexpr int kBatch = 8;                                  // instructions of loads in flight
            const int chunk = lane % kChunks, sub = lane / kChunks;
            for (int t = 0;; ++t) {
                const int slot = t % kOutSlots;
                if (!__all_sync(0xffffffffu, mbar_wait(&out_full[slot], (t / kOutSlots) & 1, ctl, kErrTimeoutOut)))
                    break;
                const int u = s_out_unit[slot];
                __syncwarp();
                if (lane == 0) mbar_arrive(&out_empty[slot]);  // the unit index has been read
                if (u < 0) break;
                const UnitGeo ug = geo(u);
                // a unit's rows: 256 rows of one head, or 128 rows of each of two heads
#pragma unroll 1
                for (int part = 0; part < (kPairs ? 2 : 1); ++part) {
                const int row0 = part ? ug.row0[1] : ug.row0[0], h = part ? ug.head[1] : ug.head[0], n = ug.n;
                const int rows = min(kUnitRows, p.Lq - row0);
                const long long base = (long long)n * p.o_nb3 + (long long)h * p.o_nb1 + (long long)chunk * 16;
                for (int r0 = 0; r0 < rows; r0 += kBatch * kRowsPerInstr) {
                    uint4 v[kBatch];
#pragma unroll
                    for (int i = 0; i < kBatch; ++i) {
                        const int row = r0 + i * kRowsPerInstr + sub;
                        if (row < rows)
                            v[i] = __ldcg(reinterpret_cast<const uint4*>(static_cast<const char*>(p.out) + base +
                                                                         (long long)(row0 + row) * p.o_nb2));
                    }
#pragma unroll 1
                    for (int d = 0; d < p.n_peer_out; ++d) {
#pragma unroll
                        for (int i = 0; i < kBatch; ++i) {
                            const int row = r0 + i * kRowsPerInstr + sub;
                            if (row < rows)
                                *reinterpret_cast<uint4*>(p.peer_out[d] + base + (long long)(row0 + row) * p.o_nb2) = v[i];
                        }
                    }
                }
                }
            }
            // the peers' copies are complete and visible system-wide before this CTA retires
            __threadfence_system();
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------ softmax / correction / epilogue
        const int wg = (warp - 4) >> 2;
        const int r = ((warp & 3) << 5) + lane;          // TMEM lane = row within the Q tile
        const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tS = tmem + lane_addr + wg * 128;
        const uint32_t tO = tmem + lane_addr + 256 + wg * 128;
        const int g4 = kPairs ? (r >> 6) : wg * 2 + (r >> 6);  // 64-row group of this row within the unit
        const float sl2 = p.scale_log2;
        uint32_t g = 0;      // tiles this Q tile needed so far: phase of s_full / p_full
        uint32_t units = 0;  // units in which this Q tile had work: phase of o_full / o_free
        bool ok = true;
        int t = 0;  // units taken (the last, u < 0, ends the loop): also the copy-out ring position
        for (; ok; ++t) {
            const int b = t % kLB;
            if (!(ok = __all_sync(0xffffffffu, mbar_wait(&list_full[b], (t / kLB) & 1, ctl, kErrTimeoutList)))) break;
            const int u = s_unit[b];
            if (u < 0) break;
            const int n_iter = s_nkept[b];
            const int lk_eff = s_lkeff[b];
            const UnitGeo ug = geo(u);
            const int h = wg ? ug.head[1] : ug.head[0], n = ug.n;  // selects: no dynamic indexing
            const uint32_t* list = kSparse ? lists + b * kMaxKvTiles : nullptr;
            const int qrow = (wg ? ug.row0[1] : ug.row0[0]) + r;
            const bool row_valid = qrow < p.Lq;
            float m = -INFINITY, l = 0.f;
            int k = 0;  // tiles of this unit processed by this warpgroup
            for (int j = 0; j < n_iter; ++j) {
                const uint32_t e = entry(list, j);
                if (!need(e, wg)) continue;  // all four sub-tiles masked for this Q tile
                const int kbase = (int)(e >> 16) * kBlockN;
                const uint32_t c0 = (e >> (4 * g4)) & 3u, c1 = (e >> (4 * g4 + 2)) & 3u;
                if (!(ok = __all_sync(0xffffffffu, mbar_wait(&s_full[wg], g & 1, ctl, kErrTimeoutS)))) break;
                tc_fence_after();

                // Mixed tiles: add the additive mask (divided by scale, so that scale*(s + m/scale) =
                // scale*s + m) into S in TMEM, 32 columns at a time.  c0/c1 are warp-uniform (a warp's
                // 32 rows lie in one 64-row group).
                if (c0 == kTileMixed || c1 == kTileMixed) {
                    // this row's mask values (only mixed tiles read them, so the pointer is made here)
                    const uint16_t* mrow = nullptr;
                    if (p.mask && row_valid)
                        mrow = reinterpret_cast<const uint16_t*>(
                            reinterpret_cast<const char*>(p.mask) + (long long)(n % p.mn) * p.m_nb3 +
                            (long long)(h % p.mh) * p.m_nb2 + (long long)qrow * p.m_nb1);
#pragma unroll 1
                    for (int c = 0; c < 4; ++c) {
                        if ((c < 2 ? c0 : c1) != kTileMixed) continue;
                        uint32_t x[32];
                        tmem_ld32_sync(tS + c * 32, x);
                        if (mrow) {
#pragma unroll
                            for (int i = 0; i < 32; ++i) {
                                const int key = kbase + c * 32 + i;
                                if (key < lk_eff) {
                                    const float mv = __half2float(__ushort_as_half(__ldg(mrow + key)));
                                    x[i] = __float_as_uint(fmaf(mv, p.inv_scale, __uint_as_float(x[i])));
                                }
                            }
                        }
                        tmem_st32(tS + c * 32, x);
                    }
                    tmem_wait_st();
                }
                uint32_t su[128];
                tmem_ld128_sync(tS, su);
                // Skipped halves and keys past the valid length become -inf.
                const int lim = lk_eff - kbase;
                const int lim0 = c0 == kTileSkip ? 0 : lim;
                const int lim1 = c1 == kTileSkip ? 0 : lim;
                if (lim0 < 64 || lim1 < 128) {
#pragma unroll
                    for (int c = 0; c < 128; ++c)
                        if (c >= (c < 64 ? lim0 : lim1)) su[c] = __float_as_uint(-INFINITY);
                }
                float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#if KD_FMHA_MAX3
#pragma unroll
                for (int c = 0; c < 128; c += 8) {
                    mx0 = fmax3(mx0, __uint_as_float(su[c]), __uint_as_float(su[c + 1]));
                    mx1 = fmax3(mx1, __uint_as_float(su[c + 2]), __uint_as_float(su[c + 3]));
                    mx2 = fmax3(mx2, __uint_as_float(su[c + 4]), __uint_as_float(su[c + 5]));
                    mx3 = fmax3(mx3, __uint_as_float(su[c + 6]), __uint_as_float(su[c + 7]));
                }
#else
#pragma unroll
                for (int c = 0; c < 128; c += 4) {
                    mx0 = fmaxf(mx0, __uint_as_float(su[c]));
                    mx1 = fmaxf(mx1, __uint_as_float(su[c + 1]));
                    mx2 = fmaxf(mx2, __uint_as_float(su[c + 2]));
                    mx3 = fmaxf(mx3, __uint_as_float(su[c + 3]));
                }
#endif
                const float m_tile = fmax3(mx0, mx1, fmaxf(mx2, mx3)) * sl2;
                const float m_new = fmaxf(m, m_tile);
                const bool resc = m_new > m + (kQ2 ? kRescaleThresholdQ2 : kRescaleThreshold);
                const bool warp_resc = __any_sync(0xffffffffu, resc);
                float alpha = 1.0f;
                if (resc) {
                    alpha = ex2_approx(m - m_new);
                    l *= alpha;
                    m = m_new;
                }
                const float neg_mu = (m == -INFINITY) ? 0.f : -m;
                // Dense lists: scores of even and odd keys go through packed f32x2 FMA and add (the
                // row sum kept as two partial sums, even keys and odd keys, exactly as the scalar
                // form below).  The masked instantiation keeps the scalar form: its extra live
                // state leaves no room for the register pairs.
                const uint64_t sl2x2 = f2_pack(sl2, sl2), nmux2 = f2_pack(neg_mu, neg_mu);
                uint64_t rs2 = f2_pack(0.f, 0.f);
                float rs0 = 0.f, rs1 = 0.f;
                // P for 32 keys -> 16 packed columns of S_i's TMEM
                auto p_chunk = [&](int c) {
                    uint32_t pk[16];
                    // Short-key instantiation: a 32-key chunk wholly past the valid keys (the padded
                    // tail of a text sequence) is all zeros -- no exponentials.  The warp-uniform
                    // branch stays out of the long-key kernel, whose chunks the compiler interleaves.
                    if constexpr (kQ2) {
                        if (32 * c >= (c < 2 ? lim0 : lim1)) {
#pragma unroll
                            for (int i = 0; i < 16; ++i) pk[i] = 0u;
                            tmem_st16(tS + c * 16, pk);
                            return;
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        float xa, xb;
                        if constexpr (!kSparse) {
                            f2_unpack(fma_f32x2(f2_pack(__uint_as_float(su[c * 32 + 2 * i]),
                                                        __uint_as_float(su[c * 32 + 2 * i + 1])),
                                                sl2x2, nmux2),
                                      xa, xb);
                        } else {
                            xa = fmaf(__uint_as_float(su[c * 32 + 2 * i]), sl2, neg_mu);
                            xb = fmaf(__uint_as_float(su[c * 32 + 2 * i + 1]), sl2, neg_mu);
                        }
                        float a, bb;
                        if (((kD == kHeadDim64 ? kPolyPairsD64 : kPolyPairs) >> i) & 1u) {
                            exp2_poly2(xa, xb, a, bb);
                        } else {
                            a = ex2_approx(xa);
                            bb = ex2_approx(xb);
                        }
                        if constexpr (!kSparse) {
                            rs2 = add_f32x2(rs2, f2_pack(a, bb));
                        } else {
                            rs0 += a;
                            rs1 += bb;
                        }
                        pk[i] = Pack2<T>::pack(a, bb);
                    }
                    tmem_st16(tS + c * 16, pk);
                };
                p_chunk(0);
                p_chunk(1);
                // Rescale O_i (PV_i of the previous tile is complete: its commit preceded S_i's).  It only
                // has to precede the first PV_i MMA of this tile; the first 64 scores are dead here.
                if (warp_resc && k > 0) {
#pragma unroll 1
                    for (int c = 0; c < 4; ++c) {
                        uint32_t o[32];
                        tmem_ld32_sync(tO + c * 32, o);
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st32(tO + c * 32, o);
                    }
                }
                if (kSplitP) {
                    tmem_wait_st();
                    tc_fence_before();
                    mbar_arrive(&p_half[wg]);
                }
                p_chunk(2);
                p_chunk(3);
                tmem_wait_st();
                if constexpr (!kSparse) f2_unpack(rs2, rs0, rs1);
                l += rs0 + rs1;
                tc_fence_before();
                mbar_arrive(&p_full[wg]);
                ++g;
                ++k;
            }
            if (!ok) break;
            mbar_arrive(&list_empty[b]);

            // epilogue: O_i / l -> out rows, LSE
            TO* orow = nullptr;
            if (row_valid)
                orow = reinterpret_cast<TO*>(reinterpret_cast<char*>(p.out) + (long long)n * p.o_nb3 +
                                             (long long)qrow * p.o_nb2 + (long long)h * p.o_nb1);
            if (k > 0) {
                if (!(ok = __all_sync(0xffffffffu, mbar_wait(&o_full[wg], units & 1, ctl, kErrTimeoutO)))) break;
                tc_fence_after();
                uint32_t ov[128];
                tmem_ld128_sync(tO, ov);
                tc_fence_before();
                mbar_arrive(&o_free[wg]);  // the next unit's PV_i may overwrite O_i now
                const uint32_t qb_unit = units % kQBufs;  // the unit's Q buffer (dense lists: every unit has work)
                ++units;
                const float inv = l > 0.f ? 1.0f / l : 0.f;
                if constexpr (kQ2 && !std::is_same<TO, float>::value) {
                    if (p.tma_out) {
                        // Short-key epilogue: the O tile goes to shared memory (this unit's Q tile wg, no
                        // longer read once o_full fired) in the swizzled layout of a TMA tile, and one thread
                        // writes it with two tensor stores -- whole 128-byte lines instead of 32-byte pieces
                        // of 32 rows per instruction, whose drain held up the warpgroup's next unit.
                        const uint32_t stg = smem_u32(smem + kSmemQ + (qb_unit * kQTiles + wg) * kTileBytes);
#pragma unroll
                        for (int c = 0; c < 16; ++c) {
                            uint32_t w[4];
#pragma unroll
                            for (int i = 0; i < 4; ++i)
                                w[i] = Pack2<TO>::pack(__uint_as_float(ov[8 * c + 2 * i]) * inv,
                                                       __uint_as_float(ov[8 * c + 2 * i + 1]) * inv);
                            st_shared_v4(stg + (c >> 3) * kBoxBytes + (uint32_t)r * 128u +
                                             ((uint32_t)((c & 7) ^ (r & 7)) << 4),
                                         w[0], w[1], w[2], w[3]);
                        }
                        fence_proxy_async_smem();
                        named_bar_sync(1 + wg, kBlockM);
                        if (r == 0) {
                            const int row0 = wg ? ug.row0[1] : ug.row0[0];
#pragma unroll
                            for (int bx = 0; bx < 2; ++bx)
                                if (bx < nbox) tma_store_4d(&tmO, stg + bx * kBoxBytes, bx * 64, h, row0, n);
                            bulk_commit_group();
                            bulk_wait_group_read0();  // the staging tile has been read: the Q buffer may refill
                            mbar_arrive(&q_empty[qb_unit]);
                        }
                        orow = nullptr;
                    }
                }
                if (orow) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        if (c * 32 >= kD) break;
                        float v[32];
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(ov[c * 32 + i]) * inv;
                        if (p.out_v8)
                            store_row32_v8<TO>(orow + c * 32, v);
                        else
                            store_row32<TO>(orow + c * 32, v);
                    }
                }
            } else if (orow) {
                float z[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) z[i] = 0.f;
#pragma unroll 1
                for (int c = 0; c < kD / 32; ++c) store_row32<TO>(orow + c * 32, z);
            }
            if (row_valid && p.lse)
                p.lse[((long long)n * p.H + h) * p.Lq + qrow] = (l > 0.f) ? (m + log2f(l)) * kLn2 : -INFINITY;
            // head sharding: hand the unit's locally stored rows to the copy-out warp
            if (p.n_peer_out && !(ok = publish_out(t, u))) break;
        }
        // tell the copy-out warp there are no more units (after an abort it leaves on its own)
        if (ok && p.n_peer_out) publish_out(t, -1);
        if (kQ2 && p.tma_out && r == 0) bulk_wait_group0();  // this thread's tensor stores have completed
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

template <typename T, typename TO, int kD>
cudaError_t launch_t(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV, const CUtensorMap& tmO,
                     const FmhaParams& p, cudaStream_t st) {
    // a mask (tile classes) selects the instantiation that skips K/V tiles per Q tile
    // head-pair units when every head shares one mask plane (p.head_pairs, set by the host)
    // without a mask, a short key sequence selects the double-buffered-Q instantiation
    const bool q2 = !p.tile_cls && p.Lk <= kQ2MaxKeys;
    auto kern = p.tile_cls ? (p.head_pairs ? fmha_fwd_kernel<T, TO, true, true, false, kD>
                                           : fmha_fwd_kernel<T, TO, true, false, false, kD>)
                           : (q2 ? fmha_fwd_kernel<T, TO, false, false, true, kD>
                                 : fmha_fwd_kernel<T, TO, false, false, false, kD>);
    // set on every launch: the attribute belongs to the current device, and the call is cheap
    const int smem_bytes = p.tile_cls ? Layout<true>::kSmemAlloc
                                      : (q2 ? Layout<false, true>::kSmemAlloc : Layout<false>::kSmemAlloc);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (e != cudaSuccess) return e;
    // Persistent: one CTA per SM (never more CTAs than units); units are handed out by p.work_counter,
    // which also balances units of unequal cost (masks, kv_len).
    const long long units = p.tile_cls && p.head_pairs
                                ? (long long)((p.Lq + kBlockM - 1) / kBlockM) * (p.H / 2) * p.N
                                : (long long)((p.Lq + kRowsPerCta - 1) / kRowsPerCta) * p.H * p.N;
    const int grid = (int)(units < p.num_ctas ? units : p.num_ctas);
    if (grid <= 0) return cudaSuccess;
    kern<<<grid, kThreads, smem_bytes, st>>>(tmQ, tmK, tmV, tmO, p);
    return cudaGetLastError();
}


template <int kD>
cudaError_t launch_d(OpType op, OutType ot, const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                     const CUtensorMap& tmO, const FmhaParams& p, cudaStream_t st) {
    if (op == OpType::BF16) {
        if (ot == OutType::F32) return launch_t<__nv_bfloat16, float, kD>(tmQ, tmK, tmV, tmO, p, st);
        if (ot == OutType::BF16) return launch_t<__nv_bfloat16, __nv_bfloat16, kD>(tmQ, tmK, tmV, tmO, p, st);
        return launch_t<__nv_bfloat16, __half, kD>(tmQ, tmK, tmV, tmO, p, st);
    }
    if (ot == OutType::F32) return launch_t<__half, float, kD>(tmQ, tmK, tmV, tmO, p, st);
    if (ot == OutType::BF16) return launch_t<__half, __nv_bfloat16, kD>(tmQ, tmK, tmV, tmO, p, st);
    return launch_t<__half, __half, kD>(tmQ, tmK, tmV, tmO, p, st);
}

}  // namespace

int fmha_smem_bytes() { return Layout<true>::kSmemAlloc; }

cudaError_t launch_fmha(OpType op, OutType ot, const CUtensorMap& tmQ, const CUtensorMap& tmK,
                        const CUtensorMap& tmV, const CUtensorMap& tmO, const FmhaParams& p, cudaStream_t st) {
    if (p.D == kHeadDim64) return launch_d<kHeadDim64>(op, ot, tmQ, tmK, tmV, tmO, p, st);
    if (p.D != kHeadDim) return cudaErrorInvalidValue;
    return launch_d<kHeadDim>(op, ot, tmQ, tmK, tmV, tmO, p, st);
}


}  // namespace kd
