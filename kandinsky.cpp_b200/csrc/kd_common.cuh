// kd_common.cuh -- sm_100a building blocks shared by the libkd_attn kernels:
// mbarriers with bounded waits, TMA tile loads, tcgen05 (TMEM alloc, MMA,
// commit, TMEM load/store) and the shared-memory matrix descriptors.
//
// Descriptor bit layouts follow the PTX ISA "tcgen05 matrix descriptor" and
// "instruction descriptor" tables (also encoded by CUTLASS's
// cute::UMMA::SmemDescriptor / InstrDescriptor); tests/test_descriptors.py
// checks the encoders below against CUTLASS's on the CPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace kd {

// Device error word bits (kd_attn_device_status reads them).
enum : unsigned {
    kErrTimeoutQ = 1u << 0,      // Q tile never arrived
    kErrTimeoutKVFull = 1u << 1, // K/V stage never filled
    kErrTimeoutKVEmpty = 1u << 2,// K/V stage never released by the MMA
    kErrTimeoutS = 1u << 3,      // S tile never completed
    kErrTimeoutP = 1u << 4,      // P tile never published by softmax
    kErrTimeoutO = 1u << 5,      // O accumulator never completed
    kErrBadLaunch = 1u << 6,     // launch geometry the kernel does not support
    kErrTimeoutDrain = 1u << 7,  // in-flight copies / MMAs did not drain on the abort path
    kErrTimeoutList = 1u << 8,   // a unit's K/V tile list was never published / released
    kErrTimeoutOut = 1u << 9,    // head-sharded copy-out: a unit's rows never published / slot never freed
    kErrSelfTest = 1u << 10,     // kd_attn_selftest_wait: the wait nothing releases ran out (expected)
};

struct DevCtl {
    unsigned* err;               // sticky device error word (bits above)
    unsigned* abort_flag;        // set by the first CTA that gives up; the others stop early
    unsigned long long wait_ns;  // bound on any single wait
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase with the given parity to complete.  Never spins forever:
// after ctl.wait_ns of wall time (or once another CTA has flagged an abort) it
// records `code` in the device error word and returns false; the caller then
// unwinds its role without issuing further work.
// With honor_abort = false (the drain path) only the time bound ends the wait.
// sleep_ns > 0 backs off between polls, for waiters that are off the critical
// path and should not take issue slots from the warps that are on it.
__device__ __forceinline__ bool mbar_wait_poll(uint64_t* bar, uint32_t parity, const DevCtl ctl, unsigned code, bool honor_abort,
                    unsigned sleep_ns) {
    const unsigned long long t0 = globaltimer_ns();
    for (uint32_t n = 1;; ++n) {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 700
        if (sleep_ns) __nanosleep(sleep_ns);
#endif
        if (mbar_try_wait(bar, parity)) return true;
        if ((n & 63u) == 0) {
            if (honor_abort && *reinterpret_cast<volatile unsigned*>(ctl.abort_flag)) return false;
            if (globaltimer_ns() - t0 > ctl.wait_ns) {
                atomicOr(ctl.err, code);
                atomicExch(ctl.abort_flag, 1u);
                return false;
            }
        }
    }
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const DevCtl& ctl, unsigned code,
                                          bool honor_abort = true, unsigned sleep_ns = 0) {
    if (mbar_try_wait(bar, parity)) return true;
    return mbar_wait_poll(bar, parity, ctl, code, honor_abort, sleep_ns);
}

// Generic-proxy shared-memory writes become visible to the async proxy (TMA, tcgen05.mma operands)
// once the writing thread executes this fence; a barrier or mbarrier then publishes them.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
// Named barrier over `threads` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------------------------ TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// 4-D tiled load into this CTA's shared memory, completing `bytes` on `bar`.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

// 4-D tiled store from this CTA's shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, uint32_t src, int c0, int c1, int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// The shared memory of every committed bulk store of this thread has been read.
__device__ __forceinline__ void bulk_wait_group_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Every committed bulk store of this thread has completed.
__device__ __forceinline__ void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// The MMA and commit helpers below are executed by a whole converged warp; one lane chosen by
// elect.sync inside the asm issues the instruction.  Keeping the issuing code warp-uniform (rather
// than branching on a lane index) lets it run on the uniform datapath: measured on B200 with eight
// softmax-like warps busy on the same SM, back-to-back 128x128x16 MMAs issued this way sustain
// 64 cycles each, against 88 when issued from inside an `if (lane == 0)` branch.

// Arrive once on `bar` when every tcgen05 async op issued so far by the issuing thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(
            smem_u32(bar))
        : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T-ish per the descriptors (kind::f16, fp32 accumulate).
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Load 32 consecutive 32-bit TMEM columns of this thread's lane and wait for
// them in the same asm block, so no use of the values can be scheduled
// before tcgen05.wait::ld.
__device__ __forceinline__ void tmem_ld32_sync(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

// Two x32 loads (64 columns) issued back to back, one wait.
__device__ __forceinline__ void tmem_ld64_sync(uint32_t taddr, uint32_t (&r)[64]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
        "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]),
          "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]),
          "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]),
          "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]),
          "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr), "r"(taddr + 32u)
        : "memory");
}

// 128 consecutive columns of this thread's lane (four x32 loads, one wait in the same asm block).
__device__ __forceinline__ void tmem_ld128_sync(uint32_t taddr, uint32_t (&r)[128]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%128];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%129];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95}, [%130];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%96,%97,%98,%99,%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,%112,%113,%114,%115,%116,%117,%118,%119,%120,%121,%122,%123,%124,%125,%126,%127}, [%131];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]),"=r"(r[1]),"=r"(r[2]),"=r"(r[3]),"=r"(r[4]),"=r"(r[5]),"=r"(r[6]),"=r"(r[7]),"=r"(r[8]),"=r"(r[9]),"=r"(r[10]),"=r"(r[11]),"=r"(r[12]),"=r"(r[13]),"=r"(r[14]),"=r"(r[15]),"=r"(r[16]),"=r"(r[17]),"=r"(r[18]),"=r"(r[19]),"=r"(r[20]),"=r"(r[21]),"=r"(r[22]),"=r"(r[23]),"=r"(r[24]),"=r"(r[25]),"=r"(r[26]),"=r"(r[27]),"=r"(r[28]),"=r"(r[29]),"=r"(r[30]),"=r"(r[31]),"=r"(r[32]),"=r"(r[33]),"=r"(r[34]),"=r"(r[35]),"=r"(r[36]),"=r"(r[37]),"=r"(r[38]),"=r"(r[39]),"=r"(r[40]),"=r"(r[41]),"=r"(r[42]),"=r"(r[43]),"=r"(r[44]),"=r"(r[45]),"=r"(r[46]),"=r"(r[47]),"=r"(r[48]),"=r"(r[49]),"=r"(r[50]),"=r"(r[51]),"=r"(r[52]),"=r"(r[53]),"=r"(r[54]),"=r"(r[55]),"=r"(r[56]),"=r"(r[57]),"=r"(r[58]),"=r"(r[59]),"=r"(r[60]),"=r"(r[61]),"=r"(r[62]),"=r"(r[63]),"=r"(r[64]),"=r"(r[65]),"=r"(r[66]),"=r"(r[67]),"=r"(r[68]),"=r"(r[69]),"=r"(r[70]),"=r"(r[71]),"=r"(r[72]),"=r"(r[73]),"=r"(r[74]),"=r"(r[75]),"=r"(r[76]),"=r"(r[77]),"=r"(r[78]),"=r"(r[79]),"=r"(r[80]),"=r"(r[81]),"=r"(r[82]),"=r"(r[83]),"=r"(r[84]),"=r"(r[85]),"=r"(r[86]),"=r"(r[87]),"=r"(r[88]),"=r"(r[89]),"=r"(r[90]),"=r"(r[91]),"=r"(r[92]),"=r"(r[93]),"=r"(r[94]),"=r"(r[95]),"=r"(r[96]),"=r"(r[97]),"=r"(r[98]),"=r"(r[99]),"=r"(r[100]),"=r"(r[101]),"=r"(r[102]),"=r"(r[103]),"=r"(r[104]),"=r"(r[105]),"=r"(r[106]),"=r"(r[107]),"=r"(r[108]),"=r"(r[109]),"=r"(r[110]),"=r"(r[111]),"=r"(r[112]),"=r"(r[113]),"=r"(r[114]),"=r"(r[115]),"=r"(r[116]),"=r"(r[117]),"=r"(r[118]),"=r"(r[119]),"=r"(r[120]),"=r"(r[121]),"=r"(r[122]),"=r"(r[123]),"=r"(r[124]),"=r"(r[125]),"=r"(r[126]),"=r"(r[127])
        : "r"(taddr), "r"(taddr + 32u), "r"(taddr + 64u), "r"(taddr + 96u)
        : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------------ descriptors
// Shared-memory matrix descriptor, SWIZZLE_128B, version 1 (sm_100):
//   bits [0,14)  start address >> 4      bits [16,30) leading byte offset >> 4
//   bits [32,46) stride byte offset >> 4 bits [46,48) version (1)
//   bits [49,52) base offset (0: tiles are 1024-byte aligned)
//   bits [61,64) layout: 2 = SWIZZLE_128B
// K-major (rows of 64 16-bit elements = 128 B, 8-row atoms 1024 B apart):
//   LBO unused by the hardware for swizzled K-major (set to 1), SBO = 1024.
// MN-major (the 64-element runs along M/N, K rows 128 B apart):
//   LBO = bytes between 64-element M/N blocks, SBO = bytes between 8-row K groups.
__host__ __device__ constexpr uint64_t make_sw128_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
__host__ __device__ constexpr uint64_t desc_k_sw128(uint32_t saddr) { return make_sw128_desc(saddr, 16, 1024); }
// The same descriptor as two words.  The low word holds the start address and the leading byte
// offset; the descriptors of the K-steps of one tile differ only in the start address, so an MMA
// loop builds the low word once and adds (byte offset >> 4) per step.  Shared-memory addresses
// stay below 2^18, so the 14-bit address field never carries into the LBO field.
__host__ __device__ constexpr uint32_t sw128_desc_lo(uint32_t saddr, uint32_t lbo_bytes) {
    return ((saddr >> 4) & 0x3FFFu) | (((lbo_bytes >> 4) & 0x3FFFu) << 16);
}
__host__ __device__ constexpr uint32_t sw128_desc_hi(uint32_t sbo_bytes) {
    return ((sbo_bytes >> 4) & 0x3FFFu) | (1u << 14) | (2u << 29);
}
__host__ __device__ constexpr uint64_t desc_join(uint32_t lo, uint32_t hi) { return ((uint64_t)hi << 32) | lo; }
static_assert(desc_join(sw128_desc_lo(0x1400u, 16) + (0x4020u >> 4), sw128_desc_hi(1024)) ==
                  make_sw128_desc(0x1400u + 0x4020u, 16, 1024),
              "split K-major descriptor");
static_assert(desc_join(sw128_desc_lo(0x31C00u, 16384) + (0x3800u >> 4), sw128_desc_hi(1024)) ==
                  make_sw128_desc(0x31C00u + 0x3800u, 16384, 1024),
              "split MN-major descriptor");
__host__ __device__ constexpr uint64_t desc_mn_sw128(uint32_t saddr, uint32_t lbo) {
    return make_sw128_desc(saddr, lbo, 1024);
}

// Instruction descriptor for tcgen05.mma kind::f16 with fp32 accumulation:
//   [4,6) D format (1 = f32)  [7,10) A format  [10,13) B format (0 = f16, 1 = bf16)
//   [15] A major (0 = K)  [16] B major (0 = K, 1 = MN)  [17,23) N >> 3  [24,29) M >> 4
__host__ __device__ constexpr uint32_t idesc_f16_f32acc(bool bf16, int M, int N, bool b_mn_major) {
    return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((b_mn_major ? 1u : 0u) << 16) |
           ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ------------------------------------------------------------------ math
// Packed pairs of f32 (sm_100 f32x2 arithmetic): one instruction for two independent
// round-to-nearest operations, bit-identical to the two scalar ones.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 2^x on the FMA/ALU pipes, used for part of the softmax exponentials so the MUFU
// unit is not the only exp2 engine.  Range split 2^x = 2^n * 2^f with n = rint(x)
// (add/subtract 1.5*2^23, which also leaves n in the low mantissa bits) and
// f in [-0.5, 0.5]; 2^f by a degree-3 polynomial whose coefficients were fitted
// for this library by a Remez exchange minimising the maximum relative error on
// [-0.5, 0.5] (7.5e-5 = 2^-13.7, far below the 2^-9 half-ulp of the bf16 P it
// feeds); n is added to the exponent field.  The argument is clamped at -126 so
// the exponent field cannot underflow (p in [0.70, 1.42] has field 126 or 127),
// and anything at or below -126 (including -inf scores) returns exactly 0.
__device__ __forceinline__ float exp2_poly(float x) {
    constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
    constexpr float c0 = 0.999928057f, c1 = 0.693260968f, c2 = 0.242611125f, c3 = 0.0551716685f;
    const float xc = fmaxf(x, -126.0f);
    const float t = xc + kShift;
    const float f = xc - (t - kShift);
    const float p = fmaf(fmaf(fmaf(c3, f, c2), f, c1), f, c0);
    const float r = __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
    return x > -126.0f ? r : 0.0f;
}

// Two exp2_poly evaluations with packed f32x2 arithmetic: the same clamp, range split, polynomial and
// exponent insertion, each f32x2 operation bit-identical to the two scalar ones -- so the results equal
// exp2_poly(xa), exp2_poly(xb) exactly, in about two thirds of the issue slots.
__device__ __forceinline__ void exp2_poly2(float xa, float xb, float& ya, float& yb) {
    constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
    const uint64_t xc = f2_pack(fmaxf(xa, -126.0f), fmaxf(xb, -126.0f));
    const uint64_t sh = f2_pack(kShift, kShift);
    const uint64_t t = add_f32x2(xc, sh);
    const uint64_t n = add_f32x2(t, f2_pack(-kShift, -kShift));      // t - shift, exact
    const uint64_t f = fma_f32x2(n, f2_pack(-1.0f, -1.0f), xc);       // xc - (t - shift), one rounding
    uint64_t q = fma_f32x2(f2_pack(0.0551716685f, 0.0551716685f), f, f2_pack(0.242611125f, 0.242611125f));
    q = fma_f32x2(q, f, f2_pack(0.693260968f, 0.693260968f));
    q = fma_f32x2(q, f, f2_pack(0.999928057f, 0.999928057f));
    float pa, pb, ta, tb;
    f2_unpack(q, pa, pb);
    f2_unpack(t, ta, tb);
    const float ra = __int_as_float(__float_as_int(pa) + (__float_as_int(ta) << 23));
    const float rb = __int_as_float(__float_as_int(pb) + (__float_as_int(tb) << 23));
    ya = xa > -126.0f ? ra : 0.0f;
    yb = xb > -126.0f ? rb : 0.0f;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

template <typename T>
struct Pack2;
template <>
struct Pack2<__nv_bfloat16> {
    static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
        __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&v);
    }
};
template <>
struct Pack2<__half> {
    static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
        __half2 v = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&v);
    }
};

}  // namespace kd
