// Host-only check: libkd_attn's tcgen05 descriptor encoders (kd_common.cuh)
// against CUTLASS's definitions of the same bit fields
// (cute::UMMA::SmemDescriptor, cute::UMMA::make_instr_desc).
// Prints "OK" or the first mismatch.  Built and run by tests/test_descriptors.py.
#include <cstdio>
#include <cute/arch/mma_sm100_desc.hpp>
#include <cute/numeric/numeric_types.hpp>

#include "kd_common.cuh"

using namespace cute;

static int check_smem(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    UMMA::SmemDescriptor d;
    d.desc_ = 0;
    d.version_ = 1;
    d.lbo_mode_ = 0;
    d.layout_type_ = uint8_t(UMMA::LayoutType::SWIZZLE_128B);
    d.start_address_ = uint16_t(addr >> 4);
    d.base_offset_ = 0;
    d.leading_byte_offset_ = uint16_t(lbo >> 4);
    d.stride_byte_offset_ = uint16_t(sbo >> 4);
    uint64_t mine = kd::make_sw128_desc(addr, lbo, sbo);
    if (mine != d.desc_) {
        printf("smem desc mismatch addr=%u lbo=%u sbo=%u mine=%016llx cutlass=%016llx\n", addr, lbo, sbo,
               (unsigned long long)mine, (unsigned long long)d.desc_);
        return 1;
    }
    return 0;
}

template <class T>
static int check_idesc(bool bf16, int M, int N, bool b_mn) {
    uint32_t ref;
    if (b_mn) ref = uint32_t(UMMA::make_instr_desc<T, T, float, 128, 128, UMMA::Major::K, UMMA::Major::MN>());
    else      ref = uint32_t(UMMA::make_instr_desc<T, T, float, 128, 128, UMMA::Major::K, UMMA::Major::K>());
    uint32_t mine = kd::idesc_f16_f32acc(bf16, M, N, b_mn);
    if (mine != ref) {
        printf("instr desc mismatch bf16=%d b_mn=%d mine=%08x cutlass=%08x\n", (int)bf16, (int)b_mn, mine, ref);
        return 1;
    }
    return 0;
}

int main() {
    int bad = 0;
    for (uint32_t addr : {0u, 1024u, 33792u, 65536u + 96u, 200704u + 32u})
        bad += check_smem(addr, 16, 1024) + check_smem(addr, 16384, 1024);
    // the K-major helper must be exactly LBO 16 (encoded 1), SBO 1024
    if (kd::desc_k_sw128(4096) != kd::make_sw128_desc(4096, 16, 1024)) { printf("desc_k_sw128\n"); bad++; }
    if (kd::desc_mn_sw128(4096, 16384) != kd::make_sw128_desc(4096, 16384, 1024)) { printf("desc_mn_sw128\n"); bad++; }
    bad += check_idesc<bfloat16_t>(true, 128, 128, false);
    bad += check_idesc<bfloat16_t>(true, 128, 128, true);
    bad += check_idesc<half_t>(false, 128, 128, false);
    bad += check_idesc<half_t>(false, 128, 128, true);
    if (!bad) printf("OK\n");
    return bad ? 1 : 0;
}
