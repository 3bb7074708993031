// The C++ host layer (kandinsky.cpp_b200/host/kd_ops.hpp) against the CPU oracle (oracle/kd_oracle.c,
// test infrastructure), on seeded inputs:
//   kd::ops::attention      -- plain flash branch, grouped-query heads, an f16 mask
//   kd::dit_self_attention  -- RMSNorm (non-unit gains) + 3D RoPE + flash
//   kd::dit_cross_attention -- RMSNorm + flash over text states with per-sequence valid lengths
//   kd::ops::linear         -- f16 weight + bias against a double-precision product
//   kd::dit_self_attention_block -- Linears + RMSNorm + RoPE + flash + out_layer against the oracle's
//                              pieces composed on the CPU (operands rounded to bf16 where the GPU rounds)
// and the error behaviour of ops::attention (false + a logged reason, nothing launched).
// Gates: cosine >= 0.99995 and max-abs <= 2e-2 x output RMS against the oracle's fp64 mode.
// `--cpu` checks only the host-side pieces (tensor views, constants, no-device failure).
// Prints "OK" and exits 0 on success.  Built and run by tests/test_host_cpp.py.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

#include "kd_ops.hpp"
#include "kd_oracle.h"

static int g_fail = 0;
#define CHECK(cond, ...)                                  \
    do {                                                  \
        if (!(cond)) {                                    \
            printf("FAIL %s:%d: ", __FILE__, __LINE__);   \
            printf(__VA_ARGS__);                          \
            printf("\n");                                 \
            ++g_fail;                                     \
        }                                                 \
    } while (0)

static std::vector<float> randn(uint64_t seed, uint32_t offset, size_t n) {
    std::vector<float> v(n);
    kdo_philox_randn(seed, offset, n, v.data(), 4);
    return v;
}

static kdo_tensor head_view(const void* data, int32_t type, int64_t L, int64_t H, int64_t N) {
    // [C = H*128, L, N] seen as [128, L, H, N]
    const int64_t es = type == KDO_F32 ? 4 : 2;
    kdo_tensor t{};
    t.data = data;
    t.type = type;
    t.ne[0] = 128; t.ne[1] = L; t.ne[2] = H; t.ne[3] = N;
    t.nb[0] = es; t.nb[1] = es * 128 * H; t.nb[2] = es * 128; t.nb[3] = es * 128 * H * L;
    return t;
}

static void gates(const char* what, const std::vector<float>& got, const std::vector<float>& ref) {
    double dot = 0, ng = 0, nr = 0, maxabs = 0, ss = 0;
    for (size_t i = 0; i < ref.size(); ++i) {
        dot += (double)got[i] * ref[i];
        ng += (double)got[i] * got[i];
        nr += (double)ref[i] * ref[i];
        maxabs = std::fmax(maxabs, std::fabs((double)got[i] - ref[i]));
        ss += (double)ref[i] * ref[i];
    }
    const double cos = dot / std::sqrt(ng * nr + 1e-300), rms = std::sqrt(ss / ref.size());
    printf("%-24s cos %.7f  maxabs/rms %.3e\n", what, cos, maxabs / rms);
    CHECK(cos >= 0.99995, "%s cosine %.7f", what, cos);
    CHECK(maxabs <= 2e-2 * rms, "%s max-abs %.3e > 2e-2 x rms %.3e", what, maxabs, rms);
}

struct Dev {
    void* p = nullptr;
    explicit Dev(size_t bytes) { cudaMalloc(&p, bytes); }
    ~Dev() { cudaFree(p); }
};

static void* upload(Dev& d, const void* src, size_t bytes) {
    cudaMemcpy(d.p, src, bytes, cudaMemcpyHostToDevice);
    return d.p;
}

static int cpu_checks() {
    float dummy;
    kd::Tensor t = kd::Tensor::contiguous(&dummy, KD_ATTN_TYPE_F16, 128, 7, 3, 2);
    CHECK(t.nb[0] == 2 && t.nb[1] == 256 && t.nb[2] == 256 * 7 && t.nb[3] == 256 * 21, "contiguous strides");
    CHECK(t.bytes() == 256u * 42u, "bytes");
    const kd_tensor v = t.view();
    CHECK(v.data == &dummy && v.type == KD_ATTN_TYPE_F16 && v.ne[1] == 7 && v.nb[3] == t.nb[3], "view");
    const kd::CrossDiTAttentionConfig c = kd::CrossDiTAttentionConfig::pro_video();
    CHECK(c.head_dim == 128 && c.axes_dims[0] + c.axes_dims[1] + c.axes_dims[2] == 128 && c.rope_theta == 10000.f &&
              c.scale_factor[1] == 2.f && c.norm_eps == 1e-6f,
          "pro_video constants");
    return 0;
}

// bf16 rounding of each element (the GEMM's operand type), kept as f32
static std::vector<float> bf16_round(const std::vector<float>& a) {
    std::vector<uint16_t> b(a.size());
    std::vector<float> r(a.size());
    kdo_convert(a.data(), (int64_t)a.size(), KDO_BF16, b.data());
    kdo_to_f32(b.data(), KDO_BF16, (int64_t)b.size(), r.data());
    return r;
}

// y[m][c] = sum_k x[m][k] w[c][k] + b[c] in double, rounded to f32 (ops::linear on the CPU)
static std::vector<float> cpu_linear(const std::vector<float>& x, const std::vector<float>& w, const float* b,
                                     int64_t M, int64_t K, int64_t C) {
    std::vector<float> y((size_t)M * C);
    for (int64_t m = 0; m < M; ++m)
        for (int64_t c = 0; c < C; ++c) {
            double acc = b ? b[c] : 0.0;
            for (int64_t k = 0; k < K; ++k) acc += (double)x[m * K + k] * w[c * K + k];
            y[m * C + c] = (float)acc;
        }
    return y;
}

int main(int argc, char** argv) {
    const bool cpu_only = argc > 1 && strcmp(argv[1], "--cpu") == 0;
    cpu_checks();
    if (cpu_only) {
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
            cudaGetLastError();
            kd::Context ctx(0);  // no device: creation fails cleanly, every call returns false
            CHECK(!ctx.ok() && ctx.create_status() != KD_ATTN_OK, "context without a device");
            kd::Tensor x;
            CHECK(!kd::ops::attention(ctx, x, x, x, 4, x), "call on a failed context");
        }
        printf(g_fail ? "FAILED\n" : "OK\n");
        return g_fail ? 1 : 0;
    }

    kd::Context ctx(0);
    if (!ctx.ok()) {
        printf("FAIL: kd_attn_create: status %d\n", (int)ctx.create_status());
        return 1;
    }

    // ---- ops::attention: GQA 4:2, f16 operands, an f16 mask with -inf blocks, f32 output
    {
        const int64_t N = 2, H = 4, Hkv = 2, Lq = 200, Lk = 300, C = H * 128, Ckv = Hkv * 128;
        std::vector<float> q = randn(11, 0, N * Lq * C), k = randn(11, 1, N * Lk * Ckv), v = randn(11, 2, N * Lk * Ckv);
        std::vector<uint16_t> mask((size_t)Lq * Lk);
        for (int64_t i = 0; i < Lq; ++i)
            for (int64_t j = 0; j < Lk; ++j)
                mask[i * Lk + j] = (((i / 64) + (j / 64)) % 3 == 1 && j > 10) ? 0xFC00u : kdo_f32_to_f16(0.25f * (float)((i + j) % 5) - 0.5f);
        Dev dq(q.size() * 4), dk(k.size() * 4), dv(v.size() * 4), dm(mask.size() * 2), dout(N * Lq * C * 4);
        kd::Tensor tq = kd::Tensor::contiguous(upload(dq, q.data(), q.size() * 4), KD_ATTN_TYPE_F32, C, Lq, N);
        kd::Tensor tk = kd::Tensor::contiguous(upload(dk, k.data(), k.size() * 4), KD_ATTN_TYPE_F32, Ckv, Lk, N);
        kd::Tensor tv = kd::Tensor::contiguous(upload(dv, v.data(), v.size() * 4), KD_ATTN_TYPE_F32, Ckv, Lk, N);
        kd::Tensor tm = kd::Tensor::contiguous(upload(dm, mask.data(), mask.size() * 2), KD_ATTN_TYPE_F16, Lk, Lq, 1, 1);
        kd::Tensor to = kd::Tensor::contiguous(dout.p, KD_ATTN_TYPE_F32, C, Lq, N);
        const bool ok = kd::ops::attention(ctx, tq, tk, tv, H, to, &tm, true, false, KD_ATTN_TYPE_F16);
        CHECK(ok && ctx.device_status(), "ops::attention: %s", ctx.last_error().c_str());
        std::vector<float> got(N * Lq * C);
        cudaMemcpy(got.data(), dout.p, got.size() * 4, cudaMemcpyDeviceToHost);
        std::vector<uint16_t> k16(k.size()), v16(v.size());
        kdo_convert(k.data(), (int64_t)k.size(), KDO_F16, k16.data());
        kdo_convert(v.data(), (int64_t)v.size(), KDO_F16, v16.data());
        const kdo_tensor oq = head_view(q.data(), KDO_F32, Lq, H, N), ok16 = head_view(k16.data(), KDO_F16, Lk, Hkv, N),
                         ov16 = head_view(v16.data(), KDO_F16, Lk, Hkv, N);
        kdo_tensor om{};
        om.data = mask.data();
        om.type = KDO_F16;
        om.ne[0] = Lk; om.ne[1] = Lq; om.ne[2] = 1; om.ne[3] = 1;
        om.nb[0] = 2; om.nb[1] = 2 * Lk; om.nb[2] = 2 * Lk * Lq; om.nb[3] = om.nb[2];
        std::vector<float> ref(N * Lq * C);
        const int rc = kdo_flash_attn_ext(&oq, &ok16, &ov16, &om, 1.0f / std::sqrt(128.0f), nullptr, KDO_MODE_EXACT,
                                          ref.data(), nullptr, 8);
        CHECK(rc == 0, "oracle rc %d", rc);
        gates("ops::attention GQA+mask", got, ref);
        // invalid GQA ratio (3 query heads over 2 K/V heads): false, nothing launched
        kd::Tensor tq3 = kd::Tensor::contiguous(dq.p, KD_ATTN_TYPE_F32, 3 * 128, Lq, N);
        kd::Tensor to3 = kd::Tensor::contiguous(dout.p, KD_ATTN_TYPE_F32, 3 * 128, Lq, N);
        CHECK(!kd::ops::attention(ctx, tq3, tk, tv, 3, to3), "invalid GQA ratio accepted");
        CHECK(ctx.last_error().find("GQA") != std::string::npos, "GQA error text: %s", ctx.last_error().c_str());
        CHECK(!kd::ops::attention(ctx, tq, tk, tv, H, to, nullptr, true, /*causal=*/true), "causal accepted");
    }

    // ---- dit_self_attention: RMSNorm with gains + 3D RoPE ({1,2,2} scale) + flash, bf16 operands
    {
        const int64_t N = 2, H = 3, C = H * 128;
        const int32_t grid[3] = {2, 8, 12};
        const int64_t L = grid[0] * grid[1] * grid[2];
        std::vector<float> q = randn(21, 0, N * L * C), k = randn(21, 1, N * L * C), v = randn(21, 2, N * L * C);
        std::vector<float> gq(128), gk(128);
        for (int i = 0; i < 128; ++i) {
            gq[i] = 0.5f + (float)i / 128.0f;
            gk[i] = 1.5f - (float)i / 256.0f;
        }
        Dev dq(q.size() * 4), dk(k.size() * 4), dv(v.size() * 4), dgq(512), dgk(512), dout(N * L * C * 2);
        kd::Tensor tq = kd::Tensor::contiguous(upload(dq, q.data(), q.size() * 4), KD_ATTN_TYPE_F32, C, L, N);
        kd::Tensor tk = kd::Tensor::contiguous(upload(dk, k.data(), k.size() * 4), KD_ATTN_TYPE_F32, C, L, N);
        kd::Tensor tv = kd::Tensor::contiguous(upload(dv, v.data(), v.size() * 4), KD_ATTN_TYPE_F32, C, L, N);
        upload(dgq, gq.data(), 512);
        upload(dgk, gk.data(), 512);
        kd::Tensor to = kd::Tensor::contiguous(dout.p, KD_ATTN_TYPE_BF16, C, L, N);
        const kd::CrossDiTAttentionConfig cfg = kd::CrossDiTAttentionConfig::pro_video();
        const bool ok = kd::dit_self_attention(ctx, tq, tk, tv, H, (const float*)dgq.p, (const float*)dgk.p, grid, cfg, to);
        CHECK(ok && ctx.device_status(), "dit_self_attention: %s", ctx.last_error().c_str());
        std::vector<uint16_t> got16(N * L * C);
        cudaMemcpy(got16.data(), dout.p, got16.size() * 2, cudaMemcpyDeviceToHost);
        std::vector<float> got(got16.size());
        kdo_to_f32(got16.data(), KDO_BF16, (int64_t)got16.size(), got.data());
        // oracle: rms_norm -> rope -> round to bf16 -> flash (fp64)
        std::vector<float> qn(q.size()), kn(k.size()), table((size_t)L * 128);
        kdo_rms_norm_heads(q.data(), N * L * H, 128, gq.data(), cfg.norm_eps, qn.data(), 8);
        kdo_rms_norm_heads(k.data(), N * L * H, 128, gk.data(), cfg.norm_eps, kn.data(), 8);
        kdo_visual_rope_table(grid[0], grid[1], grid[2], cfg.axes_dims, cfg.scale_factor, cfg.rope_theta, table.data());
        kdo_rope_apply(qn.data(), L, N, (int)H, 128, table.data(), 8);
        kdo_rope_apply(kn.data(), L, N, (int)H, 128, table.data(), 8);
        std::vector<uint16_t> q16(q.size()), k16(k.size()), v16(v.size());
        kdo_convert(qn.data(), (int64_t)q.size(), KDO_BF16, q16.data());
        kdo_convert(kn.data(), (int64_t)k.size(), KDO_BF16, k16.data());
        kdo_convert(v.data(), (int64_t)v.size(), KDO_BF16, v16.data());
        const kdo_tensor oq = head_view(q16.data(), KDO_BF16, L, H, N), okk = head_view(k16.data(), KDO_BF16, L, H, N),
                         ovv = head_view(v16.data(), KDO_BF16, L, H, N);
        std::vector<float> ref(N * L * C);
        const int rc = kdo_flash_attn_ext(&oq, &okk, &ovv, nullptr, 1.0f / std::sqrt(128.0f), nullptr, KDO_MODE_EXACT,
                                          ref.data(), nullptr, 8);
        CHECK(rc == 0, "oracle rc %d", rc);
        gates("dit_self_attention", got, ref);
    }

    // ---- dit_cross_attention: RMSNorm, no RoPE, text states of 77 tokens, valid lengths {77, 40}
    {
        const int64_t N = 2, H = 2, Lq = 256, Lt = 77, C = H * 128;
        std::vector<float> q = randn(31, 0, N * Lq * C), k = randn(31, 1, N * Lt * C), v = randn(31, 2, N * Lt * C);
        const int32_t kv_len[2] = {77, 40};
        Dev dq(q.size() * 4), dk(k.size() * 4), dv(v.size() * 4), dl(8), dout(N * Lq * C * 4);
        kd::Tensor tq = kd::Tensor::contiguous(upload(dq, q.data(), q.size() * 4), KD_ATTN_TYPE_F32, C, Lq, N);
        kd::Tensor tk = kd::Tensor::contiguous(upload(dk, k.data(), k.size() * 4), KD_ATTN_TYPE_F32, C, Lt, N);
        kd::Tensor tv = kd::Tensor::contiguous(upload(dv, v.data(), v.size() * 4), KD_ATTN_TYPE_F32, C, Lt, N);
        upload(dl, kv_len, 8);
        kd::Tensor to = kd::Tensor::contiguous(dout.p, KD_ATTN_TYPE_F32, C, Lq, N);
        const kd::CrossDiTAttentionConfig cfg = kd::CrossDiTAttentionConfig::pro_video();
        const bool ok = kd::dit_cross_attention(ctx, tq, tk, tv, H, nullptr, nullptr, (const int32_t*)dl.p, nullptr, cfg, to);
        CHECK(ok && ctx.device_status(), "dit_cross_attention: %s", ctx.last_error().c_str());
        std::vector<float> got(N * Lq * C);
        cudaMemcpy(got.data(), dout.p, got.size() * 4, cudaMemcpyDeviceToHost);
        std::vector<float> qn(q.size()), kn(k.size());
        kdo_rms_norm_heads(q.data(), N * Lq * H, 128, nullptr, cfg.norm_eps, qn.data(), 8);
        kdo_rms_norm_heads(k.data(), N * Lt * H, 128, nullptr, cfg.norm_eps, kn.data(), 8);
        std::vector<uint16_t> q16(q.size()), k16(k.size()), v16(v.size());
        kdo_convert(qn.data(), (int64_t)q.size(), KDO_BF16, q16.data());
        kdo_convert(kn.data(), (int64_t)k.size(), KDO_BF16, k16.data());
        kdo_convert(v.data(), (int64_t)v.size(), KDO_BF16, v16.data());
        const kdo_tensor oq = head_view(q16.data(), KDO_BF16, Lq, H, N), okk = head_view(k16.data(), KDO_BF16, Lt, H, N),
                         ovv = head_view(v16.data(), KDO_BF16, Lt, H, N);
        std::vector<float> ref(N * Lq * C);
        const int rc = kdo_flash_attn_ext(&oq, &okk, &ovv, nullptr, 1.0f / std::sqrt(128.0f), kv_len, KDO_MODE_EXACT,
                                          ref.data(), nullptr, 8);
        CHECK(rc == 0, "oracle rc %d", rc);
        gates("dit_cross_attention", got, ref);
    }

    // ---- ops::linear: f32 x [256, 100, 2], f16 weight [256 -> 512] with bias, f32 y
    {
        const int64_t N = 2, L = 100, K = 256, C = 512, M = N * L;
        std::vector<float> x = randn(41, 0, M * K), w = randn(41, 1, C * K), b = randn(41, 2, C);
        for (float& e : w) e *= 0.0625f;
        std::vector<uint16_t> w16(w.size());
        kdo_convert(w.data(), (int64_t)w.size(), KDO_F16, w16.data());
        std::vector<float> wf(w.size());
        kdo_to_f32(w16.data(), KDO_F16, (int64_t)w16.size(), wf.data());
        Dev dx(x.size() * 4), dw(w16.size() * 2), db(b.size() * 4), dy(M * C * 4);
        kd::Tensor tx = kd::Tensor::contiguous(upload(dx, x.data(), x.size() * 4), KD_ATTN_TYPE_F32, K, L, N);
        kd::Linear lin;
        lin.weight = upload(dw, w16.data(), w16.size() * 2);
        lin.type = KD_ATTN_TYPE_F16;
        lin.in_features = K;
        lin.out_features = C;
        lin.nb1 = (size_t)K * 2;
        lin.bias = (const float*)upload(db, b.data(), b.size() * 4);
        kd::Tensor ty = kd::Tensor::contiguous(dy.p, KD_ATTN_TYPE_F32, C, L, N);
        const bool ok = kd::ops::linear(ctx, tx, lin, ty);
        CHECK(ok && ctx.device_status(), "ops::linear: %s", ctx.last_error().c_str());
        std::vector<float> got(M * C);
        cudaMemcpy(got.data(), dy.p, got.size() * 4, cudaMemcpyDeviceToHost);
        gates("ops::linear", got, cpu_linear(bf16_round(x), bf16_round(wf), b.data(), M, K, C));
        kd::Linear bad = lin;
        bad.out_features = 320;  // not a multiple of 256
        CHECK(!kd::ops::linear(ctx, tx, bad, ty), "out_features 320 accepted");
    }

    // ---- dit_self_attention_block: x [256, 64, 1] -> Linears (f16) -> RMSNorm + RoPE -> flash -> out_layer
    {
        const int64_t N = 1, H = 2, C = H * 128;
        const int32_t grid[3] = {2, 4, 8};
        const int64_t L = grid[0] * grid[1] * grid[2], M = N * L;
        std::vector<float> x = randn(51, 0, M * C);
        std::vector<float> wf[4], bias[4];
        std::vector<uint16_t> w16[4];
        Dev dw0(C * C * 2), dw1(C * C * 2), dw2(C * C * 2), dw3(C * C * 2), db0(C * 4), db1(C * 4), db2(C * 4),
            db3(C * 4);
        Dev* dws[4] = {&dw0, &dw1, &dw2, &dw3};
        Dev* dbs[4] = {&db0, &db1, &db2, &db3};
        kd::Linear lin[4];
        for (int i = 0; i < 4; ++i) {
            std::vector<float> w = randn(52, (uint32_t)i, C * C);
            for (float& e : w) e *= 0.0625f;
            w16[i].resize(w.size());
            kdo_convert(w.data(), (int64_t)w.size(), KDO_F16, w16[i].data());
            wf[i].resize(w.size());
            kdo_to_f32(w16[i].data(), KDO_F16, (int64_t)w.size(), wf[i].data());
            bias[i] = randn(53, (uint32_t)i, C);
            lin[i].weight = upload(*dws[i], w16[i].data(), w16[i].size() * 2);
            lin[i].type = KD_ATTN_TYPE_F16;
            lin[i].in_features = C;
            lin[i].out_features = C;
            lin[i].nb1 = (size_t)C * 2;
            lin[i].bias = (const float*)upload(*dbs[i], bias[i].data(), C * 4);
        }
        std::vector<float> gq(128), gk(128);
        for (int i = 0; i < 128; ++i) {
            gq[i] = 0.75f + (float)i / 256.0f;
            gk[i] = 1.25f - (float)i / 512.0f;
        }
        Dev dx(x.size() * 4), dgq(512), dgk(512), dy(M * C * 4);
        upload(dgq, gq.data(), 512);
        upload(dgk, gk.data(), 512);
        kd::Tensor tx = kd::Tensor::contiguous(upload(dx, x.data(), x.size() * 4), KD_ATTN_TYPE_F32, C, L, N);
        kd::Tensor ty = kd::Tensor::contiguous(dy.p, KD_ATTN_TYPE_F32, C, L, N);
        const kd::CrossDiTAttentionConfig cfg = kd::CrossDiTAttentionConfig::pro_video();
        const bool ok = kd::dit_self_attention_block(ctx, tx, lin[0], lin[1], lin[2], lin[3], (const float*)dgq.p,
                                                     (const float*)dgk.p, grid, cfg, ty);
        CHECK(ok && ctx.device_status(), "dit_self_attention_block: %s", ctx.last_error().c_str());
        std::vector<float> got(M * C);
        cudaMemcpy(got.data(), dy.p, got.size() * 4, cudaMemcpyDeviceToHost);
        // CPU: bf16 x and weights -> projections -> RMSNorm -> RoPE -> bf16 operands -> flash (fp64)
        //      -> bf16 attention output -> out_layer with bf16 weight
        const std::vector<float> xr = bf16_round(x);
        std::vector<float> q = cpu_linear(xr, bf16_round(wf[0]), bias[0].data(), M, C, C);
        std::vector<float> k = cpu_linear(xr, bf16_round(wf[1]), bias[1].data(), M, C, C);
        std::vector<float> v = cpu_linear(xr, bf16_round(wf[2]), bias[2].data(), M, C, C);
        std::vector<float> qn(q.size()), kn(k.size()), table((size_t)L * 128);
        kdo_rms_norm_heads(q.data(), M * H, 128, gq.data(), cfg.norm_eps, qn.data(), 8);
        kdo_rms_norm_heads(k.data(), M * H, 128, gk.data(), cfg.norm_eps, kn.data(), 8);
        kdo_visual_rope_table(grid[0], grid[1], grid[2], cfg.axes_dims, cfg.scale_factor, cfg.rope_theta, table.data());
        kdo_rope_apply(qn.data(), L, N, (int)H, 128, table.data(), 8);
        kdo_rope_apply(kn.data(), L, N, (int)H, 128, table.data(), 8);
        std::vector<uint16_t> q16(q.size()), k16(k.size()), v16(v.size());
        kdo_convert(qn.data(), (int64_t)q.size(), KDO_BF16, q16.data());
        kdo_convert(kn.data(), (int64_t)k.size(), KDO_BF16, k16.data());
        kdo_convert(v.data(), (int64_t)v.size(), KDO_BF16, v16.data());
        const kdo_tensor oq = head_view(q16.data(), KDO_BF16, L, H, N), okk = head_view(k16.data(), KDO_BF16, L, H, N),
                         ovv = head_view(v16.data(), KDO_BF16, L, H, N);
        std::vector<float> attn(M * C);
        const int rc = kdo_flash_attn_ext(&oq, &okk, &ovv, nullptr, 1.0f / std::sqrt(128.0f), nullptr, KDO_MODE_EXACT,
                                          attn.data(), nullptr, 8);
        CHECK(rc == 0, "oracle rc %d", rc);
        gates("dit_self_attention_block", got, cpu_linear(bf16_round(attn), bf16_round(wf[3]), bias[3].data(), M, C, C));
    }

    printf(g_fail ? "FAILED\n" : "OK\n");
    return g_fail ? 1 : 0;
}
