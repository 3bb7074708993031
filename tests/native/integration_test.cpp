// CPU test of integration/ (the ggml-side shim): compiled against the declarations-only ggml stub
// with a fake ggml graph builder (records custom nodes) and a fake libkd_attn (records every call
// and returns a chosen status), so it needs neither ggml nor a GPU.  Checks the ggml_tensor ->
// kd_tensor mapping, the build-time fallback to the reference's ops::attention wherever
// libkd_attn would not take the call (the role of ggml_backend_supports_op at ops.hpp:179-181),
// the node callbacks' library calls, and the batch-2 pairing of the two CFG halves.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "ggml.h"
#include "kd_attn.h"

// ------------------------------------------------------------------ fake ggml graph builder
struct ggml_context {};
static std::vector<ggml_tensor*> g_nodes;
static std::vector<ggml_custom_op_t> g_funs;
static std::vector<void*> g_user;

extern "C" ggml_tensor* ggml_custom_4d(ggml_context*, enum ggml_type type, int64_t ne0, int64_t ne1, int64_t ne2,
                                       int64_t ne3, ggml_tensor** args, int n_args, ggml_custom_op_t fun, int,
                                       void* userdata) {
    ggml_tensor* t = new ggml_tensor();
    t->type = type;
    t->ne[0] = ne0; t->ne[1] = ne1; t->ne[2] = ne2; t->ne[3] = ne3;
    t->nb[0] = 4;
    for (int i = 1; i < 4; ++i) t->nb[i] = t->nb[i - 1] * (size_t)t->ne[i - 1];
    for (int i = 0; i < n_args; ++i) t->src[i] = args[i];
    t->data = reinterpret_cast<void*>(0x7000000);  // where the backend would have placed it
    g_nodes.push_back(t);
    g_funs.push_back(fun);
    g_user.push_back(userdata);
    return t;
}
extern "C" int64_t ggml_nelements(const ggml_tensor* t) { return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]; }

// the reference's ops::attention (src/core/ops.hpp:107): here only a recorder
static int g_reference_calls = 0;
static ggml_tensor g_reference_result;
namespace ops {
inline ggml_tensor* attention(ggml_context*, ggml_backend_t, ggml_tensor*, ggml_tensor*, ggml_tensor*, int64_t,
                              ggml_tensor* = nullptr, bool = false, bool = false) {
    ++g_reference_calls;
    return &g_reference_result;
}
}  // namespace ops

// ------------------------------------------------------------------ fake libkd_attn
struct Call {
    const char* fn = nullptr;
    kd_tensor q{}, k{}, v{}, m{}, o{};
    bool has_mask = false;
    int32_t n_head = 0, op_type = -1;
    const float* qg = nullptr;
    const float* kg = nullptr;
    const kd_rope3d* rope = nullptr;
};
static std::vector<Call> g_calls;
static kd_attn_status g_status = KD_ATTN_OK;
extern "C" {
kd_attn_status kd_attn_attention(kd_attn_ctx*, const kd_tensor* q, const kd_tensor* k, const kd_tensor* v,
                                 int32_t n_head, const kd_tensor* mask, int32_t op_type, kd_tensor* out, float*,
                                 void*) {
    Call c;
    c.fn = "attention"; c.q = *q; c.k = *k; c.v = *v; c.o = *out; c.n_head = n_head; c.op_type = op_type;
    if (mask) { c.m = *mask; c.has_mask = true; }
    g_calls.push_back(c);
    return g_status;
}
kd_attn_status kd_attn_self_attention(kd_attn_ctx*, const kd_tensor* q, const kd_tensor* k, const kd_tensor* v,
                                      int32_t n_head, const float* qg, const float* kg, float, const kd_rope3d* rope,
                                      int32_t op_type, kd_tensor* out, float*, void*) {
    Call c;
    c.fn = "self_attention"; c.q = *q; c.k = *k; c.v = *v; c.o = *out; c.n_head = n_head; c.op_type = op_type;
    c.qg = qg; c.kg = kg; c.rope = rope;
    g_calls.push_back(c);
    return g_status;
}
static kd_linear g_block_w[4];
static kd_tensor g_block_x, g_block_y;
kd_attn_status kd_attn_self_attention_block(kd_attn_ctx*, const kd_tensor* x, const kd_linear* wq, const kd_linear* wk,
                                            const kd_linear* wv, const kd_linear* wo, int32_t n_head, const float* qg,
                                            const float* kg, float, const kd_rope3d* rope, kd_tensor* y, void*) {
    Call c;
    c.fn = "self_attention_block"; c.n_head = n_head; c.qg = qg; c.kg = kg; c.rope = rope;
    g_block_x = *x; g_block_y = *y;
    g_block_w[0] = *wq; g_block_w[1] = *wk; g_block_w[2] = *wv; g_block_w[3] = *wo;
    g_calls.push_back(c);
    return g_status;
}
const char* kd_attn_last_error(const kd_attn_ctx*) { return "fake"; }
}

#include "ops_attention_kd.hpp"

// ------------------------------------------------------------------ helpers
static int g_fail = 0;
#define CHECK(c)                                                          \
    do {                                                                  \
        if (!(c)) {                                                       \
            fprintf(stderr, "%s:%d: CHECK failed: %s\n", __FILE__, __LINE__, #c); \
            ++g_fail;                                                     \
        }                                                                 \
    } while (0)

static ggml_tensor make(enum ggml_type type, int64_t ne0, int64_t ne1, int64_t ne2, uintptr_t addr) {
    ggml_tensor t{};
    t.type = type;
    t.ne[0] = ne0; t.ne[1] = ne1; t.ne[2] = ne2; t.ne[3] = 1;
    t.nb[0] = type == GGML_TYPE_F32 ? 4 : 2;
    for (int i = 1; i < 4; ++i) t.nb[i] = t.nb[i - 1] * (size_t)t.ne[i - 1];
    t.data = reinterpret_cast<void*>(addr);
    return t;
}
static bool same(const kd_tensor& a, const ggml_tensor& g, int32_t type) {
    if (a.data != g.data || a.type != type) return false;
    for (int i = 0; i < 4; ++i)
        if (a.ne[i] != g.ne[i] || a.nb[i] != g.nb[i]) return false;
    return true;
}

int main() {
    ggml_context gctx;
    kd_attn_ctx* fake_ctx = reinterpret_cast<kd_attn_ctx*>(0x10);
    const int64_t C = 4096, L = 1280, N = 1, H = 32;

    // 1. type and layout mapping (ne/nb/data field by field, ggml type ids)
    {
        ggml_tensor t = make(GGML_TYPE_BF16, 128, 7, 3, 0x1000);
        t.nb[2] = 4096;  // a gapped stride survives the mapping
        kd_tensor k{};
        CHECK(kd_bridge::kd_from_ggml(&t, &k) && same(k, t, KD_ATTN_TYPE_BF16));
        ggml_tensor q8 = make(GGML_TYPE_Q8_0, 128, 7, 3, 0x1000);
        CHECK(!kd_bridge::kd_from_ggml(&q8, &k));
    }
    ggml_tensor q = make(GGML_TYPE_F32, C, L, N, 0x100000);
    ggml_tensor k = make(GGML_TYPE_F32, C, L, N, 0x200000);
    ggml_tensor v = make(GGML_TYPE_F32, C, L, N, 0x300000);

    // 2. build-time support test
    CHECK(kd_bridge::supports_attention(&q, &k, &v, H, nullptr));
    CHECK(kd_bridge::supports_attention(&q, &k, &v, 64, nullptr));        // head_dim 64 (the lite video model)
    CHECK(!kd_bridge::supports_attention(&q, &k, &v, 16, nullptr));       // head_dim 256
    ggml_tensor kg = make(GGML_TYPE_F32, 1024, L, N, 0x200000), vg = make(GGML_TYPE_F32, 1024, L, N, 0x300000);
    CHECK(kd_bridge::supports_attention(&q, &kg, &vg, H, nullptr));       // GQA 32 : 8
    ggml_tensor qh = make(GGML_TYPE_F16, C, L, N, 0x100000);
    CHECK(!kd_bridge::supports_attention(&qh, &k, &v, H, nullptr));       // ops::attention feeds f32
    ggml_tensor vq = make(GGML_TYPE_F32, 512, 4096, 1, 0x500000), vk = make(GGML_TYPE_F32, 512, 4096, 1, 0x600000),
                vv = make(GGML_TYPE_F32, 512, 4096, 1, 0x700000);
    CHECK(kd_bridge::supports_attention(&vq, &vk, &vv, 1, nullptr));      // VAE mid block: one head of 512
    CHECK(!kd_bridge::supports_attention(&vq, &vk, &vv, 2, nullptr));     // two heads of 256
    ggml_tensor mf = make(GGML_TYPE_F32, L, L, 1, 0x400000), mh = make(GGML_TYPE_F16, L, L, 1, 0x400000);
    CHECK(!kd_bridge::supports_attention(&vq, &vk, &vv, 1, &mh));
    CHECK(!kd_bridge::supports_attention(&q, &k, &v, H, &mf));
    CHECK(kd_bridge::supports_attention(&q, &k, &v, H, &mh));

    // 3. disabled bridge, non-flash, causal, unsupported shapes: the reference's own path
    g_reference_calls = 0;
    CHECK(ops_kd::attention(&gctx, nullptr, &q, &k, &v, H, nullptr, true) == &g_reference_result);
    kd_bridge::state().ctx = fake_ctx;
    CHECK(ops_kd::attention(&gctx, nullptr, &q, &k, &v, H, nullptr, false) == &g_reference_result);
    CHECK(ops_kd::attention(&gctx, nullptr, &q, &k, &v, H, nullptr, true, true) == &g_reference_result);
    CHECK(ops_kd::attention(&gctx, nullptr, &q, &k, &v, 16, nullptr, true) == &g_reference_result);
    CHECK(g_reference_calls == 4 && g_nodes.empty());

    // 4. supported flash call: one custom node; its callback calls kd_attn_attention on the mapping
    ggml_tensor* node = ops_kd::attention(&gctx, nullptr, &q, &k, &v, H, &mh, true);
    CHECK(node && node != &g_reference_result && g_nodes.size() == 1);
    CHECK(node->ne[0] == C && node->ne[1] == L && node->ne[2] == N && node->type == GGML_TYPE_F32);
    g_funs[0](node, 1, 4, g_user[0]);  // worker threads other than 0 do nothing
    CHECK(g_calls.empty());
    g_funs[0](node, 0, 4, g_user[0]);
    CHECK(g_calls.size() == 1 && !strcmp(g_calls[0].fn, "attention"));
    CHECK(same(g_calls[0].q, q, KD_ATTN_TYPE_F32) && same(g_calls[0].k, k, KD_ATTN_TYPE_F32) &&
          same(g_calls[0].v, v, KD_ATTN_TYPE_F32) && same(g_calls[0].o, *node, KD_ATTN_TYPE_F32));
    CHECK(g_calls[0].has_mask && same(g_calls[0].m, mh, KD_ATTN_TYPE_F16));
    CHECK(g_calls[0].n_head == H && g_calls[0].op_type == KD_ATTN_TYPE_F16);  // ggml semantics: f16 K/V
    CHECK(kd_bridge::state().last_status == KD_ATTN_OK);

    // 5. a library error at compute time is reported through the bridge state
    g_status = KD_ATTN_ERR_UNSUPPORTED;
    g_funs[0](node, 0, 1, g_user[0]);
    CHECK(kd_bridge::state().last_status == KD_ATTN_ERR_UNSUPPORTED);
    g_status = KD_ATTN_OK;

    // 6. the fused DiT self-attention node (crossdit.hpp:132-150)
    static float gains[2][128];
    kd_bridge::DitAttentionParams prm;
    prm.n_head = (int32_t)H;
    prm.q_gain = gains[0];
    prm.k_gain = gains[1];
    prm.rope.axes_dim[0] = 32; prm.rope.axes_dim[1] = 48; prm.rope.axes_dim[2] = 48;
    prm.rope.grid[0] = 5; prm.rope.grid[1] = 16; prm.rope.grid[2] = 16;
    prm.rope.scale_factor[0] = 1; prm.rope.scale_factor[1] = 2; prm.rope.scale_factor[2] = 2;
    prm.rope.theta = 10000.f;
    g_calls.clear();
    ggml_tensor* dnode = ops_kd::dit_self_attention(&gctx, &q, &k, &v, &prm);
    CHECK(dnode && g_nodes.size() == 2);
    g_funs[1](dnode, 0, 1, g_user[1]);
    CHECK(g_calls.size() == 1 && !strcmp(g_calls[0].fn, "self_attention"));
    CHECK(g_calls[0].qg == gains[0] && g_calls[0].kg == gains[1] && g_calls[0].rope == &prm.rope);
    CHECK(same(g_calls[0].q, q, KD_ATTN_TYPE_F32) && same(g_calls[0].o, *dnode, KD_ATTN_TYPE_F32));
    prm.rope.grid[0] = 6;  // grid no longer covers L: the call site keeps its own code
    CHECK(ops_kd::dit_self_attention(&gctx, &q, &k, &v, &prm) == nullptr);
    prm.rope.grid[0] = 5;

    // 6b. the whole DiTSelfAttention::forward as one node, GGUF weight types kept (q8_0 Q/K/V, q4_0 out_layer)
    {
        ggml_tensor x = make(GGML_TYPE_F32, C, L, N, 0x800000);
        ggml_tensor w[4], b[4];
        for (int i = 0; i < 4; ++i) {
            w[i] = make(i < 3 ? GGML_TYPE_Q8_0 : GGML_TYPE_Q4_0, C, C, 1, 0x900000 + 0x100000 * i);
            w[i].nb[1] = (size_t)C / 32 * (i < 3 ? 34 : 18);  // ggml row size of the block types
            b[i] = make(GGML_TYPE_F32, C, 1, 1, 0xd00000 + 0x10000 * i);
        }
        ggml_tensor* wp[4] = {&w[0], &w[1], &w[2], &w[3]};
        ggml_tensor* bp[4] = {&b[0], &b[1], nullptr, &b[3]};  // to_value without a bias
        const size_t before = g_nodes.size();
        g_calls.clear();
        ggml_tensor* bnode = ops_kd::dit_self_attention_block(&gctx, &x, wp, bp, &prm);
        CHECK(bnode && g_nodes.size() == before + 1);
        CHECK(bnode->ne[0] == C && bnode->ne[1] == L && bnode->ne[2] == N);
        g_funs.back()(bnode, 0, 1, g_user.back());
        CHECK(g_calls.size() == 1 && !strcmp(g_calls[0].fn, "self_attention_block"));
        CHECK(same(g_block_x, x, KD_ATTN_TYPE_F32) && same(g_block_y, *bnode, KD_ATTN_TYPE_F32));
        CHECK(g_block_w[0].type == KD_ATTN_TYPE_Q8_0 && g_block_w[3].type == KD_ATTN_TYPE_Q4_0);
        CHECK(g_block_w[1].data == w[1].data && g_block_w[1].nb1 == w[1].nb[1] && g_block_w[1].ne[0] == C);
        CHECK(g_block_w[0].bias == b[0].data && g_block_w[2].bias == nullptr);
        CHECK(g_calls[0].qg == gains[0] && g_calls[0].rope == &prm.rope && g_calls[0].n_head == prm.n_head);
        ggml_tensor bad = w[1];
        bad.type = (enum ggml_type)3;  // q4_1: not a type the GEMM expands
        ggml_tensor* wbad[4] = {&w[0], &bad, &w[2], &w[3]};
        CHECK(ops_kd::dit_self_attention_block(&gctx, &x, wbad, bp, &prm) == nullptr);
        ggml_tensor wsmall = make(GGML_TYPE_F16, C, 384, 1, 0x900000);  // 384 outputs: not a multiple of 256
        ggml_tensor* wsm[4] = {&w[0], &w[1], &w[2], &wsmall};
        CHECK(ops_kd::dit_self_attention_block(&gctx, &x, wsm, bp, &prm) == nullptr);
    }

    // 7. CFG halves as one batch-2 call (pipeline.cpp:1571-1592 runs two batch-1 forwards)
    {
        const size_t half = (size_t)C * L * 4 + 4096;  // second buffer 4 KB past the end of the first
        ggml_tensor c[4], u[4];
        const ggml_tensor* cp[4];
        const ggml_tensor* up[4];
        for (int i = 0; i < 4; ++i) {
            c[i] = make(GGML_TYPE_F32, C, L, 1, 0x10000000 + i * 0x10000000ull);
            u[i] = make(GGML_TYPE_F32, C, L, 1, 0x10000000 + i * 0x10000000ull + half);
            cp[i] = &c[i];
            up[i] = &u[i];
        }
        kd_tensor pair{};
        CHECK(kd_bridge::cfg_pair(&c[0], &u[0], &pair));
        CHECK(pair.ne[2] == 2 && pair.nb[2] == half && pair.data == c[0].data && pair.nb[1] == c[0].nb[1]);
        CHECK(!kd_bridge::cfg_pair(&u[0], &c[0], &pair));  // must be in address order
        ggml_tensor odd = u[0];
        odd.data = reinterpret_cast<char*>(odd.data) + 4;
        CHECK(!kd_bridge::cfg_pair(&c[0], &odd, &pair));  // stride not a multiple of 16 bytes
        ggml_tensor overlap = u[0];
        overlap.data = reinterpret_cast<char*>(c[0].data) + 16;
        CHECK(!kd_bridge::cfg_pair(&c[0], &overlap, &pair));
        g_calls.clear();
        CHECK(kd_bridge::cfg_pair_self_attention(cp, up, prm) == KD_ATTN_OK);
        CHECK(g_calls.size() == 1 && g_calls[0].q.ne[2] == 2 && g_calls[0].o.nb[2] == half);
        up[2] = &odd;
        CHECK(kd_bridge::cfg_pair_self_attention(cp, up, prm) == KD_ATTN_ERR_UNSUPPORTED);
    }

    for (ggml_tensor* t : g_nodes) delete t;
    if (g_fail) {
        printf("%d check(s) failed\n", g_fail);
        return 1;
    }
    printf("ALL OK\n");
    return 0;
}
