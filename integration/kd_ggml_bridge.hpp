// kd_ggml_bridge.hpp -- maps kandinsky.cpp's ggml tensors onto libkd_attn's C ABI.
//
// The reference builds attention as ggml graph nodes (ops::attention, src/core/ops.hpp:107-207);
// libkd_attn computes on device pointers.  This header is the seam between the two:
//   - kd_from_ggml: a ggml_tensor {type, ne[4], nb[4], data} is a kd_tensor field by field
//     (ggml type ids F32 = 0, F16 = 1, BF16 = 30 are libkd_attn's);
//   - supports_attention: the shape/type test libkd_attn applies, made at graph-build time, so the
//     caller keeps ggml's own path for what the library does not cover -- the role of
//     ggml_backend_supports_op in ops.hpp:179-181;
//   - linear_from_ggml / supports_self_attention_block: a Linear's ggml weight (f32/f16/bf16/q4_0/q8_0)
//     and bias as a kd_linear, and the build-time test for DiTSelfAttention::forward as one node;
//   - attention_node / dit_self_attention_node / dit_block_node: ggml custom-op callbacks that run the library on
//     the node's tensors (device memory: the node is computed where the tensors live, i.e. the DiT
//     graph is split at each attention node -- INTEGRATION.md);
//   - cfg_pair_*: the two classifier-free-guidance halves (two batch-1 forwards in the reference,
//     src/pipeline.cpp:1571-1592) as ONE batch-2 call, without a copy: the second half's buffer
//     becomes sequence 1 by its address difference from the first.
// Header-only; needs ggml.h (or integration/stub/ggml.h) and include/kd_attn.h.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstdio>

#include "ggml.h"
#include "kd_attn.h"

namespace kd_bridge {

// Context and stream the callbacks use (set once by the application when libkd_attn is active).
struct State {
    kd_attn_ctx* ctx = nullptr;
    void* stream = nullptr;        // cudaStream_t of the CUDA backend
    int32_t op_type = KD_ATTN_TYPE_F16;  // ggml semantics: K/V cast to f16 (ops.hpp:167-169)
    int last_status = KD_ATTN_OK;  // status of the last call made by a callback
};
inline State& state() {
    static State s;
    return s;
}
inline bool enabled() { return state().ctx != nullptr; }

inline bool type_of(enum ggml_type t, int32_t* out) {
    switch (t) {
        case GGML_TYPE_F32: *out = KD_ATTN_TYPE_F32; return true;
        case GGML_TYPE_F16: *out = KD_ATTN_TYPE_F16; return true;
        case GGML_TYPE_BF16: *out = KD_ATTN_TYPE_BF16; return true;
        default: return false;  // quantised and other types stay on ggml's path
    }
}

// ggml_tensor -> kd_tensor; false for a type libkd_attn does not take.
inline bool kd_from_ggml(const ggml_tensor* t, kd_tensor* out) {
    if (!t || !type_of(t->type, &out->type)) return false;
    out->data = t->data;
    for (int i = 0; i < 4; ++i) {
        out->ne[i] = t->ne[i];
        out->nb[i] = t->nb[i];
    }
    return true;
}

// Would kd_attn_attention accept ops::attention(q, k, v, n_head, mask, flash = true)?  q [C, Lq, N],
// k/v [C_kv, Lk, N] f32 with head_dim 128 or 64, GQA ratio integral, f16 mask [Lk, >=Lq] or none -- or the
// VAE mid block's single head of 512 channels (vae.hpp:89): packed rows, no mask.
inline bool supports_attention(const ggml_tensor* q, const ggml_tensor* k, const ggml_tensor* v, int64_t n_head,
                               const ggml_tensor* mask) {
    if (!q || !k || !v || n_head <= 0 || q->ne[0] % n_head) return false;
    const int64_t d = q->ne[0] / n_head;
    if (d == 512 && n_head == 1) {
        const ggml_tensor* t[3] = {q, k, v};
        for (const ggml_tensor* x : t)
            if (x->type != GGML_TYPE_F32 || x->ne[0] != 512 || x->nb[0] != 4 || x->nb[1] != 512 * 4 || x->ne[3] != 1)
                return false;
        return !mask && k->ne[1] == v->ne[1] && k->ne[2] == q->ne[2] && v->ne[2] == q->ne[2];
    }
    if ((d != 128 && d != 64) || k->ne[0] % d || v->ne[0] != k->ne[0] || q->ne[3] != 1 || k->ne[3] != 1 ||
        v->ne[3] != 1)
        return false;
    const int64_t n_kv = k->ne[0] / d;
    if (n_kv <= 0 || n_head % n_kv || k->ne[1] != v->ne[1] || k->ne[2] != q->ne[2] || v->ne[2] != q->ne[2]) return false;
    if (q->type != GGML_TYPE_F32 || k->type != GGML_TYPE_F32 || v->type != GGML_TYPE_F32) return false;
    if (q->nb[0] != 4 || k->nb[0] != 4 || v->nb[0] != 4) return false;
    if (mask && (mask->type != GGML_TYPE_F16 || mask->ne[0] < k->ne[1] || mask->ne[1] < q->ne[1])) return false;
    return true;
}

// Custom-op callback of ops_kd::attention: dst [C, Lq, N] f32 = the flash branch of ops::attention on
// dst->src[0..2] (q, k, v) and optional src[3] (mask); userdata = n_head.
inline void attention_node(ggml_tensor* dst, int ith, int /*nth*/, void* userdata) {
    if (ith != 0) return;
    State& s = state();
    kd_tensor q, k, v, m, o;
    const bool has_mask = dst->src[3] != nullptr;
    if (!s.ctx || !kd_from_ggml(dst->src[0], &q) || !kd_from_ggml(dst->src[1], &k) || !kd_from_ggml(dst->src[2], &v) ||
        (has_mask && !kd_from_ggml(dst->src[3], &m)) || !kd_from_ggml(dst, &o)) {
        s.last_status = KD_ATTN_ERR_INVALID_ARGUMENT;
        return;
    }
    s.last_status = kd_attn_attention(s.ctx, &q, &k, &v, (int32_t)(intptr_t)userdata, has_mask ? &m : nullptr,
                                      s.op_type, &o, nullptr, s.stream);
    if (s.last_status != KD_ATTN_OK)
        fprintf(stderr, "kd_bridge: kd_attn_attention failed (%d): %s\n", s.last_status, kd_attn_last_error(s.ctx));
}

// Parameters of a fused DiT self-attention node (crossdit.hpp:132-150): RMSNorm gains of the q/k
// norms (device, [head_dim]) and the token grid of the 3D RoPE.
struct DitAttentionParams {
    int32_t n_head = 32;
    const float* q_gain = nullptr;
    const float* k_gain = nullptr;
    float eps = 1e-6f;
    kd_rope3d rope{};
    bool use_rope = true;
};

// Custom-op callback: dst [C, L, N] = attention(RMSNorm+RoPE(q), RMSNorm+RoPE(k), v) from the raw
// to_query/to_key/to_value outputs dst->src[0..2] -- crossdit.hpp:132-150 in one library call.
inline void dit_self_attention_node(ggml_tensor* dst, int ith, int /*nth*/, void* userdata) {
    if (ith != 0) return;
    State& s = state();
    const DitAttentionParams* a = static_cast<const DitAttentionParams*>(userdata);
    kd_tensor q, k, v, o;
    if (!s.ctx || !a || !kd_from_ggml(dst->src[0], &q) || !kd_from_ggml(dst->src[1], &k) ||
        !kd_from_ggml(dst->src[2], &v) || !kd_from_ggml(dst, &o)) {
        s.last_status = KD_ATTN_ERR_INVALID_ARGUMENT;
        return;
    }
    s.last_status = kd_attn_self_attention(s.ctx, &q, &k, &v, a->n_head, a->q_gain, a->k_gain, a->eps,
                                           a->use_rope ? &a->rope : nullptr, s.op_type, &o, nullptr, s.stream);
    if (s.last_status != KD_ATTN_OK)
        fprintf(stderr, "kd_bridge: kd_attn_self_attention failed (%d): %s\n", s.last_status,
                kd_attn_last_error(s.ctx));
}

// A Linear's parameters (module.hpp:97-103: weight ggml [in, out], f32 bias [out] or none) as a kd_linear.
inline bool linear_from_ggml(const ggml_tensor* w, const ggml_tensor* b, kd_linear* out) {
    if (!w) return false;
    switch (w->type) {
        case GGML_TYPE_F32: out->type = KD_ATTN_TYPE_F32; break;
        case GGML_TYPE_F16: out->type = KD_ATTN_TYPE_F16; break;
        case GGML_TYPE_BF16: out->type = KD_ATTN_TYPE_BF16; break;
        case GGML_TYPE_Q4_0: out->type = KD_ATTN_TYPE_Q4_0; break;
        case GGML_TYPE_Q8_0: out->type = KD_ATTN_TYPE_Q8_0; break;
        default: return false;
    }
    if (b && (b->type != GGML_TYPE_F32 || b->ne[0] != w->ne[1])) return false;
    out->data = w->data;
    out->ne[0] = w->ne[0];
    out->ne[1] = w->ne[1];
    out->nb1 = w->nb[1];
    out->bias = b ? static_cast<const float*>(b->data) : nullptr;
    return true;
}

// Would kd_attn_self_attention_block take DiTSelfAttention::forward(x) with these parameters?  x [C, L, N]
// f32 with C = n_head * d, d = 128 or 64, the four Linears [C, C] (out_layer [C, C_out]) of types the GEMM
// expands, C and C_out multiples of 256, a RoPE grid covering L.
inline bool supports_self_attention_block(const ggml_tensor* x, const ggml_tensor* const w[4],
                                          const ggml_tensor* const b[4], int64_t n_head, const kd_rope3d* rope) {
    if (!x || x->type != GGML_TYPE_F32 || x->nb[0] != 4 || x->ne[3] != 1 || n_head <= 0) return false;
    const int64_t C = x->ne[0];
    if ((C != n_head * 128 && C != n_head * 64) || C % 256) return false;
    for (int i = 0; i < 4; ++i) {
        kd_linear l{};
        if (!linear_from_ggml(w[i], b[i], &l) || l.ne[0] != C || l.ne[1] % 256 || (i < 3 && l.ne[1] != C)) return false;
    }
    return !rope || (int64_t)rope->grid[0] * rope->grid[1] * rope->grid[2] == x->ne[1];
}

// Custom-op callback: dst [C_out, L, N] f32 = DiTSelfAttention::forward (crossdit.hpp:117-154) of
// dst->src[0] = x, with src[1..8] = to_query, to_key, to_value, out_layer (weight, bias) pairs (a null
// bias slot = no bias) and the norms / RoPE of `userdata` (a DitAttentionParams).
inline void dit_block_node(ggml_tensor* dst, int ith, int /*nth*/, void* userdata) {
    if (ith != 0) return;
    State& s = state();
    const DitAttentionParams* a = static_cast<const DitAttentionParams*>(userdata);
    kd_tensor x, y;
    kd_linear w[4];
    bool ok = s.ctx && a && kd_from_ggml(dst->src[0], &x) && kd_from_ggml(dst, &y);
    for (int i = 0; i < 4 && ok; ++i) ok = linear_from_ggml(dst->src[1 + 2 * i], dst->src[2 + 2 * i], &w[i]);
    if (!ok) {
        s.last_status = KD_ATTN_ERR_INVALID_ARGUMENT;
        return;
    }
    s.last_status = kd_attn_self_attention_block(s.ctx, &x, &w[0], &w[1], &w[2], &w[3], a->n_head, a->q_gain,
                                                 a->k_gain, a->eps, a->use_rope ? &a->rope : nullptr, &y, s.stream);
    if (s.last_status != KD_ATTN_OK)
        fprintf(stderr, "kd_bridge: kd_attn_self_attention_block failed (%d): %s\n", s.last_status,
                kd_attn_last_error(s.ctx));
}

// Two batch-1 tensors [C, L, 1] of the same shape, type and row stride (the conditional and the
// unconditional half of a CFG step) seen as one [C, L, 2] tensor whose sequence stride is the
// address difference of their buffers.  The first argument must lie below the second and the
// difference be a multiple of 16 bytes (TMA strides); otherwise false and the caller makes two calls.
inline bool cfg_pair(const ggml_tensor* a, const ggml_tensor* b, kd_tensor* out) {
    kd_tensor ta, tb;
    if (!kd_from_ggml(a, &ta) || !kd_from_ggml(b, &tb) || ta.type != tb.type) return false;
    for (int i = 0; i < 4; ++i)
        if (ta.ne[i] != tb.ne[i] || (i < 2 && ta.nb[i] != tb.nb[i])) return false;
    if (ta.ne[2] != 1 || ta.ne[3] != 1) return false;
    const char* pa = static_cast<const char*>(ta.data);
    const char* pb = static_cast<const char*>(tb.data);
    if (pb <= pa || (size_t)(pb - pa) % 16) return false;
    const size_t span = ta.nb[1] * (size_t)ta.ne[1];
    if ((size_t)(pb - pa) < span) return false;  // the halves must not overlap
    *out = ta;
    out->ne[2] = 2;
    out->nb[2] = (size_t)(pb - pa);
    out->nb[3] = out->nb[2] * 2;
    return true;
}

// One batch-2 DiT self-attention for both CFG halves (pipeline.cpp:1571-1592 runs two batch-1
// forwards): q/k/v/out of the conditional and unconditional forward, each [C, L, 1].  Returns
// KD_ATTN_ERR_UNSUPPORTED when the buffers cannot be paired (the caller then makes two calls).
inline int cfg_pair_self_attention(const ggml_tensor* const cond[4], const ggml_tensor* const uncond[4],
                                   const DitAttentionParams& a) {
    State& s = state();
    if (!s.ctx) return KD_ATTN_ERR_INVALID_ARGUMENT;
    kd_tensor t[4];
    for (int i = 0; i < 4; ++i)
        if (!cfg_pair(cond[i], uncond[i], &t[i])) return KD_ATTN_ERR_UNSUPPORTED;
    return kd_attn_self_attention(s.ctx, &t[0], &t[1], &t[2], a.n_head, a.q_gain, a.k_gain, a.eps,
                                  a.use_rope ? &a.rope : nullptr, s.op_type, &t[3], nullptr, s.stream);
}

}  // namespace kd_bridge
