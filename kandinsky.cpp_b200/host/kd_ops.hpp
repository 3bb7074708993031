// kd_ops.hpp -- the C++ host side of libkd_attn: the reference's operator interface for the
// CrossDiT attention path, re-expressed over the C ABI in include/kd_attn.h.
//
// kandinsky.cpp builds ggml graphs; the functions below are what its graph code calls on this
// path, with the same names, argument meanings and error behaviour, but they run on device
// buffers immediately (enqueued on a CUDA stream) instead of adding graph nodes:
//
//   kd::ops::attention            src/core/ops.hpp:107-207  (ops::attention, flash branch)
//   kd::ops::linear               src/core/ops.hpp:27-42    (ops::linear: mul_mat + bias)
//   kd::Linear                    src/core/module.hpp:87-110 (Linear's weight and bias)
//   kd::dit_self_attention_block  src/models/crossdit.hpp:117-154 (DiTSelfAttention::forward whole:
//                                 to_query/to_key/to_value, norms, RoPE, attention, out_layer)
//   kd::dit_cross_attention_block src/models/crossdit.hpp:174-200 (DiTCrossAttention::forward whole)
//   kd::dit_self_attention        src/models/crossdit.hpp:132-150 (DiTSelfAttention::forward
//                                 between the Q/K/V Linears and out_layer)
//   kd::dit_cross_attention       src/models/crossdit.hpp:186-198 (DiTCrossAttention::forward)
//   kd::CrossDiTAttentionConfig   src/models/crossdit.hpp:48-56,67-75 (lite_video / pro_video constants used here)
//
// Errors: like ops::attention (which logs LOG_ERROR and returns nullptr on an invalid GQA
// ratio, ops.hpp:136-139) these return false and report through the library's log callback;
// kd::Context::last_error() holds the text.  There is no fallback: a shape the kernels do not
// cover (head_dim other than 128 or 64, the causal / non-flash branch) returns false with the reason.
//
// Header-only; link libkd_attn.so.  No CUDA headers are needed: streams are passed as void*.
#pragma once

#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>

#include "kd_attn.h"

namespace kd {

// A device tensor in ggml's convention (ne = sizes, nb = byte strides, dim 0 fastest).
struct Tensor {
    void* data = nullptr;
    int32_t type = KD_ATTN_TYPE_F32;
    int64_t ne[4] = {1, 1, 1, 1};
    size_t nb[4] = {0, 0, 0, 0};

    static size_t type_size(int32_t t) { return t == KD_ATTN_TYPE_F32 ? 4 : 2; }

    // Contiguous tensor of the given sizes (ggml_new_tensor_4d's strides).
    static Tensor contiguous(void* data, int32_t type, int64_t ne0, int64_t ne1 = 1, int64_t ne2 = 1,
                             int64_t ne3 = 1) {
        Tensor t;
        t.data = data;
        t.type = type;
        t.ne[0] = ne0;
        t.ne[1] = ne1;
        t.ne[2] = ne2;
        t.ne[3] = ne3;
        t.nb[0] = type_size(type);
        for (int i = 1; i < 4; ++i) t.nb[i] = t.nb[i - 1] * (size_t)t.ne[i - 1];
        return t;
    }

    size_t bytes() const { return nb[3] * (size_t)ne[3]; }

    kd_tensor view() const {
        kd_tensor k{};
        k.data = data;
        k.type = type;
        for (int i = 0; i < 4; ++i) {
            k.ne[i] = ne[i];
            k.nb[i] = nb[i];
        }
        return k;
    }
};

// The constants of a CrossDiTConfig that this path reads (crossdit.hpp:48-56,67-75, rope.hpp:60):
// pro_video (and lite_image) head_dim 128 = 32 + 48 + 48 rotary dims; lite_video head_dim 64 =
// 16 + 24 + 24; scale_factor {1, 2, 2}, theta 1e4, RMSNorm eps 1e-6.
struct CrossDiTAttentionConfig {
    int32_t head_dim = 128;
    int32_t axes_dims[3] = {32, 48, 48};
    float scale_factor[3] = {1.f, 2.f, 2.f};
    float rope_theta = 10000.f;
    float norm_eps = 1e-6f;
    int32_t op_type = KD_ATTN_TYPE_BF16;  // operand type of the flash kernel (ggml: f16)

    static CrossDiTAttentionConfig pro_video() { return CrossDiTAttentionConfig{}; }
    static CrossDiTAttentionConfig lite_video() {
        CrossDiTAttentionConfig c;
        c.head_dim = 64;
        c.axes_dims[0] = 16;
        c.axes_dims[1] = 24;
        c.axes_dims[2] = 24;
        return c;
    }
    bool supported() const { return head_dim == 128 || head_dim == 64; }
};

// A Linear layer's parameters as Linear::init_params allocates them (module.hpp:97-103): the weight, ggml
// [in_features, out_features] of type f32 / f16 / bf16 / q4_0 / q8_0 (row r = output feature r, nb1 bytes
// apart), and an f32 bias [out_features] or none.
struct Linear {
    const void* weight = nullptr;
    int32_t type = KD_ATTN_TYPE_F16;
    int64_t in_features = 0, out_features = 0;
    size_t nb1 = 0;
    const float* bias = nullptr;

    kd_linear view() const {
        kd_linear l{};
        l.data = weight;
        l.type = type;
        l.ne[0] = in_features;
        l.ne[1] = out_features;
        l.nb1 = nb1;
        l.bias = bias;
        return l;
    }
};

// Owns one kd_attn_ctx (per device).  Move-only.
class Context {
public:
    explicit Context(int device = 0, kd_attn_log_cb log_cb = nullptr, void* log_user = nullptr) {
        kd_attn_init init{};
        init.device = device;
        init.n_ranks = 1;
        init.rank = 0;
        init.log_cb = log_cb;
        init.log_user_data = log_user;
        status_ = kd_attn_create(&init, &ctx_);
    }
    ~Context() {
        if (ctx_) kd_attn_destroy(ctx_);
    }
    Context(const Context&) = delete;
    Context& operator=(const Context&) = delete;
    Context(Context&& o) noexcept : ctx_(o.ctx_), status_(o.status_) { o.ctx_ = nullptr; }

    bool ok() const { return ctx_ != nullptr; }
    kd_attn_status create_status() const { return status_; }
    kd_attn_ctx* get() const { return ctx_; }
    std::string last_error() const { return ctx_ ? kd_attn_last_error(ctx_) : "context not created"; }
    // Synchronises `stream` and reports device-side wait timeouts (kd_attn_device_status).
    bool device_status(void* stream = nullptr) const { return ctx_ && kd_attn_device_status(ctx_, stream) == KD_ATTN_OK; }

private:
    kd_attn_ctx* ctx_ = nullptr;
    kd_attn_status status_ = KD_ATTN_ERR_INVALID_ARGUMENT;
};

namespace ops {

// ops::attention(ctx, backend, q, k, v, n_head, mask, flash, causal) (ops.hpp:107-207):
//   q: [C, L_q, N] (C = n_head * 128), k, v: [C_kv, L_k, N] with n_head % (C_kv / 128) == 0 (GQA),
//   mask: nullptr or f16 in the flash orientation [>=L_k, >=L_q, mh, mn],
//   out: [C, L_q, N] (f32, or the operand type).  Only the flash branch exists here: flash = false
//   or causal = true returns false (the caller keeps its ggml path, as for any unsupported op).
inline bool attention(Context& ctx, const Tensor& q, const Tensor& k, const Tensor& v, int64_t n_head, Tensor& out,
                      const Tensor* mask = nullptr, bool flash = true, bool causal = false,
                      int32_t op_type = KD_ATTN_TYPE_F16, void* stream = nullptr) {
    if (!ctx.ok() || !flash || causal || n_head <= 0 || n_head > INT32_MAX) return false;
    const kd_tensor tq = q.view(), tk = k.view(), tv = v.view();
    kd_tensor to = out.view();
    kd_tensor tm{};
    if (mask) tm = mask->view();
    return kd_attn_attention(ctx.get(), &tq, &tk, &tv, (int32_t)n_head, mask ? &tm : nullptr, op_type, &to, nullptr,
                             stream) == KD_ATTN_OK;
}

// ops::linear(ctx, x, w, b) (ops.hpp:27-42): y = x W^T + b with x [in, L, N] (f32, or bf16 read in place)
// and y [out, L, N] (f32, bf16 or f16).  false on shapes or types the GEMM does not take.
inline bool linear(Context& ctx, const Tensor& x, const Linear& w, Tensor& y, void* stream = nullptr) {
    if (!ctx.ok()) return false;
    const kd_tensor tx = x.view();
    const kd_linear tw = w.view();
    kd_tensor ty = y.view();
    return kd_attn_linear(ctx.get(), &tx, &tw, &ty, stream) == KD_ATTN_OK;
}

}  // namespace ops

// DiTSelfAttention::forward (crossdit.hpp:117-154) whole, from the hidden states x [C, L, N] f32 to the
// out_layer output y [C_out, L, N]: the Q/K/V Linears fused with the per-head RMSNorm and 3D RoPE, the
// flash attention, out_layer.  The operands are bf16 whatever cfg.op_type says.
inline bool dit_self_attention_block(Context& ctx, const Tensor& x, const Linear& to_query, const Linear& to_key,
                                     const Linear& to_value, const Linear& out_layer, const float* query_norm_w,
                                     const float* key_norm_w, const int32_t grid[3],
                                     const CrossDiTAttentionConfig& cfg, Tensor& y, void* stream = nullptr) {
    if (!ctx.ok() || !cfg.supported() || to_query.out_features % cfg.head_dim) return false;
    kd_rope3d rope{};
    for (int a = 0; a < 3; ++a) {
        rope.axes_dim[a] = cfg.axes_dims[a];
        rope.grid[a] = grid[a];
        rope.scale_factor[a] = cfg.scale_factor[a];
    }
    rope.theta = cfg.rope_theta;
    const kd_tensor tx = x.view();
    const kd_linear wq = to_query.view(), wk = to_key.view(), wv = to_value.view(), wo = out_layer.view();
    kd_tensor ty = y.view();
    const int32_t n_head = (int32_t)(to_query.out_features / cfg.head_dim);
    return kd_attn_self_attention_block(ctx.get(), &tx, &wq, &wk, &wv, &wo, n_head, query_norm_w, key_norm_w,
                                        cfg.norm_eps, &rope, &ty, stream) == KD_ATTN_OK;
}

// DiTCrossAttention::forward (crossdit.hpp:174-200) whole: x_query [C, Lq, N] visual and x_kv [C, Lk, N]
// text hidden states (f32) to out_layer's output y [C_out, Lq, N]; RMSNorm on Q and K, no RoPE; the text's
// valid lengths as kv_len (device int32 [N]) and/or an f16 mask, either may be null.
inline bool dit_cross_attention_block(Context& ctx, const Tensor& x_query, const Tensor& x_kv, const Linear& to_query,
                                      const Linear& to_key, const Linear& to_value, const Linear& out_layer,
                                      const float* query_norm_w, const float* key_norm_w, const int32_t* kv_len,
                                      const Tensor* mask, const CrossDiTAttentionConfig& cfg, Tensor& y,
                                      void* stream = nullptr) {
    if (!ctx.ok() || !cfg.supported() || to_query.out_features % cfg.head_dim) return false;
    const kd_tensor tq = x_query.view(), tkv = x_kv.view();
    const kd_linear wq = to_query.view(), wk = to_key.view(), wv = to_value.view(), wo = out_layer.view();
    kd_tensor tm{};
    if (mask) tm = mask->view();
    kd_tensor ty = y.view();
    const int32_t n_head = (int32_t)(to_query.out_features / cfg.head_dim);
    return kd_attn_cross_attention_block(ctx.get(), &tq, &tkv, &wq, &wk, &wv, &wo, n_head, query_norm_w, key_norm_w,
                                         cfg.norm_eps, mask ? &tm : nullptr, kv_len, &ty, stream) == KD_ATTN_OK;
}

// DiTSelfAttention::forward from the Q/K/V projections to the input of out_layer
// (crossdit.hpp:132-150): per-head RMSNorm of Q and K with the query_norm / key_norm weights
// (device f32 [head_dim], or nullptr for unit gain), 3D RoPE over the (frames, height, width) token
// grid with the config's axes and scale factors, flash attention.  q, k, v, out: [C, L, N].
inline bool dit_self_attention(Context& ctx, const Tensor& q, const Tensor& k, const Tensor& v, int64_t n_head,
                               const float* query_norm_w, const float* key_norm_w, const int32_t grid[3],
                               const CrossDiTAttentionConfig& cfg, Tensor& out, void* stream = nullptr) {
    if (!ctx.ok() || !cfg.supported() || n_head <= 0 || n_head > INT32_MAX) return false;
    kd_rope3d rope{};
    for (int a = 0; a < 3; ++a) {
        rope.axes_dim[a] = cfg.axes_dims[a];
        rope.grid[a] = grid[a];
        rope.scale_factor[a] = cfg.scale_factor[a];
    }
    rope.theta = cfg.rope_theta;
    const kd_tensor tq = q.view(), tk = k.view(), tv = v.view();
    kd_tensor to = out.view();
    return kd_attn_self_attention(ctx.get(), &tq, &tk, &tv, (int32_t)n_head, query_norm_w, key_norm_w, cfg.norm_eps,
                                  &rope, cfg.op_type, &to, nullptr, stream) == KD_ATTN_OK;
}

// DiTCrossAttention::forward from the projections to out_layer's input (crossdit.hpp:186-198):
// visual queries against text keys/values, RMSNorm on Q and K, no RoPE.  The text's valid
// lengths come either as kv_len (device int32 [N]) or as an f16 mask; both may be null.
inline bool dit_cross_attention(Context& ctx, const Tensor& q, const Tensor& k, const Tensor& v, int64_t n_head,
                                const float* query_norm_w, const float* key_norm_w, const int32_t* kv_len,
                                const Tensor* mask, const CrossDiTAttentionConfig& cfg, Tensor& out,
                                void* stream = nullptr) {
    if (!ctx.ok() || !cfg.supported() || n_head <= 0 || n_head > INT32_MAX) return false;
    const kd_tensor tq = q.view(), tk = k.view(), tv = v.view();
    kd_tensor to = out.view();
    kd_tensor tm{};
    if (mask) tm = mask->view();
    return kd_attn_cross_attention(ctx.get(), &tq, &tk, &tv, (int32_t)n_head, query_norm_w, key_norm_w,
                                   cfg.norm_eps, mask ? &tm : nullptr, kv_len, cfg.op_type, &to, nullptr,
                                   stream) == KD_ATTN_OK;
}

}  // namespace kd
