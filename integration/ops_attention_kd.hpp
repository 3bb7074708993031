// ops_attention_kd.hpp -- kandinsky.cpp's attention call sites routed through libkd_attn.
//
// ops_kd::attention has the signature of the reference's ops::attention (src/core/ops.hpp:107-114)
// and is a drop-in for it.  Its flash branch (ops.hpp:164-185) becomes one ggml custom node that
// runs kd_attn_attention on the node's tensors; everything libkd_attn does not cover -- the
// non-flash and causal paths (Qwen, CLIP, VAE3D), head_dim != 128 (the VAE2D mid block), quantised
// or non-f32 inputs -- is decided at graph-build time and goes to the reference's own
// ops::attention unchanged, as the reference itself falls back when ggml_backend_supports_op
// rejects the flash node (ops.hpp:179-181).
//
// ops_kd::dit_self_attention is the fused form for DiTSelfAttention::forward (crossdit.hpp:132-150):
// RMSNorm of q and k, 3D RoPE, attention, from the raw to_query/to_key/to_value outputs, as one node.
// It returns nullptr when the library does not cover the call; the call site then keeps its code.
// ops_kd::dit_self_attention_block is the whole module (crossdit.hpp:117-154) as one node: the Linears
// with their GGUF weights, the norms, RoPE, attention and out_layer.
//
// Include after the reference's core/ops.hpp (for ops::attention) and after ggml.h.
#pragma once

#include "kd_ggml_bridge.hpp"

namespace ops_kd {

inline ggml_tensor* attention(ggml_context* ctx, ggml_backend_t backend, ggml_tensor* q, ggml_tensor* k,
                              ggml_tensor* v, int64_t n_head, ggml_tensor* mask = nullptr, bool flash = false,
                              bool causal = false) {
    if (!flash || causal || !kd_bridge::enabled() || !kd_bridge::supports_attention(q, k, v, n_head, mask))
        return ops::attention(ctx, backend, q, k, v, n_head, mask, flash, causal);
    // The reference passes the mask transposed to ggml_flash_attn_ext (ops.hpp:172-174); libkd_attn
    // takes ggml's flash orientation [Lk, Lq], the layout ggml_flash_attn_ext documents -- the
    // CrossDiT call sites pass no mask (crossdit.hpp:327,356,611).
    ggml_tensor* args[4] = {q, k, v, mask};
    return ggml_custom_4d(ctx, GGML_TYPE_F32, q->ne[0], q->ne[1], q->ne[2], 1, args, mask ? 4 : 3,
                          kd_bridge::attention_node, 1, reinterpret_cast<void*>((intptr_t)n_head));
}

// q, k, v: the to_query / to_key / to_value outputs [C, L, N] (f32).  `params` must outlive the
// graph's computation (the node keeps a pointer to it).
inline ggml_tensor* dit_self_attention(ggml_context* ctx, ggml_tensor* q, ggml_tensor* k, ggml_tensor* v,
                                       const kd_bridge::DitAttentionParams* params) {
    if (!kd_bridge::enabled() || !params || !kd_bridge::supports_attention(q, k, v, params->n_head, nullptr) ||
        q->ne[1] != k->ne[1] || k->ne[0] != q->ne[0])
        return nullptr;
    if (params->use_rope &&
        (int64_t)params->rope.grid[0] * params->rope.grid[1] * params->rope.grid[2] != q->ne[1])
        return nullptr;
    ggml_tensor* args[3] = {q, k, v};
    return ggml_custom_4d(ctx, GGML_TYPE_F32, q->ne[0], q->ne[1], q->ne[2], 1, args, 3,
                          kd_bridge::dit_self_attention_node, 1, const_cast<kd_bridge::DitAttentionParams*>(params));
}

// DiTSelfAttention::forward (crossdit.hpp:117-154) whole as one node: x [C, L, N] f32 and the module's
// parameters (to_query, to_key, to_value, out_layer weights and biases; a bias may be null) -> the
// out_layer output [C_out, L, N] f32.  The weights stay in their GGUF types (q4_0 / q8_0 / f16 / bf16 /
// f32).  nullptr when the library does not cover the call; the call site then keeps its code.
inline ggml_tensor* dit_self_attention_block(ggml_context* ctx, ggml_tensor* x, ggml_tensor* const w[4],
                                             ggml_tensor* const b[4], const kd_bridge::DitAttentionParams* params) {
    if (!kd_bridge::enabled() || !params ||
        !kd_bridge::supports_self_attention_block(x, w, b, params->n_head, params->use_rope ? &params->rope : nullptr))
        return nullptr;
    ggml_tensor* args[9] = {x, w[0], b[0], w[1], b[1], w[2], b[2], w[3], b[3]};
    return ggml_custom_4d(ctx, GGML_TYPE_F32, w[3]->ne[1], x->ne[1], x->ne[2], 1, args, 9, kd_bridge::dit_block_node, 1,
                          const_cast<kd_bridge::DitAttentionParams*>(params));
}

}  // namespace ops_kd
