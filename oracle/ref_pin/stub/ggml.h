/* Declarations-only stand-in for the ggml API names that the reference's
 * src/rope.hpp mentions inside rope::apply.  rope::apply is never called by
 * the pin driver, so nothing here is defined or linked; it only lets the
 * reference's table builders (get_freqs, compute_text_rope,
 * compute_visual_rope) and src/rng.hpp compile from their own sources. */
#pragma once
#include <stddef.h>
#include <stdint.h>
struct ggml_context;
struct ggml_tensor { int64_t ne[4]; size_t nb[4]; };
ggml_tensor* ggml_reshape_4d(ggml_context*, ggml_tensor*, int64_t, int64_t, int64_t, int64_t);
ggml_tensor* ggml_view_4d(ggml_context*, ggml_tensor*, int64_t, int64_t, int64_t, int64_t,
                          size_t, size_t, size_t, size_t);
ggml_tensor* ggml_cont(ggml_context*, ggml_tensor*);
ggml_tensor* ggml_mul(ggml_context*, ggml_tensor*, ggml_tensor*);
ggml_tensor* ggml_sub(ggml_context*, ggml_tensor*, ggml_tensor*);
ggml_tensor* ggml_add(ggml_context*, ggml_tensor*, ggml_tensor*);
ggml_tensor* ggml_concat(ggml_context*, ggml_tensor*, ggml_tensor*, int);
ggml_tensor* ggml_permute(ggml_context*, ggml_tensor*, int, int, int, int);
