/* Declarations-only stand-in for the parts of ggml's public API (ggml.h) that integration/
 * compiles against, so the shim builds without a ggml checkout.  Names, the field names of
 * ggml_tensor used by the shim, the type ids and the function signatures follow ggml's public
 * header; nothing is implemented here.  Compiling against real ggml replaces this file. */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GGML_MAX_DIMS 4
#define GGML_MAX_SRC 10

enum ggml_type { GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1, GGML_TYPE_Q4_0 = 2, GGML_TYPE_Q8_0 = 8, GGML_TYPE_BF16 = 30 };
enum ggml_prec { GGML_PREC_DEFAULT = 0, GGML_PREC_F32 = 10 };

struct ggml_context;
struct ggml_backend;
typedef struct ggml_backend* ggml_backend_t;

struct ggml_tensor {
    enum ggml_type type;
    int64_t ne[GGML_MAX_DIMS]; /* elements per dim, dim 0 fastest */
    size_t nb[GGML_MAX_DIMS];  /* stride in bytes per dim */
    struct ggml_tensor* src[GGML_MAX_SRC];
    void* data;
    char name[64];
};

typedef void (*ggml_custom_op_t)(struct ggml_tensor* dst, int ith, int nth, void* userdata);

struct ggml_tensor* ggml_custom_4d(struct ggml_context* ctx, enum ggml_type type, int64_t ne0, int64_t ne1,
                                   int64_t ne2, int64_t ne3, struct ggml_tensor** args, int n_args,
                                   ggml_custom_op_t fun, int n_tasks, void* userdata);
int64_t ggml_nelements(const struct ggml_tensor* tensor);

#ifdef __cplusplus
}
#endif
