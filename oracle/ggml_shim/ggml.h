// Minimal stand-in for the parts of ggml.h that the reference's conv kernel files
// (src/directconv.cpp, src/winograd.cpp) touch, so those files compile UNMODIFIED
// into the CPU oracle library oracle/_ref/libvdref.so.
//
// TEST INFRASTRUCTURE ONLY. Nothing in the product path includes this header.
//
// The six names the reference uses (ggml_tensor, ggml_context, ggml_custom_4d,
// ggml_nelements, GGML_TYPE_F32, GGML_N_TASKS_MAX) are declared with the
// signatures those call sites need:
//   ggml_custom_4d(ctx, type, ne0, ne1, ne2, ne3, args, n_args, fun, n_tasks, ud)
//   (call sites: src/winograd.cpp:646-647, src/directconv.cpp:1456-1457,1505-1507).
// ggml itself is an empty submodule in the reference checkout, so this is written
// from those call sites only.
//
// Semantics of this shim: EAGER. ggml_custom_4d allocates dst in the context
// arena and immediately runs fun(dst, ith, nth, userdata) for ith = 0..nth-1 on
// an OpenMP team, which is exactly the contract the reference's custom-op
// callbacks are written against (each ith processes its own slice).
#pragma once
#include <cstddef>
#include <cstdint>

enum ggml_type { GGML_TYPE_F32 = 0 };

#define GGML_N_TASKS_MAX (-1)
#define GGML_MAX_SRC 10

struct ggml_context;

struct ggml_tensor {
    enum ggml_type type;
    int64_t ne[4];
    size_t nb[4];
    struct ggml_tensor* src[GGML_MAX_SRC];
    void* data;
};

typedef void (*ggml_custom_op_t)(struct ggml_tensor* dst, int ith, int nth, void* userdata);

struct ggml_tensor* ggml_custom_4d(struct ggml_context* ctx, enum ggml_type type,
                                   int64_t ne0, int64_t ne1, int64_t ne2, int64_t ne3,
                                   struct ggml_tensor** args, int n_args,
                                   ggml_custom_op_t fun, int n_tasks, void* userdata);

int64_t ggml_nelements(const struct ggml_tensor* t);

// ---- shim-only helpers (not ggml API; used by oracle/ref_glue.cpp) ----------
struct ggml_context* shim_ctx_new(void);
void shim_ctx_free(struct ggml_context* ctx);
// Wrap caller memory (not owned) as an f32 tensor with contiguous strides.
struct ggml_tensor* shim_wrap_f32(struct ggml_context* ctx, float* data,
                                  int64_t ne0, int64_t ne1, int64_t ne2, int64_t ne3);
// Allocate a new f32 tensor in the context arena (owned by ctx).
struct ggml_tensor* shim_new_f32(struct ggml_context* ctx,
                                 int64_t ne0, int64_t ne1, int64_t ne2, int64_t ne3);
void shim_set_threads(int n);
int shim_get_threads(void);
