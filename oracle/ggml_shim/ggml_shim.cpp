// Eager implementation of the ggml shim declared in ggml.h (test infrastructure
// only; see that header). A context is an arena of tensors; custom ops run at
// construction time on an OpenMP team of shim_get_threads() threads.
#include "ggml.h"

#include <omp.h>
#include <cstdlib>
#include <cstring>
#include <vector>

struct ggml_context {
    std::vector<ggml_tensor*> tensors;
    std::vector<void*> buffers;
};

static int g_threads = 1;

void shim_set_threads(int n) { g_threads = n > 0 ? n : 1; }
int shim_get_threads(void) { return g_threads; }

ggml_context* shim_ctx_new(void) { return new ggml_context(); }

void shim_ctx_free(ggml_context* ctx) {
    if (!ctx) return;
    for (ggml_tensor* t : ctx->tensors) delete t;
    for (void* b : ctx->buffers) std::free(b);
    delete ctx;
}

static ggml_tensor* make_tensor(ggml_context* ctx, int64_t ne0, int64_t ne1, int64_t ne2,
                                int64_t ne3) {
    ggml_tensor* t = new ggml_tensor();
    std::memset(t, 0, sizeof(*t));
    t->type = GGML_TYPE_F32;
    t->ne[0] = ne0; t->ne[1] = ne1; t->ne[2] = ne2; t->ne[3] = ne3;
    t->nb[0] = sizeof(float);
    t->nb[1] = t->nb[0] * (size_t)ne0;
    t->nb[2] = t->nb[1] * (size_t)ne1;
    t->nb[3] = t->nb[2] * (size_t)ne2;
    ctx->tensors.push_back(t);
    return t;
}

ggml_tensor* shim_wrap_f32(ggml_context* ctx, float* data, int64_t ne0, int64_t ne1,
                           int64_t ne2, int64_t ne3) {
    ggml_tensor* t = make_tensor(ctx, ne0, ne1, ne2, ne3);
    t->data = data;
    return t;
}

ggml_tensor* shim_new_f32(ggml_context* ctx, int64_t ne0, int64_t ne1, int64_t ne2,
                          int64_t ne3) {
    ggml_tensor* t = make_tensor(ctx, ne0, ne1, ne2, ne3);
    const size_t bytes = (size_t)ne0 * ne1 * ne2 * ne3 * sizeof(float);
    void* p = nullptr;
    if (posix_memalign(&p, 64, bytes ? bytes : 64) != 0) std::abort();
    std::memset(p, 0, bytes);
    ctx->buffers.push_back(p);
    t->data = p;
    return t;
}

int64_t ggml_nelements(const ggml_tensor* t) {
    return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3];
}

ggml_tensor* ggml_custom_4d(ggml_context* ctx, ggml_type type, int64_t ne0, int64_t ne1,
                            int64_t ne2, int64_t ne3, ggml_tensor** args, int n_args,
                            ggml_custom_op_t fun, int n_tasks, void* userdata) {
    (void)type;
    ggml_tensor* dst = shim_new_f32(ctx, ne0, ne1, ne2, ne3);
    for (int i = 0; i < n_args && i < GGML_MAX_SRC; ++i) dst->src[i] = args[i];
    const int nth = (n_tasks > 0 && n_tasks < g_threads) ? n_tasks : g_threads;
    if (nth == 1) {
        fun(dst, 0, 1, userdata);
    } else {
#pragma omp parallel num_threads(nth)
        { fun(dst, omp_get_thread_num(), nth, userdata); }
    }
    return dst;
}
