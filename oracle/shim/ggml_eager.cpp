// Eager stand-in for the ggml operators the reference's PatchEncoder calls
// (src/modules/backbone/patchenc.cpp), so that file compiles and runs as
// written without ggml.  TEST INFRASTRUCTURE ONLY: it is linked into
// oracle/_ref/libdtts_ref.so and nothing else.
//
// Each operator is restated from ggml's published semantics (ggml.h / the
// CPU backend of the llama.cpp tree the reference builds against; version not
// pinned by the reference, CMakeLists.txt:7-10):
//   ggml_mul_mat(a, b)  dst[i1][i0] = sum_k a[i0][k] * b[i1][k]   (a: ne0 = K,
//                       ne1 = N; b: ne0 = K, ne1 = M; dst: ne0 = N, ne1 = M),
//                       a's dims 2/3 broadcast over b's
//   ggml_add / ggml_mul elementwise, b repeated over a (a.ne[i] % b.ne[i] == 0)
//   ggml_rms_norm       per ne0-row: sum of x*x in double, mean as float,
//                       y = x * (1 / sqrtf(mean + eps))
//   ggml_silu           x / (1 + expf(-x))
//   ggml_rope mode 0    pairs (i0, i0+1) of each head rotated by theta_i0 =
//                       p * base^(-i0/n_dims), theta advanced by repeated
//                       multiplication with powf(base, -2/n_dims) from p,
//                       base 10000, cosf/sinf; NEOX (mode 2) pairs (i, i + n_dims/2)
//   ggml_permute        ne[axis_i] = a.ne[i], nb[axis_i] = a.nb[i] (a view)
//   reshape / view      views of the same bytes; cont copies to row-major
// Every operator evaluates immediately; ggml_graph_compute_with_ctx does
// nothing.  The reference reads node data only after computing the graph that
// produces it, so eager evaluation returns the values deferred evaluation
// would.
#include "ggml.h"
#include "ggml-cpu.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

struct ggml_context {
    std::vector<ggml_tensor *> tensors;
    std::vector<void *> buffers;
};

struct ggml_cgraph {
    int unused;
};

namespace {

ggml_cgraph g_graph_token = {0};

[[noreturn]] void fail(const char *what) {
    std::fprintf(stderr, "ggml stand-in: %s\n", what);
    std::abort();
}

size_t elsize(ggml_type t) { return t == GGML_TYPE_I32 ? sizeof(int32_t) : sizeof(float); }

char *base(const ggml_tensor *t) { return (char *)t->data + t->view_offs; }

ggml_tensor *header(ggml_context *ctx, ggml_type type, const int64_t ne[4]) {
    ggml_tensor *t = new ggml_tensor();
    t->type = type;
    for (int i = 0; i < 4; i++) t->ne[i] = ne[i];
    t->nb[0] = elsize(type);
    for (int i = 1; i < 4; i++) t->nb[i] = t->nb[i - 1] * (size_t)t->ne[i - 1];
    t->data = nullptr;
    t->view_offs = 0;
    ctx->tensors.push_back(t);
    return t;
}

ggml_tensor *new_tensor(ggml_context *ctx, ggml_type type, const int64_t ne[4]) {
    ggml_tensor *t = header(ctx, type, ne);
    const size_t bytes = t->nb[3] * (size_t)t->ne[3];
    void *p = std::calloc(bytes ? bytes : 1, 1);
    if (!p) fail("out of memory");
    ctx->buffers.push_back(p);
    t->data = p;
    return t;
}

int64_t nelements(const ggml_tensor *t) { return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]; }

bool contiguous(const ggml_tensor *t) {
    size_t s = elsize(t->type);
    for (int i = 0; i < 4; i++) {
        if (t->ne[i] > 1 && t->nb[i] != s) return false;
        s *= (size_t)t->ne[i];
    }
    return true;
}

float &at(const ggml_tensor *t, int64_t i0, int64_t i1, int64_t i2, int64_t i3) {
    return *(float *)(base(t) + i0 * t->nb[0] + i1 * t->nb[1] + i2 * t->nb[2] + i3 * t->nb[3]);
}

ggml_tensor *view_of(ggml_context *ctx, ggml_tensor *a, const int64_t ne[4]) {
    if (!contiguous(a)) fail("reshape of a non-contiguous tensor");
    int64_t n = ne[0] * ne[1] * ne[2] * ne[3];
    if (n != nelements(a)) fail("reshape changes the element count");
    ggml_tensor *t = header(ctx, a->type, ne);
    t->data = base(a);
    return t;
}

template <class F>
ggml_tensor *binary(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b, F op) {
    for (int i = 0; i < 4; i++)
        if (b->ne[i] == 0 || a->ne[i] % b->ne[i] != 0) fail("operand cannot be repeated over the other");
    ggml_tensor *d = new_tensor(ctx, GGML_TYPE_F32, a->ne);
    for (int64_t i3 = 0; i3 < a->ne[3]; i3++)
        for (int64_t i2 = 0; i2 < a->ne[2]; i2++)
            for (int64_t i1 = 0; i1 < a->ne[1]; i1++)
                for (int64_t i0 = 0; i0 < a->ne[0]; i0++)
                    at(d, i0, i1, i2, i3) = op(at(a, i0, i1, i2, i3),
                                               at(b, i0 % b->ne[0], i1 % b->ne[1], i2 % b->ne[2], i3 % b->ne[3]));
    return d;
}

template <class F>
ggml_tensor *unary(ggml_context *ctx, ggml_tensor *a, F op) {
    ggml_tensor *d = new_tensor(ctx, GGML_TYPE_F32, a->ne);
    for (int64_t i3 = 0; i3 < a->ne[3]; i3++)
        for (int64_t i2 = 0; i2 < a->ne[2]; i2++)
            for (int64_t i1 = 0; i1 < a->ne[1]; i1++)
                for (int64_t i0 = 0; i0 < a->ne[0]; i0++) at(d, i0, i1, i2, i3) = op(at(a, i0, i1, i2, i3));
    return d;
}

}  // namespace

extern "C" {

ggml_context *ggml_init(ggml_init_params) { return new ggml_context(); }

void ggml_reset(ggml_context *ctx) {
    for (ggml_tensor *t : ctx->tensors) delete t;
    for (void *p : ctx->buffers) std::free(p);
    ctx->tensors.clear();
    ctx->buffers.clear();
}

void ggml_free(ggml_context *ctx) {
    if (!ctx) return;
    ggml_reset(ctx);
    delete ctx;
}

ggml_tensor *ggml_new_tensor_1d(ggml_context *ctx, ggml_type type, int64_t ne0) {
    const int64_t ne[4] = {ne0, 1, 1, 1};
    return new_tensor(ctx, type, ne);
}

ggml_tensor *ggml_new_tensor_2d(ggml_context *ctx, ggml_type type, int64_t ne0, int64_t ne1) {
    const int64_t ne[4] = {ne0, ne1, 1, 1};
    return new_tensor(ctx, type, ne);
}

ggml_tensor *ggml_reshape_2d(ggml_context *ctx, ggml_tensor *a, int64_t ne0, int64_t ne1) {
    const int64_t ne[4] = {ne0, ne1, 1, 1};
    return view_of(ctx, a, ne);
}

ggml_tensor *ggml_reshape_3d(ggml_context *ctx, ggml_tensor *a, int64_t ne0, int64_t ne1, int64_t ne2) {
    const int64_t ne[4] = {ne0, ne1, ne2, 1};
    return view_of(ctx, a, ne);
}

ggml_tensor *ggml_view_2d(ggml_context *ctx, ggml_tensor *a, int64_t ne0, int64_t ne1, size_t nb1, size_t offset) {
    const int64_t ne[4] = {ne0, ne1, 1, 1};
    ggml_tensor *t = header(ctx, a->type, ne);
    t->nb[0] = a->nb[0];
    t->nb[1] = nb1;
    t->nb[2] = t->nb[3] = nb1 * (size_t)ne1;
    t->data = base(a) + offset;
    return t;
}

ggml_tensor *ggml_permute(ggml_context *ctx, ggml_tensor *a, int axis0, int axis1, int axis2, int axis3) {
    const int ax[4] = {axis0, axis1, axis2, axis3};
    int seen = 0;
    for (int i = 0; i < 4; i++) {
        if (ax[i] < 0 || ax[i] > 3 || (seen >> ax[i]) & 1) fail("permute axes are not a permutation");
        seen |= 1 << ax[i];
    }
    const int64_t one[4] = {1, 1, 1, 1};
    ggml_tensor *t = header(ctx, a->type, one);
    for (int i = 0; i < 4; i++) {
        t->ne[ax[i]] = a->ne[i];
        t->nb[ax[i]] = a->nb[i];
    }
    t->data = base(a);
    return t;
}

ggml_tensor *ggml_cont(ggml_context *ctx, ggml_tensor *a) {
    return unary(ctx, a, [](float x) { return x; });
}

ggml_tensor *ggml_mul_mat(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b) {
    if (a->ne[0] != b->ne[0]) fail("mul_mat: inner dimensions differ");
    if (b->ne[2] % a->ne[2] || b->ne[3] % a->ne[3]) fail("mul_mat: batch dimensions cannot broadcast");
    const int64_t K = a->ne[0], N = a->ne[1], M = b->ne[1];
    const int64_t ne[4] = {N, M, b->ne[2], b->ne[3]};
    ggml_tensor *d = new_tensor(ctx, GGML_TYPE_F32, ne);
    const int64_t r2 = b->ne[2] / a->ne[2], r3 = b->ne[3] / a->ne[3];
    for (int64_t i3 = 0; i3 < b->ne[3]; i3++)
        for (int64_t i2 = 0; i2 < b->ne[2]; i2++) {
#pragma omp parallel for collapse(2) schedule(static)
            for (int64_t i1 = 0; i1 < M; i1++)
                for (int64_t i0 = 0; i0 < N; i0++) {
                    float s = 0.0f;
                    if (a->nb[0] == sizeof(float) && b->nb[0] == sizeof(float)) {
                        const float *ar = &at(a, 0, i0, i2 / r2, i3 / r3);
                        const float *br = &at(b, 0, i1, i2, i3);
                        for (int64_t k = 0; k < K; k++) s += ar[k] * br[k];
                    } else {
                        for (int64_t k = 0; k < K; k++) s += at(a, k, i0, i2 / r2, i3 / r3) * at(b, k, i1, i2, i3);
                    }
                    at(d, i0, i1, i2, i3) = s;
                }
        }
    return d;
}

ggml_tensor *ggml_add(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b) {
    return binary(ctx, a, b, [](float x, float y) { return x + y; });
}

ggml_tensor *ggml_mul(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b) {
    return binary(ctx, a, b, [](float x, float y) { return x * y; });
}

ggml_tensor *ggml_rms_norm(ggml_context *ctx, ggml_tensor *a, float eps) {
    ggml_tensor *d = new_tensor(ctx, GGML_TYPE_F32, a->ne);
    for (int64_t i3 = 0; i3 < a->ne[3]; i3++)
        for (int64_t i2 = 0; i2 < a->ne[2]; i2++)
            for (int64_t i1 = 0; i1 < a->ne[1]; i1++) {
                double sum = 0.0;
                for (int64_t i0 = 0; i0 < a->ne[0]; i0++) {
                    const float x = at(a, i0, i1, i2, i3);
                    sum += (double)(x * x);
                }
                const float mean = (float)(sum / (double)a->ne[0]);
                const float scale = 1.0f / sqrtf(mean + eps);
                for (int64_t i0 = 0; i0 < a->ne[0]; i0++) at(d, i0, i1, i2, i3) = at(a, i0, i1, i2, i3) * scale;
            }
    return d;
}

ggml_tensor *ggml_silu(ggml_context *ctx, ggml_tensor *a) {
    return unary(ctx, a, [](float x) { return x / (1.0f + expf(-x)); });
}

ggml_tensor *ggml_rope(ggml_context *ctx, ggml_tensor *a, ggml_tensor *pos, int n_dims, int mode) {
    if (pos->type != GGML_TYPE_I32 || pos->ne[0] != a->ne[2]) fail("rope: one position per row of dimension 2");
    if (n_dims > a->ne[0] || (n_dims & 1)) fail("rope: bad n_dims");
    const bool neox = (mode & 2) != 0;
    const float theta_scale = powf(10000.0f, -2.0f / (float)n_dims);
    ggml_tensor *d = ggml_cont(ctx, a);
    std::vector<float> cs(n_dims), sn(n_dims);
    for (int64_t i3 = 0; i3 < a->ne[3]; i3++)
        for (int64_t i2 = 0; i2 < a->ne[2]; i2++) {
            const int32_t p = ((const int32_t *)base(pos))[i2];
            float theta = (float)p;
            for (int i0 = 0; i0 < n_dims; i0 += 2) {
                cs[i0] = cosf(theta);
                sn[i0] = sinf(theta);
                theta *= theta_scale;
            }
            for (int64_t i1 = 0; i1 < a->ne[1]; i1++)
                for (int i0 = 0; i0 < n_dims; i0 += 2) {
                    const int64_t j0 = neox ? i0 / 2 : i0;
                    const int64_t j1 = neox ? i0 / 2 + n_dims / 2 : i0 + 1;
                    const float x0 = at(a, j0, i1, i2, i3), x1 = at(a, j1, i1, i2, i3);
                    at(d, j0, i1, i2, i3) = x0 * cs[i0] - x1 * sn[i0];
                    at(d, j1, i1, i2, i3) = x0 * sn[i0] + x1 * cs[i0];
                }
        }
    return d;
}

ggml_cgraph *ggml_new_graph(ggml_context *) { return &g_graph_token; }

void ggml_build_forward_expand(ggml_cgraph *, ggml_tensor *) {}

int ggml_graph_compute_with_ctx(ggml_context *, ggml_cgraph *, int) { return 0; }

}  // extern "C"
