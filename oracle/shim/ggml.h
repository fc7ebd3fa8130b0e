/* Stand-in for ggml.h so that the reference's CPU code compiles without ggml
 * (ggml / llama.cpp is a sibling checkout the reference does not vendor).
 *
 * Two uses, both test infrastructure (nothing in the product links this):
 *  - the header-only DiT math (include/dit_manual.h, include/dit.h,
 *    include/dots_tts_util.h) touches only `data` and `view_offs` (read by
 *    tensor_data(), dots_tts_util.h:10-12);
 *  - the PatchEncoder (src/modules/backbone/patchenc.cpp) builds its layers
 *    from ggml operators.  shim/ggml_eager.cpp defines the operators it calls,
 *    restated from ggml's published semantics and evaluated EAGERLY: each
 *    operator computes its result when it is created, and graph building and
 *    graph compute do nothing.  patchenc.cpp reads a node's data only after
 *    computing the graph that produces it (:118-119, :157, :182-184, :220-221,
 *    :236-237), so eager and deferred evaluation give the same values there.
 *
 * Field meanings follow ggml: ne[i] elements along dimension i (ne[0]
 * fastest), nb[i] the byte stride of dimension i. */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum ggml_type { GGML_TYPE_F32 = 0, GGML_TYPE_I32 = 26 };

struct ggml_context;
struct ggml_backend_buffer;
struct ggml_cgraph;

struct ggml_tensor {
    enum ggml_type type;
    int64_t ne[4];
    size_t  nb[4];
    void *  data;
    size_t  view_offs;
};

struct ggml_init_params {
    size_t mem_size;
    void * mem_buffer;
    int    no_alloc;
};

struct ggml_context *ggml_init(struct ggml_init_params params);
void ggml_free(struct ggml_context *ctx);
void ggml_reset(struct ggml_context *ctx);

struct ggml_tensor *ggml_new_tensor_1d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0);
struct ggml_tensor *ggml_new_tensor_2d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0, int64_t ne1);
struct ggml_tensor *ggml_reshape_2d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1);
struct ggml_tensor *ggml_reshape_3d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                    int64_t ne2);
struct ggml_tensor *ggml_view_2d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                 size_t nb1, size_t offset);
struct ggml_tensor *ggml_permute(struct ggml_context *ctx, struct ggml_tensor *a, int axis0, int axis1, int axis2,
                                 int axis3);
struct ggml_tensor *ggml_cont(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_mul_mat(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_add(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_mul(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_rms_norm(struct ggml_context *ctx, struct ggml_tensor *a, float eps);
struct ggml_tensor *ggml_silu(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_rope(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *pos, int n_dims,
                              int mode);

struct ggml_cgraph *ggml_new_graph(struct ggml_context *ctx);
void ggml_build_forward_expand(struct ggml_cgraph *cgraph, struct ggml_tensor *tensor);

#ifdef __cplusplus
}
#endif
