/* Minimal stand-in for ggml.h, enough for the reference's public headers
 * (include/dit.h, include/patchenc.h, include/dots_tts_util.h) and for the
 * drop-in's patchenc_forward, which returns its result as a new 2-D tensor
 * of the caller's context.  Test infrastructure for tests/cpp/dropin_test.cpp:
 * a real build uses ggml's own header; the fields kept here (ne, data,
 * view_offs) have ggml's meaning. */
#pragma once
#include <stddef.h>
#include <stdint.h>

enum ggml_type { GGML_TYPE_F32 = 0 };

struct ggml_context;
struct ggml_backend_buffer;

struct ggml_tensor {
    enum ggml_type type;
    int64_t ne[4];
    void *data;
    size_t view_offs;
};

struct ggml_tensor *ggml_new_tensor_2d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0, int64_t ne1);
