/* Minimal stand-in for ggml.h so that the reference's header-only DiT math
 * (include/dit_manual.h, include/dit.h, include/dots_tts_util.h) compiles
 * without ggml.  Only the fields those headers touch exist: `data` and
 * `view_offs` (read by tensor_data(), dots_tts_util.h:10-12) and `ne`.
 * Test infrastructure only: nothing in the product links this. */
#pragma once
#include <stddef.h>
#include <stdint.h>

struct ggml_context;
struct ggml_backend_buffer;

struct ggml_tensor {
    int64_t ne[4];
    void *  data;
    size_t  view_offs;
};
