/* Stand-in for ggml-cpu.h: the graph compute entry point the reference's
 * PatchEncoder calls (src/modules/backbone/patchenc.cpp:119,157,184,221,237).
 * With the eager operators of shim/ggml_eager.cpp there is nothing left to
 * compute, so it only returns success.  include/dit_manual.h includes this
 * header but uses nothing from it.  Test infrastructure only. */
#pragma once
#include "ggml.h"

#ifdef __cplusplus
extern "C" {
#endif
int ggml_graph_compute_with_ctx(struct ggml_context *ctx, struct ggml_cgraph *cgraph, int n_threads);
#ifdef __cplusplus
}
#endif
