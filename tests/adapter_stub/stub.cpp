// Test stand-ins around the op-hook adapter: the ggml fork's hook registrar
// (it only records the installed function pointers) and the reference
// megakernel's two hooks (they count the calls that reach them and claim
// nothing), plus entry points through which a test invokes the installed
// hooks the way ggml-cuda's node loop does.  Test infrastructure only.
#include "ggml.h"

#include <cuda_runtime.h>

struct ggml_backend_cuda_context;
struct ggml_cgraph;

extern "C" {
typedef bool (*ggml_cuda_op_hook_fn)(ggml_backend_cuda_context*, ggml_tensor*, cudaStream_t);
typedef void (*ggml_cuda_graph_begin_hook_fn)(ggml_backend_cuda_context*, const ggml_cgraph*);

static ggml_cuda_op_hook_fn g_op = nullptr;
static ggml_cuda_graph_begin_hook_fn g_begin = nullptr;
static int g_ref_op_calls = 0;
static int g_ref_begin_calls = 0;

void ggml_cuda_set_op_hook(ggml_cuda_op_hook_fn fn) { g_op = fn; }
void ggml_cuda_set_graph_begin_hook(ggml_cuda_graph_begin_hook_fn fn) { g_begin = fn; }

bool ggml_is_contiguous(const ggml_tensor* t) {
    const size_t es = t->type == GGML_TYPE_F32 ? 4 : 2;
    return t->nb[0] == es && t->nb[1] == t->nb[0] * t->ne[0] && t->nb[2] == t->nb[1] * t->ne[1] &&
           t->nb[3] == t->nb[2] * t->ne[2];
}

bool siglip2_op_hook(ggml_backend_cuda_context*, ggml_tensor*, cudaStream_t) {
    ++g_ref_op_calls;
    return false;
}
void siglip2_graph_begin_hook(ggml_backend_cuda_context*, const ggml_cgraph*) { ++g_ref_begin_calls; }

int stub_installed(void) { return g_op != nullptr && g_begin != nullptr; }
int stub_run_op(ggml_tensor* dst, void* stream) { return g_op(nullptr, dst, static_cast<cudaStream_t>(stream)) ? 1 : 0; }
void stub_run_begin(void) { g_begin(nullptr, nullptr); }
int stub_ref_op_calls(void) { return g_ref_op_calls; }
int stub_ref_begin_calls(void) { return g_ref_begin_calls; }
size_t stub_tensor_size(void) { return sizeof(ggml_tensor); }
}
