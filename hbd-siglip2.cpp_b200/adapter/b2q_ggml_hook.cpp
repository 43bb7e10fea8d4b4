// b2q_ggml_hook.cpp — ggml-cuda op hook that routes hbd-siglip2.cpp's
// Q8_0 x F32 mul_mat nodes to libb2q.
//
// Build this file inside hbd-siglip2.cpp, next to src/cuda/siglip2_megakernel.cu,
// against its ggml fork (the fork exports ggml_cuda_set_op_hook, declared at
// src/cuda/siglip2_megakernel.cuh:16-33) and link libb2q.so.  It needs
// ggml.h, which this repository does not carry (the reference's ggml
// submodule is empty here), so it is not compiled by this repository's build.
//
// What it does: ggml-cuda calls the hook for every graph node before running
// its own kernel; the hook claims GGML_OP_MUL_MAT nodes with a Q8_0 weight
// (src0, ne0 = K a multiple of 32) and a contiguous F32 activation (src1),
// enqueues b2q_mul_mat_q8_0_f32 on ggml's stream and returns true; anything
// else returns false and ggml runs its own kernel (the reference's fallback
// contract, src/cuda/siglip2_megakernel.cu:1186-1189).  Weights are
// registered (repacked) the first time each weight tensor is seen, keyed by
// its device pointer, which is stable for an encoder's lifetime
// (src/siglip2_vision.cpp:362-409).  The fused tails (bias, GELU, residual,
// next LayerNorm) stay ggml nodes here; the fused path is the library's own
// tower driver (b2q_vision_*, b2q_text_*).
#include "b2q.h"

#include "ggml.h"

#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <unordered_map>

struct ggml_backend_cuda_context;
extern "C" {
typedef bool (*ggml_cuda_op_hook_fn)(ggml_backend_cuda_context* ctx, ggml_tensor* dst, cudaStream_t stream);
void ggml_cuda_set_op_hook(ggml_cuda_op_hook_fn fn);
}

namespace {

std::mutex g_mutex;
std::unordered_map<const void*, b2q_weight*> g_weights;   // keyed by src0->data

// Activation scratch: set by the encoder (b2q_ggml_set_scratch) before its
// first graph, per host thread, like the megakernel's registered scratch
// (src/siglip2_megakernel.h:32-44).  Without it, shapes whose q8_1 planes fit
// the library's fixed device array use b2q_mul_mat_q8_0_f32_noalloc.
thread_local void* t_scratch = nullptr;
thread_local size_t t_scratch_bytes = 0;

b2q_weight* weight_for(const ggml_tensor* w, cudaStream_t stream) {
    std::lock_guard<std::mutex> lk(g_mutex);
    auto it = g_weights.find(w->data);
    if (it != g_weights.end()) return it->second;
    b2q_weight* h = nullptr;
    // ne0 = K (innermost), ne1 = N rows, nb1 = bytes per row of blocks
    if (b2q_weight_register(w->data, w->ne[1], w->ne[0], static_cast<int64_t>(w->nb[1]), 0, stream, &h) != B2Q_OK)
        return nullptr;
    g_weights.emplace(w->data, h);
    return h;
}

bool claim(const ggml_tensor* dst) {
    if (dst->op != GGML_OP_MUL_MAT) return false;
    const ggml_tensor* w = dst->src[0];
    const ggml_tensor* x = dst->src[1];
    if (!w || !x || w->type != GGML_TYPE_Q8_0 || x->type != GGML_TYPE_F32 || dst->type != GGML_TYPE_F32) return false;
    if (w->ne[0] % 32 != 0 || w->ne[1] % 4 != 0 || w->ne[2] != 1 || w->ne[3] != 1) return false;
    if (!ggml_is_contiguous(x) || !ggml_is_contiguous(dst) || x->ne[2] != 1 || x->ne[3] != 1) return false;
    // X may be narrower than the padded weight (4304 vs 4320): the quantizer
    // zero-extends it, which is the reference's pad_x_to_w (siglip2_vision.cpp:99-107)
    return x->ne[0] <= w->ne[0] && x->ne[0] > w->ne[0] - 32;
}

bool b2q_op_hook(ggml_backend_cuda_context* /*ctx*/, ggml_tensor* dst, cudaStream_t stream) {
    if (!claim(dst)) return false;
    const ggml_tensor* w = dst->src[0];
    const ggml_tensor* x = dst->src[1];
    b2q_weight* h = weight_for(w, stream);
    if (!h) return false;
    const int64_t M = x->ne[1], x_cols = x->ne[0];
    const size_t need = b2q_act_bytes(M, w->ne[0]);
    b2q_status st;
    if (t_scratch && need <= t_scratch_bytes)
        st = b2q_mul_mat_q8_0_f32(h, static_cast<const float*>(x->data), M, x_cols, static_cast<float*>(dst->data),
                                  t_scratch, stream);
    else if (need <= B2Q_NOALLOC_MAX_SCRATCH_BYTES)
        st = b2q_mul_mat_q8_0_f32_noalloc(h, static_cast<const float*>(x->data), M, x_cols,
                                          static_cast<float*>(dst->data), stream);
    else
        return false;   // no scratch large enough: ggml computes the node
    return st == B2Q_OK;
}

}  // namespace

extern "C" {

// Installs the hook; call once per process, after b2q_init on each device the
// encoders use and before the first graph (mirrors siglip2_megakernel::install,
// src/siglip2_megakernel.h:27).
bool b2q_ggml_install(int device) {
    if (b2q_init(device, -1) != B2Q_OK) return false;
    ggml_cuda_set_op_hook(&b2q_op_hook);
    return true;
}

// Per-host-thread activation scratch (device memory of at least
// b2q_act_bytes(max tokens, max K) bytes, owned by the caller).
void b2q_ggml_set_scratch(void* scratch, size_t bytes) {
    t_scratch = scratch;
    t_scratch_bytes = bytes;
}

// Releases every weight registered by the hook (after the encoders are gone).
void b2q_ggml_release_weights(void) {
    std::lock_guard<std::mutex> lk(g_mutex);
    for (auto& kv : g_weights) b2q_weight_release(kv.second);
    g_weights.clear();
}

}  // extern "C"
