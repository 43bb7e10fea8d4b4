// b2q_ggml_hook.cpp — ggml-cuda op hook that routes hbd-siglip2.cpp's
// Q8_0 x F32 mul_mat nodes to libb2q and hands every other node to the
// reference's own megakernel hook.
//
// Build this file inside hbd-siglip2.cpp, next to src/cuda/siglip2_megakernel.cu,
// against its ggml fork (the fork exports ggml_cuda_set_op_hook and
// ggml_cuda_set_graph_begin_hook, declared at src/cuda/siglip2_megakernel.cuh:16-33)
// and link libb2q.so.  This repository's tests build it against a stand-in
// ggml.h and a stub hook registrar (tests/adapter_stub/) and execute it.
//
// The fork has ONE op-hook slot and one graph-begin slot, and
// siglip2_megakernel::install() fills both with siglip2_op_hook and
// siglip2_graph_begin_hook (src/cuda/siglip2_megakernel.cu:1403-1404).  So
// b2q_ggml_install() must run after install(): it takes both slots and
// chains.  For every node ggml-cuda offers:
//   * GGML_OP_MUL_MAT with a Q8_0 weight (src0, K a multiple of 32) and a
//     contiguous F32 activation (src1): enqueued on ggml's stream through
//     b2q_mul_mat_q8_0_f32, return true (the reference's op hook has no
//     MUL_MAT branch, so nothing of the megakernel's is bypassed: its tail
//     anchors read this node's output as before);
//   * anything else, or a mul_mat this library cannot take: forwarded to
//     siglip2_op_hook, whose answer is returned (false lets ggml run its own
//     kernel: the fallback contract of src/cuda/siglip2_megakernel.cu:1186-1189).
// The graph-begin hook forwards to siglip2_graph_begin_hook unchanged (the
// megakernel's pattern plans, src/cuda/siglip2_megakernel.cu:1124-1131).
// Both reference hooks are declared weak: without the megakernel the adapter
// still links and forwards nothing.
//
// Weights are registered (repacked) the first time each weight tensor is
// seen, keyed by its device pointer, which is stable for an encoder's
// lifetime (src/siglip2_vision.cpp:362-409).  An encoder unload frees those
// buffers and a reload may reuse the addresses (src/siglip2_server.cpp:287-308),
// so the unload path must call b2q_ggml_release_weights() first; the cache
// also remembers the generation it was filled in and drops stale entries.
#include "b2q.h"

#include "ggml.h"

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <mutex>
#include <thread>
#include <unordered_map>

struct ggml_backend_cuda_context;
struct ggml_cgraph;
extern "C" {
typedef bool (*ggml_cuda_op_hook_fn)(ggml_backend_cuda_context* ctx, ggml_tensor* dst, cudaStream_t stream);
typedef void (*ggml_cuda_graph_begin_hook_fn)(ggml_backend_cuda_context* ctx, const ggml_cgraph* cgraph);
void ggml_cuda_set_op_hook(ggml_cuda_op_hook_fn fn);
void ggml_cuda_set_graph_begin_hook(ggml_cuda_graph_begin_hook_fn fn);
// the reference's hooks (src/cuda/siglip2_megakernel.cu:1124,1152)
__attribute__((weak)) bool siglip2_op_hook(ggml_backend_cuda_context* ctx, ggml_tensor* dst, cudaStream_t stream);
__attribute__((weak)) void siglip2_graph_begin_hook(ggml_backend_cuda_context* ctx, const ggml_cgraph* cgraph);
}

namespace {

struct Entry {
    b2q_weight* w;
    uint64_t generation;
    int64_t N, K, row_bytes;
};

std::mutex g_mutex;
std::unordered_map<const void*, Entry> g_weights;   // keyed by src0->data
std::atomic<uint64_t> g_generation{1};

// Activation scratch: registered by each encoder thread (b2q_ggml_set_scratch)
// before its first graph, like the megakernel's per-thread scratch
// (src/siglip2_megakernel.h:32-44).
thread_local void* t_scratch = nullptr;
thread_local size_t t_scratch_bytes = 0;

// Without registered scratch, a node whose q8_1 planes fit the library's
// fixed device array may use b2q_mul_mat_q8_0_f32_noalloc.  That array is
// shared by every call on a device, so only the first host thread that
// takes this path on a device may use it; any other thread without scratch
// gets `false` and ggml computes the node.
constexpr int kMaxDevices = 64;
std::atomic<std::thread::id> g_noalloc_owner[kMaxDevices];

bool may_use_noalloc() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return false;
    const std::thread::id me = std::this_thread::get_id();
    std::thread::id none{};
    if (g_noalloc_owner[dev].compare_exchange_strong(none, me)) return true;
    return none == me;
}

b2q_weight* weight_for(const ggml_tensor* w, cudaStream_t stream) {
    std::lock_guard<std::mutex> lk(g_mutex);
    const uint64_t gen = g_generation.load();
    // ne0 = K (innermost), ne1 = N rows, nb1 = bytes per row of blocks
    const int64_t N = w->ne[1], K = w->ne[0], row_bytes = static_cast<int64_t>(w->nb[1]);
    auto it = g_weights.find(w->data);
    if (it != g_weights.end()) {
        const Entry& e = it->second;
        if (e.generation == gen && e.N == N && e.K == K && e.row_bytes == row_bytes) return e.w;
        b2q_weight_release(e.w);   // registered before an unload, or another tensor now lives here
        g_weights.erase(it);
    }
    b2q_weight* h = nullptr;
    if (b2q_weight_register(w->data, N, K, row_bytes, 0, stream, &h) != B2Q_OK) return nullptr;
    g_weights.emplace(w->data, Entry{h, gen, N, K, row_bytes});
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

bool run_mul_mat(ggml_tensor* dst, cudaStream_t stream) {
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
    else if (need <= B2Q_NOALLOC_MAX_SCRATCH_BYTES && may_use_noalloc())
        st = b2q_mul_mat_q8_0_f32_noalloc(h, static_cast<const float*>(x->data), M, x_cols,
                                          static_cast<float*>(dst->data), stream);
    else
        return false;   // no usable scratch: ggml computes the node
    return st == B2Q_OK;
}

bool b2q_op_hook(ggml_backend_cuda_context* ctx, ggml_tensor* dst, cudaStream_t stream) {
    if (dst && claim(dst) && run_mul_mat(dst, stream)) return true;
    return siglip2_op_hook ? siglip2_op_hook(ctx, dst, stream) : false;
}

void b2q_graph_begin_hook(ggml_backend_cuda_context* ctx, const ggml_cgraph* cgraph) {
    if (siglip2_graph_begin_hook) siglip2_graph_begin_hook(ctx, cgraph);
}

}  // namespace

extern "C" {

// Installs both hooks, chaining to the reference's; call once per process,
// after siglip2_megakernel::install() (src/siglip2_megakernel.h:27), after
// b2q_init on each device the encoders use, and before the first graph.
bool b2q_ggml_install(int device) {
    if (b2q_init(device, -1) != B2Q_OK) return false;
    ggml_cuda_set_graph_begin_hook(&b2q_graph_begin_hook);
    ggml_cuda_set_op_hook(&b2q_op_hook);
    return true;
}

// Per-host-thread activation scratch (device memory of at least
// b2q_act_bytes(max tokens, max K) bytes, owned by the caller).  Every host
// thread that runs an encoder on a GPU shared with another encoder thread
// must register its own.
void b2q_ggml_set_scratch(void* scratch, size_t bytes) {
    t_scratch = scratch;
    t_scratch_bytes = bytes;
}

// Releases every weight registered by the hook.  Call it from the encoder
// unload path before the weight buffers are freed (ServerState::unload,
// src/siglip2_server.cpp:287-308); entries registered before it are never
// used again even if a reload reuses the same addresses.
void b2q_ggml_release_weights(void) {
    std::lock_guard<std::mutex> lk(g_mutex);
    for (auto& kv : g_weights) b2q_weight_release(kv.second.w);
    g_weights.clear();
    g_generation.fetch_add(1);
}

}  // extern "C"
