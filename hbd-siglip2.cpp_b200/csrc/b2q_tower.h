// b2q_tower.h — pieces shared by the vision and text tower drivers: device
// buffers, the named tensor set a tower loads (GGUF names, ggml types) and
// the pre-LN encoder block sequence both towers run
// (src/siglip2_vision.cpp:181-244, src/siglip2_text.cpp:108-190).
#pragma once

#include "b2q_internal.h"

#include <cuda_fp16.h>

#include <map>
#include <string>
#include <vector>

namespace b2q {

struct DevBuf {
    void* p = nullptr;
    size_t n = 0;
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    cudaError_t ensure(size_t bytes) {
        if (bytes <= n) return cudaSuccess;
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
        cudaError_t e = cudaMalloc(&p, bytes);
        if (e == cudaSuccess) n = bytes;
        return e;
    }
    template <class T>
    T* as() const {
        return static_cast<T*>(p);
    }
};

// Tensors of one tower by GGUF name: Q8_0 projections registered for the
// GEMM, F32 tensors uploaded as they are, and Q8_0 tables that are gathered
// row by row (token embeddings) kept as raw ggml blocks.
struct TensorSet {
    std::map<std::string, b2q_weight*> q8;
    std::map<std::string, DevBuf> f32;
    std::map<std::string, DevBuf> raw_q8;
    ~TensorSet() {
        for (auto& kv : q8) b2q_weight_release(kv.second);
    }
    const float* f(const std::string& n) const {
        auto it = f32.find(n);
        return it == f32.end() ? nullptr : it->second.as<float>();
    }
    const b2q_weight* w(const std::string& n) const {
        auto it = q8.find(n);
        return it == q8.end() ? nullptr : it->second;
    }
    const uint8_t* raw(const std::string& n) const {
        auto it = raw_q8.find(n);
        return it == raw_q8.end() ? nullptr : it->second.as<uint8_t>();
    }
    // ggml_type 0 (F32) or 8 (Q8_0, ne0 = K innermost, ne1 = rows); as_raw
    // keeps a Q8_0 tensor as blocks instead of registering it for the GEMM.
    b2q_status put(const std::string& name, int32_t ggml_type, const void* host_data, int64_t ne0, int64_t ne1,
                   bool as_raw, cudaStream_t s);
};

#define B2Q_TRY(expr)                    \
    do {                                 \
        b2q_status _st = (expr);         \
        if (_st != B2Q_OK) return _st;   \
    } while (0)

b2q_status gemm(const b2q_weight* w, const void* act, int64_t M, void* y, int kind, const float* bias,
                const float* residual, void* act_out, int64_t ld_out, cudaStream_t s);

// A tower's encodes replayed as CUDA graphs.  A key names everything the
// launches depend on (batch geometry, input and output addresses, buffer and
// weight addresses through the tower's generation, the device's settings
// through b2q_tune's generation).  The first call with a key launches the
// kernels one by one; the second captures them on the tower's own stream (so
// the caller's stream may be the legacy default one) and every later call
// launches the captured graph on the caller's stream.  Up to kEntries keys
// are kept (the pipelined host entry point alternates between two input
// buffers); the least recently used one is dropped.  A capture that the
// runtime refuses falls back to direct launches.
struct EncodeGraph {
    static constexpr int kEntries = 4;
    struct Entry {
        std::vector<int64_t> key;
        cudaGraphExec_t exec = nullptr;   // null: the key has run once without a graph
        uint64_t kernels = 0;             // library kernels in the graph
        uint64_t used = 0;
    };
    std::vector<Entry> entries;
    uint64_t clock = 0;
    cudaStream_t capture = nullptr;
    EncodeGraph() = default;
    EncodeGraph(const EncodeGraph&) = delete;
    EncodeGraph& operator=(const EncodeGraph&) = delete;
    ~EncodeGraph() {
        forget();
        if (capture) cudaStreamDestroy(capture);
    }
    void forget() {
        for (Entry& e : entries)
            if (e.exec) cudaGraphExecDestroy(e.exec);
        entries.clear();
    }
    Entry* find(const std::vector<int64_t>& key) {
        for (Entry& e : entries)
            if (e.key == key) return &e;
        return nullptr;
    }
    Entry& add(const std::vector<int64_t>& key) {
        if (static_cast<int>(entries.size()) == kEntries) {
            size_t lru = 0;
            for (size_t i = 1; i < entries.size(); ++i)
                if (entries[i].used < entries[lru].used) lru = i;
            if (entries[lru].exec) cudaGraphExecDestroy(entries[lru].exec);
            entries.erase(entries.begin() + static_cast<long>(lru));
        }
        entries.push_back(Entry{key, nullptr, 0, ++clock});
        return entries.back();
    }
};

// Runs `issue(stream)` (kernel launches only: no allocation, copy or
// synchronisation) through `g`.
template <class Issue>
b2q_status run_graphed(EncodeGraph& g, const std::vector<int64_t>& key, cudaStream_t s, Issue&& issue) {
    DeviceState* ds = state();
    if (!ds->graphs) {
        g.forget();
        return issue(s);
    }
    // a caller that is capturing its own graph on `s` records the kernels itself
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
        (void) cudaGetLastError();
        return issue(s);
    }
    EncodeGraph::Entry* e = g.find(key);
    if (e && e->exec) {
        e->used = ++g.clock;
        add_launches(static_cast<int64_t>(e->kernels));
        count_graph_launch();
        return cuda_check(cudaGraphLaunch(e->exec, s), "graph launch");
    }
    if (!e) {
        g.add(key);
        return issue(s);
    }
    e->used = ++g.clock;
    if (!g.capture && cudaStreamCreateWithFlags(&g.capture, cudaStreamNonBlocking) != cudaSuccess) {
        (void) cudaGetLastError();
        g.capture = nullptr;
        return issue(s);
    }
    if (cudaStreamBeginCapture(g.capture, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        (void) cudaGetLastError();
        return issue(s);
    }
    const uint64_t before = launches_now();
    const b2q_status st = issue(g.capture);
    cudaGraph_t graph = nullptr;
    const cudaError_t err = cudaStreamEndCapture(g.capture, &graph);
    const uint64_t kernels = launches_now() - before;
    cudaGraphExec_t exec = nullptr;
    const bool ok = st == B2Q_OK && err == cudaSuccess && graph &&
                    cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess;
    if (graph) cudaGraphDestroy(graph);
    if (!ok) {
        (void) cudaGetLastError();
        g.forget();
        add_launches(-static_cast<int64_t>(kernels));   // captured, never run
        if (st != B2Q_OK) return st;
        return issue(s);   // the capture was refused: launch directly
    }
    e->exec = exec;
    e->kernels = kernels;   // counted once while captured; this launch runs them once
    count_graph_launch();
    return cuda_check(cudaGraphLaunch(e->exec, s), "graph launch");
}

// B2Q_OK when every per-layer tensor `<prefix>blk.<l>.<suffix>` is present.
b2q_status check_blocks(const TensorSet& ts, const char* prefix, int n_layer);

// The n_layer pre-LN blocks over T packed tokens, residual stream x [T][H]
// updated in place:
//   LN1 -> q8_1; QKV GEMM + bias -> fp16 [Q | K | V]; attention over the
//   sequences of `tiles`; quantize; O GEMM (acc + b) + x -> x; LN2 -> q8_1;
//   fc1 GEMM gelu(acc + b) -> q8_1; fc2 GEMM (acc + b) + x -> x.
// Work buffers: qkv [T][3H] fp16, att [T][H] fp32, act_h q8_1 planes for
// (T, H), act_f for (T, ffn).  exact_attention: always the fixed-order fp32
// attention kernel (otherwise the device's B2Q_TUNE_ATTN_EXACT setting).
b2q_status run_encoder_blocks(const TensorSet& ts, const char* prefix, int n_layer, int n_head, float eps, int64_t T,
                              int64_t H, float* x, __half* qkv, float* att, void* act_h, void* act_f,
                              const void* tiles, int n_tiles, bool exact_attention, cudaStream_t s);

}  // namespace b2q
