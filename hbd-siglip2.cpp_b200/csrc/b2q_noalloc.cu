// b2q_noalloc.cu — ggml_mul_mat(W Q8_0, X F32) for callers that cannot
// allocate device memory.
//
// b2q_mul_mat_q8_0_f32 needs a caller-provided scratch buffer for the q8_1
// planes of X.  Some callers have no way to provide one: an op hook running
// inside another framework's graph executor (the ggml op-hook boundary this
// library plugs into) sees only the op's input and output tensors, and it may
// not call cudaMalloc in the middle of that executor's work, because the
// executor owns the memory plan and an allocation can synchronise the device.
// This entry point serves them: its scratch is a fixed array in this file,
// reserved on every GPU that loads the library, for as long as the process
// runs.
#include "b2q_internal.h"

#include <mutex>

namespace {

// Scratch for the q8_1 activation planes.  Its host-side name is only a
// stand-in for the device symbol; host code must use the device address
// looked up below, never &g_noalloc_scratch.
static __device__ __align__(256) uint8_t g_noalloc_scratch[B2Q_NOALLOC_MAX_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_addr[kMaxDevices] = {};   // per-device address of g_noalloc_scratch

// Looks up (once per device, with that device current) the device address of
// the scratch array.
b2q_status noalloc_scratch(int device, void** out) {
    if (device < 0 || device >= kMaxDevices) return b2q::set_error(B2Q_ERR_INVALID, "device index out of range");
    std::lock_guard<std::mutex> lk(g_noalloc_mutex);
    if (!g_noalloc_addr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return b2q::cuda_check(e, "cudaGetSymbolAddress(no-alloc scratch)");
        g_noalloc_addr[device] = p;
    }
    *out = g_noalloc_addr[device];
    return B2Q_OK;
}

}  // namespace

using namespace b2q;

extern "C" b2q_status b2q_mul_mat_q8_0_f32_noalloc(const b2q_weight* w, const float* x, int64_t M, int64_t x_cols,
                                                   float* y, void* stream) {
    B2Q_REQUIRE_STATE();
    if (!w || !x || !y) return set_error(B2Q_ERR_INVALID, "null pointer");
    if (w->device != ds->device) return set_error(B2Q_ERR_INVALID, "weight registered on another device");
    if (w->mode != ds->mode) return set_error(B2Q_ERR_INVALID, "weight registered under another operand mode");
    if (M <= 0 || x_cols <= 0 || x_cols > w->K || round_up(x_cols, 32) != w->K)
        return set_error(B2Q_ERR_SHAPE, "need M > 0 and x_cols in (K - 32, K]");
    if ((reinterpret_cast<uintptr_t>(y) & 15) != 0) return set_error(B2Q_ERR_ALIGN, "y must be 16-byte aligned");
    const ActLayout L = act_layout(M, w->K, ds->mode);
    if (L.bytes > B2Q_NOALLOC_MAX_SCRATCH_BYTES)
        return set_error(B2Q_ERR_SHAPE, "M x K too large for the fixed no-alloc scratch (" +
                                            std::to_string(L.bytes) + " bytes needed, " +
                                            std::to_string(B2Q_NOALLOC_MAX_SCRATCH_BYTES) + " available)");
    void* scratch = nullptr;
    b2q_status st = noalloc_scratch(ds->device, &scratch);
    if (st) return st;
    // Nothing in the scratch has to start at zero: the quantizer writes every
    // value and scale the GEMM reads (rows past M are never loaded).  Calls
    // share the array, so two calls whose kernels overlap on the GPU race.
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if ((st = cuda_check(launch_quantize_q8_1(x, M, x_cols, x_cols, scratch, ds->mode, s), "quantize launch")))
        return st;
    GemmArgs a{};
    a.w = w;
    a.act = scratch;
    a.M = M;
    a.epi = B2Q_EPI_NONE;
    a.out = y;
    return launch_gemm(a, s);
}
