// b2q_internal.h — host-side declarations shared by the library's .cu files.
#pragma once

#include <cstdint>
#include <cstddef>
#include <string>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include "../../include/b2q.h"

namespace b2q {

// Operand carriers for the int8 values fed to the tensor cores.
enum OpsMode : int { kOpsI8 = 0, kOpsF16 = 1 };

inline int ops_elem_bytes(int mode) { return mode == kOpsF16 ? 2 : 1; }
inline int64_t round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

// Activation buffer layout ("q8_1 planes"): for M rows of logical width K,
// Kp = round_up(K, 32), Kb = Kp / 32:
//   qs : [M][Kp] int8 values (1 byte each, or fp16 carriers in F16 mode)
//   d  : [Kb][ld] fp32 per-block scales, ld = round_up(M, 4), at byte offset
//        round_up(M*Kp*es, 256)
struct ActLayout {
    int64_t M, K, Kp, Kb, ld, es;
    size_t d_offset, bytes;
};
ActLayout act_layout(int64_t M, int64_t K, int mode);

struct DeviceState {
    int device = -1;
    int num_sms = 0;
    int mode = kOpsF16;
    uint32_t* err = nullptr;      // device error word (cudaMalloc'ed at init)
    uint64_t timeout_ns = 2000000000ull;
    int gemm_bn = 0;              // GEMM tile width: 128, 256, or 0 = by shape
    int gemm_ctas = 0;            // GEMM CTAs per SM: 1, 2 (128-column tiles), or 0 = by shape
    int attn_exact = 0;           // attention in the checker's fixed fp32 order
    int attn_kernel = 0;          // 0 = tcgen05 kernel, 1 = mma.sync kernel
    int test_stall = 0;           // GEMM producer / attention MMA issuer idle (failure-path tests)
    int graphs = 1;               // towers replay a repeated encode as a CUDA graph
    uint64_t tune_gen = 0;        // bumped by every b2q_tune call (captured graphs hold the settings)
};
DeviceState* state();             // per-thread current device state
void count_launch();              // every kernel launch of the library counts once
void add_launches(int64_t n);     // kernels of a replayed graph (negative: captured, not run)
uint64_t launches_now();
void count_graph_launch();        // a captured tower encode launched as one graph
b2q_status set_error(b2q_status st, const std::string& msg);
b2q_status cuda_check(cudaError_t e, const char* what);

// TMA descriptor creation through the driver entry point.
bool make_tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                  uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle128);

}  // namespace b2q

// Registered weight: repacked planes of a ggml Q8_0 tensor (N rows of K).
struct b2q_weight {
    int64_t N = 0, K = 0, Kb = 0;
    int mode = 0;
    int device = -1;
    int64_t Nd = 0;        // scale row pitch: N rounded up to 64 columns
    void* q = nullptr;     // [N][K] int8 (or fp16 carriers)
    float* d = nullptr;    // [Kb][Nd] fp32 (exact widening of the fp16 scales), columns
                           // permuted inside each 64-column group (scale_slot)
    CUtensorMap tm_q256, tm_q192, tm_q128, tm_q64;   // box 128 B x {256,192,128,64} rows, 128-byte swizzle
    CUtensorMap tm_d256, tm_d192, tm_d128, tm_d64;   // box {256,192,128,64} x (scales per stage)
};

// Position of column n inside its 64-column group of the weight-scale rows.
// The GEMM epilogue thread with column pairs 8g + 2q + {0,1} (g < 8, q < 4)
// of a 64-column chunk reads them as four 16-byte vectors: vector i holds
// pairs g = 2i and 2i + 1, and the four q lanes read 64 contiguous bytes.
__host__ __device__ inline int64_t scale_slot(int64_t n) {
    const int64_t c = n & 63, g = c >> 3, q = (c >> 1) & 3, e = c & 1;
    return (n & ~int64_t(63)) | (16 * (g >> 1) + 4 * q + 2 * (g & 1) + e);
}

#define B2Q_REQUIRE_STATE()                                                                 \
    b2q::DeviceState* ds = b2q::state();                                                    \
    if (!ds) return b2q::set_error(B2Q_ERR_NOT_INIT, "b2q_init was not called for this device")

namespace b2q {
// kernels (launchers return cudaError_t of the launch)
cudaError_t launch_repack_q8_0(const void* raw, int64_t N, int64_t Kb, int64_t row_bytes, int64_t Nd, int mode,
                               void* q, float* d, cudaStream_t s);
cudaError_t launch_quantize_q8_1(const float* x, int64_t M, int64_t K, int64_t ldx, void* act, int mode,
                                 cudaStream_t s);
cudaError_t launch_ln_quant(const float* x, const float* w, const float* b, float eps, int64_t M, int64_t H,
                            void* act, float* y, int mode, cudaStream_t s);

int attn_build_tiles(const int* q_off, const int* q_len, const int* k_off, const int* k_len, const int* o_off,
                     int n_seq, void* tiles, int max_tiles);
size_t attn_tiles_bytes(int n_tiles);
cudaError_t launch_attention(const __half* q, int64_t ldq, const __half* k, int64_t ldk, const __half* v,
                             int64_t ldv, const void* tiles_dev, int n_tiles, int n_head, float* out, int64_t ldo,
                             cudaStream_t s, bool force_exact = false);

struct GemmArgs {
    const b2q_weight* w;
    const void* act;
    int64_t M;
    int epi;
    const float* bias;
    const float* residual;
    void* out;
    int64_t ld_out;
    void* act_out;          // GELU_Q8 destination (activation buffer, K' = N)
    int32_t* dump;          // block sums [Kb][M][N] (debug)
};
b2q_status launch_gemm(const GemmArgs& a, cudaStream_t s);
}  // namespace b2q
