// b2q_rowops.cu — bandwidth-bound kernels that feed the GEMM:
//   * Q8_0 weight repack (once per weight, at registration);
//   * q8_1 activation quantize (src/cuda/siglip2_custom_mmq.cu:51-97);
//   * LayerNorm + affine fused with the q8_1 quantize of its output
//     (src/cuda/siglip2_megakernel.cu:81-138 + the quantize that follows).
//
// Row kernels: one warp per row; a lane owns float4 chunk c at element
// (c*32 + lane)*4, so one 32-element q8_1 block spans 8 consecutive lanes and
// its absmax needs three xor-shuffles.  A CTA covers 32 rows and stages the
// per-block scales in shared memory so the [Kb][ld] scale plane is written
// with coalesced 128-byte rows.
#include "b2q_internal.h"
#include "b2q_numerics.cuh"

#include <cuda_fp16.h>

namespace b2q {

constexpr int kRowsPerCta = 32;
constexpr int kRowWarps = 8;
constexpr int kMaxKb = 160;   // scale staging capacity: K up to 5120

ActLayout act_layout(int64_t M, int64_t K, int mode) {
    ActLayout L;
    L.M = M;
    L.K = K;
    L.Kp = round_up(K, 32);
    L.Kb = L.Kp / 32;
    L.ld = round_up(M, 4);
    L.es = ops_elem_bytes(mode);
    L.d_offset = static_cast<size_t>(round_up(M * L.Kp * L.es, 256));
    L.bytes = L.d_offset + static_cast<size_t>(L.Kb * L.ld * 4);
    return L;
}

// ------------------------------------------------------------------ repack
// raw: N rows of Kb blocks {fp16 d; int8 q[32]} (34 bytes, 2-byte aligned).
template <int kOps>
__global__ void repack_q8_0_kernel(const uint8_t* __restrict__ raw, int64_t N, int64_t Kb, int64_t row_bytes,
                                   int64_t Nd, void* __restrict__ q, float* __restrict__ d) {
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;   // one block per thread
    if (idx >= N * Kb) return;
    const int64_t n = idx / Kb, kb = idx % Kb;
    const uint8_t* blk = raw + n * row_bytes + kb * 34;
    const uint16_t dh = static_cast<uint16_t>(blk[0]) | (static_cast<uint16_t>(blk[1]) << 8);
    d[kb * Nd + scale_slot(n)] = __half2float(__ushort_as_half(dh));
    const int64_t K = Kb * 32;
    if constexpr (kOps == kOpsF16) {
        __half* out = static_cast<__half*>(q) + n * K + kb * 32;
        for (int j = 0; j < 32; ++j) out[j] = __int2half_rn(static_cast<int8_t>(blk[2 + j]));
    } else {
        int8_t* out = static_cast<int8_t*>(q) + n * K + kb * 32;
        for (int j = 0; j < 32; ++j) out[j] = static_cast<int8_t>(blk[2 + j]);
    }
}

cudaError_t launch_repack_q8_0(const void* raw, int64_t N, int64_t Kb, int64_t row_bytes, int64_t Nd, int mode,
                               void* q, float* d, cudaStream_t s) {
    const int64_t total = N * Kb;
    const int threads = 256;
    const unsigned grid = static_cast<unsigned>((total + threads - 1) / threads);
    if (mode == kOpsF16)
        repack_q8_0_kernel<kOpsF16><<<grid, threads, 0, s>>>(static_cast<const uint8_t*>(raw), N, Kb, row_bytes, Nd, q,
                                                             d);
    else
        repack_q8_0_kernel<kOpsI8><<<grid, threads, 0, s>>>(static_cast<const uint8_t*>(raw), N, Kb, row_bytes, Nd, q,
                                                            d);
    count_launch();
    return cudaGetLastError();
}

// ------------------------------------------------------------------ helpers
// Quantize the 4 values a lane holds (its float4 chunk) given the 8-lane
// block absmax, store them and (lane%8 == 0) the scale into shared staging.
template <int kOps>
__device__ __forceinline__ void store_q4(void* qrow, int64_t col, float4 v, float amax) {
    const float inv = q8_inv_scale(amax);
    if constexpr (kOps == kOpsF16) {
        // rounding on the fp32 adder, no clamp needed (q8_round_adder2), and
        // the integers packed into their fp16 carriers exactly
        const float2 q01 = q8_round_adder2(make_float2(v.x, v.y), inv);
        const float2 q23 = q8_round_adder2(make_float2(v.z, v.w), inv);
        __half2 a = __floats2half2_rn(q01.x, q01.y);
        __half2 b = __floats2half2_rn(q23.x, q23.y);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&a);
        u.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(static_cast<__half*>(qrow) + col) = u;
    } else {
        const int q0 = q8_round(v.x, inv), q1 = q8_round(v.y, inv), q2 = q8_round(v.z, inv), q3 = q8_round(v.w, inv);
        const uint32_t u = (static_cast<uint32_t>(q0) & 0xFFu) | ((static_cast<uint32_t>(q1) & 0xFFu) << 8) |
                           ((static_cast<uint32_t>(q2) & 0xFFu) << 16) | ((static_cast<uint32_t>(q3) & 0xFFu) << 24);
        *reinterpret_cast<uint32_t*>(static_cast<int8_t*>(qrow) + col) = u;
    }
}

__device__ __forceinline__ float block8_absmax(float4 v) {
    float a = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 4));
    return a;
}

// Write the staged scales sd[kb][r] (r < rows) of this CTA's rows to the
// scale plane d[kb][ld] with 32-float coalesced rows.
__device__ __forceinline__ void flush_scales(const float* sd, int64_t Kb, int rows, float* d, int64_t ld, int64_t m0) {
    for (int64_t i = threadIdx.x; i < Kb * kRowsPerCta; i += blockDim.x) {
        const int64_t kb = i / kRowsPerCta;
        const int r = static_cast<int>(i % kRowsPerCta);
        if (r < rows) d[kb * ld + m0 + r] = sd[kb * kRowsPerCta + r];
    }
}

// ------------------------------------------------------------------ quantize
template <int kOps>
__global__ void __launch_bounds__(kRowWarps * 32)
quantize_q8_1_kernel(const float* __restrict__ x, int64_t M, int64_t K, int64_t ldx, void* __restrict__ qs,
                     float* __restrict__ d, int64_t Kp, int64_t ld) {
    __shared__ float sd[kMaxKb * kRowsPerCta];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t m0 = static_cast<int64_t>(blockIdx.x) * kRowsPerCta;
    const int rows = static_cast<int>(M - m0 < kRowsPerCta ? M - m0 : kRowsPerCta);
    const bool vec = (K % 4 == 0) && (ldx % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
    for (int r = warp; r < rows; r += kRowWarps) {
        const int64_t m = m0 + r;
        const float* xr = x + m * ldx;
        void* qrow = kOps == kOpsF16 ? static_cast<void*>(static_cast<__half*>(qs) + m * Kp)
                                     : static_cast<void*>(static_cast<int8_t*>(qs) + m * Kp);
        for (int64_t c0 = 0; c0 < Kp; c0 += 128) {
            const int64_t col = c0 + lane * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (col + 3 < K && vec) {
                v = *reinterpret_cast<const float4*>(xr + col);
            } else {
                if (col + 0 < K) v.x = xr[col + 0];
                if (col + 1 < K) v.y = xr[col + 1];
                if (col + 2 < K) v.z = xr[col + 2];
                if (col + 3 < K) v.w = xr[col + 3];
            }
            const float amax = block8_absmax(v);
            if (col < Kp) {
                store_q4<kOps>(qrow, col, v, amax);
                if ((lane & 7) == 0) sd[(col / 32) * kRowsPerCta + r] = q8_scale(amax);
            }
        }
    }
    __syncthreads();
    flush_scales(sd, Kp / 32, rows, d, ld, m0);
}

// Rows of a compile-time width (kChunks x 128 values, 16-byte aligned): all of
// a row's loads are issued before any of it is quantized, so a warp keeps
// kChunks 16-byte loads in flight instead of one.  Same element rule, same
// outputs as quantize_q8_1_kernel.
template <int kOps, int kChunks>
__global__ void __launch_bounds__(kRowWarps * 32)
quantize_rows_kernel(const float* __restrict__ x, int64_t M, int64_t ldx, void* __restrict__ qs,
                     float* __restrict__ d, int64_t ld) {
    constexpr int K = kChunks * 128;
    constexpr int Kb = K / 32;
    __shared__ float sd[Kb * kRowsPerCta];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t m0 = static_cast<int64_t>(blockIdx.x) * kRowsPerCta;
    const int rows = static_cast<int>(M - m0 < kRowsPerCta ? M - m0 : kRowsPerCta);
    for (int r = warp; r < rows; r += kRowWarps) {
        const int64_t m = m0 + r;
        const float4* xr = reinterpret_cast<const float4*>(x + m * ldx);
        float4 v[kChunks];
#pragma unroll
        for (int c = 0; c < kChunks; ++c) v[c] = xr[c * 32 + lane];
        void* qrow = kOps == kOpsF16 ? static_cast<void*>(static_cast<__half*>(qs) + m * K)
                                     : static_cast<void*>(static_cast<int8_t*>(qs) + m * K);
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
            const int col = c * 128 + lane * 4;
            const float amax = block8_absmax(v[c]);
            store_q4<kOps>(qrow, col, v[c], amax);
            if ((lane & 7) == 0) sd[(col / 32) * kRowsPerCta + r] = q8_scale(amax);
        }
    }
    __syncthreads();
    flush_scales(sd, Kb, rows, d, ld, m0);
}

template <int kOps, int kChunks>
static bool launch_quantize_rows(const float* x, int64_t M, int64_t K, int64_t ldx, void* qs, float* d, int64_t ld,
                                 unsigned grid, cudaStream_t s) {
    if (K != kChunks * 128 || (ldx % 4) != 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0) return false;
    quantize_rows_kernel<kOps, kChunks><<<grid, kRowWarps * 32, 0, s>>>(x, M, ldx, qs, d, ld);
    return true;
}

cudaError_t launch_quantize_q8_1(const float* x, int64_t M, int64_t K, int64_t ldx, void* act, int mode,
                                 cudaStream_t s) {
    const ActLayout L = act_layout(M, K, mode);
    if (L.Kb > kMaxKb) return cudaErrorInvalidValue;
    float* d = reinterpret_cast<float*>(static_cast<uint8_t*>(act) + L.d_offset);
    const unsigned grid = static_cast<unsigned>((M + kRowsPerCta - 1) / kRowsPerCta);
    // the tower's widths: the attention output (1152) and the patch vectors (768)
    const bool fast = mode == kOpsF16 ? (launch_quantize_rows<kOpsF16, 9>(x, M, K, ldx, act, d, L.ld, grid, s) ||
                                         launch_quantize_rows<kOpsF16, 6>(x, M, K, ldx, act, d, L.ld, grid, s))
                                      : (launch_quantize_rows<kOpsI8, 9>(x, M, K, ldx, act, d, L.ld, grid, s) ||
                                         launch_quantize_rows<kOpsI8, 6>(x, M, K, ldx, act, d, L.ld, grid, s));
    if (fast) {
        count_launch();
        return cudaGetLastError();
    }
    if (mode == kOpsF16)
        quantize_q8_1_kernel<kOpsF16><<<grid, kRowWarps * 32, 0, s>>>(x, M, K, ldx, act, d, L.Kp, L.ld);
    else
        quantize_q8_1_kernel<kOpsI8><<<grid, kRowWarps * 32, 0, s>>>(x, M, K, ldx, act, d, L.Kp, L.ld);
    count_launch();
    return cudaGetLastError();
}

// ------------------------------------------------------------------ LN + quantize
// Sum order (shared with the CPU checker): lane partials over its chunks in
// ascending c, elements x,y,z,w in order (s += v, ss = fma(v, v, ss)), then an
// xor butterfly 16, 8, 4, 2, 1.  mean = s/H, var = ss/H - mean*mean,
// inv = 1/sqrt(var + eps) (correctly rounded), y = ((x - mean)*inv)*w + b.
template <int kOps, int kChunks>
__global__ void __launch_bounds__(kRowWarps * 32)
ln_quant_kernel(const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ b, float eps,
                int64_t M, void* __restrict__ qs, float* __restrict__ d, int64_t ld, float* __restrict__ y) {
    constexpr int H = kChunks * 128;
    constexpr int Kb = H / 32;
    __shared__ float sd[Kb * kRowsPerCta];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t m0 = static_cast<int64_t>(blockIdx.x) * kRowsPerCta;
    const int rows = static_cast<int>(M - m0 < kRowsPerCta ? M - m0 : kRowsPerCta);
    for (int r = warp; r < rows; r += kRowWarps) {
        const int64_t m = m0 + r;
        const float4* xr = reinterpret_cast<const float4*>(x + m * H);
        float4 v[kChunks];
        float s = 0.0f, ss = 0.0f;
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
            v[c] = xr[c * 32 + lane];
            s = __fadd_rn(s, v[c].x); ss = __fmaf_rn(v[c].x, v[c].x, ss);
            s = __fadd_rn(s, v[c].y); ss = __fmaf_rn(v[c].y, v[c].y, ss);
            s = __fadd_rn(s, v[c].z); ss = __fmaf_rn(v[c].z, v[c].z, ss);
            s = __fadd_rn(s, v[c].w); ss = __fmaf_rn(v[c].w, v[c].w, ss);
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
            ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
        }
        const float mean = __fdiv_rn(s, static_cast<float>(H));
        const float msq = __fdiv_rn(ss, static_cast<float>(H));
        const float var = __fsub_rn(msq, __fmul_rn(mean, mean));
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
        void* qrow = kOps == kOpsF16 ? static_cast<void*>(static_cast<__half*>(qs) + m * H)
                                     : static_cast<void*>(static_cast<int8_t*>(qs) + m * H);
        const float4* w4 = reinterpret_cast<const float4*>(w);
        const float4* b4 = reinterpret_cast<const float4*>(b);
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
            const float4 ww = w4[c * 32 + lane], bb = b4[c * 32 + lane];
            float4 o;
            o.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[c].x, mean), inv), ww.x), bb.x);
            o.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[c].y, mean), inv), ww.y), bb.y);
            o.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[c].z, mean), inv), ww.z), bb.z);
            o.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[c].w, mean), inv), ww.w), bb.w);
            if (y) reinterpret_cast<float4*>(y + m * H)[c * 32 + lane] = o;
            const float amax = block8_absmax(o);
            const int64_t col = (c * 32 + lane) * 4;
            store_q4<kOps>(qrow, col, o, amax);
            if ((lane & 7) == 0) sd[(col / 32) * kRowsPerCta + r] = q8_scale(amax);
        }
    }
    __syncthreads();
    flush_scales(sd, Kb, rows, d, ld, m0);
}

cudaError_t launch_ln_quant(const float* x, const float* w, const float* b, float eps, int64_t M, int64_t H,
                            void* act, float* y, int mode, cudaStream_t s) {
    const ActLayout L = act_layout(M, H, mode);
    float* d = reinterpret_cast<float*>(static_cast<uint8_t*>(act) + L.d_offset);
    const unsigned grid = static_cast<unsigned>((M + kRowsPerCta - 1) / kRowsPerCta);
#define B2Q_LN_CASE(CH)                                                                                          \
    case CH:                                                                                                    \
        if (mode == kOpsF16)                                                                                    \
            ln_quant_kernel<kOpsF16, CH><<<grid, kRowWarps * 32, 0, s>>>(x, w, b, eps, M, act, d, L.ld, y);     \
        else                                                                                                    \
            ln_quant_kernel<kOpsI8, CH><<<grid, kRowWarps * 32, 0, s>>>(x, w, b, eps, M, act, d, L.ld, y);      \
        break;
    switch (H / 128) {
        B2Q_LN_CASE(1)
        B2Q_LN_CASE(2)
        B2Q_LN_CASE(9)
        default:
            return cudaErrorInvalidValue;
    }
#undef B2Q_LN_CASE
    count_launch();
    return cudaGetLastError();
}

}  // namespace b2q
