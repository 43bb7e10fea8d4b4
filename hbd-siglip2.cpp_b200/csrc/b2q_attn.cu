// b2q_attn.cu — head_dim-72 attention over packed variable-length sequences.
//
// Replaces the reference's flash_attn_ext call with its QKV-prep and post-FA
// copies (src/siglip2_vision.cpp:111-175, src/cuda/siglip2_megakernel.cu:
// 166-267,358-394): Q, K and V are read straight from the fp16 rows the QKV
// GEMM epilogue writes ([token][Q | K | V], head h at column h*72 of each),
// the 72 -> 80 zero padding exists only in shared memory, and the output is
// written contiguous as [token][h*72 + d] fp32, the layout the output
// projection's quantizer reads.  Softmax in fp32 with scale 1/sqrt(72); K and
// V are fp16 as in the reference (siglip2_vision.cpp:164-165).
//
// One CTA = 64 query rows of one head of one sequence (4 warps x 16 rows),
// streaming that sequence's keys in 64-row tiles (double-buffered cp.async),
// online softmax (FlashAttention-2 form) on mma.sync m16n8k16 tensor-core
// fragments.  Every image of a batch is its own sequence, so no padding or
// masking across images is needed; keys past a sequence's end are masked.
#include "b2q_internal.h"
#include "b2q_numerics.cuh"

#include <cuda_fp16.h>

namespace b2q {

namespace {

constexpr int kDH = 72;           // head dim
constexpr int kRowH = 88;         // smem row stride in halves (176 B: conflict-free ldmatrix)
constexpr int kQT = 64;           // query rows per CTA
constexpr int kKT = 64;           // key rows per tile
constexpr int kWarps = 4;

struct AttnTile {
    int q_row0;     // first query row (in Q's row space)
    int q_rows;     // valid query rows in this tile (<= 64)
    int k_row0;     // first key row of the sequence
    int k_len;      // keys in the sequence
    int o_row0;     // output row of the tile's first query
    int pad[3];
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
    const int bytes = valid ? 16 : 0;   // 0 source bytes -> zero fill
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(smem)), "l"(gmem), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_addr(p)));
}
__device__ __forceinline__ void ldmatrix_x2(uint32_t (&r)[2], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(smem_addr(p)));
}
__device__ __forceinline__ void ldmatrix_x2_trans(uint32_t (&r)[2], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
                 : "=r"(r[0]), "=r"(r[1])
                 : "r"(smem_addr(p)));
}

// D(16x8 f32) += A(16x16 f16, row) * B(16x8 f16, col)
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// (a, b) = head + tail: head = fp16(a, b), tail = fp16 of the remainders.
__device__ __forceinline__ void split_half2(float a, float b, uint32_t& head, uint32_t& tail) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    const __half2 t = __floats2half2_rn(a - hf.x, b - hf.y);
    head = *reinterpret_cast<const uint32_t*>(&h);
    tail = *reinterpret_cast<const uint32_t*>(&t);
}

// Copy `rows` rows of 72 halves (9 x 16 B) starting at src (row stride ld
// halves) into smem [64][88]; rows >= rows are zero-filled.
__device__ __forceinline__ void load_rows(__half* dst, const __half* src, int64_t ld, int rows) {
    for (int i = threadIdx.x; i < 64 * 9; i += kWarps * 32) {
        const int r = i / 9, c = i % 9;
        const bool valid = r < rows;
        const __half* g = valid ? src + static_cast<int64_t>(r) * ld + c * 8 : src;
        cp_async16(dst + r * kRowH + c * 8, g, valid);
    }
}

__global__ void __launch_bounds__(kWarps * 32)
attention_kernel(const __half* __restrict__ q, int64_t ldq, const __half* __restrict__ k, int64_t ldk,
                 const __half* __restrict__ v, int64_t ldv, const AttnTile* __restrict__ tiles,
                 float* __restrict__ out, int64_t ldo, float scale_log2) {
    extern __shared__ __align__(128) uint8_t attn_smem[];
    __half* sQ = reinterpret_cast<__half*>(attn_smem);
    __half* sK[2] = {sQ + kQT * kRowH, sQ + (kQT + kKT) * kRowH};
    __half* sV[2] = {sQ + (kQT + 2 * kKT) * kRowH, sQ + (kQT + 3 * kKT) * kRowH};

    const AttnTile t = tiles[blockIdx.x];
    const int head = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const __half* qh = q + static_cast<int64_t>(t.q_row0) * ldq + head * kDH;
    const __half* kh = k + static_cast<int64_t>(t.k_row0) * ldk + head * kDH;
    const __half* vh = v + static_cast<int64_t>(t.k_row0) * ldv + head * kDH;

    // zero the padded columns 72..79 of every buffer once (cp.async never writes them)
    for (int r = threadIdx.x; r < kQT; r += kWarps * 32) {
        *reinterpret_cast<uint4*>(sQ + r * kRowH + kDH) = make_uint4(0, 0, 0, 0);
        for (int b = 0; b < 2; ++b) {
            *reinterpret_cast<uint4*>(sK[b] + r * kRowH + kDH) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(sV[b] + r * kRowH + kDH) = make_uint4(0, 0, 0, 0);
        }
    }
    load_rows(sQ, qh, ldq, t.q_rows);
    const int n_kt = (t.k_len + kKT - 1) / kKT;
    load_rows(sK[0], kh, ldk, min(kKT, t.k_len));
    load_rows(sV[0], vh, ldv, min(kKT, t.k_len));
    cp_async_commit();

    // per-warp state: rows warp*16 + {lane/4, lane/4 + 8}
    float o[9][4];   // output columns 0..71 as 9 n-tiles of 8
#pragma unroll
    for (int i = 0; i < 9; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};
    uint32_t qa[5][4];

    for (int kt = 0; kt < n_kt; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < n_kt) {
            const int k0 = (kt + 1) * kKT;
            load_rows(sK[buf ^ 1], kh + static_cast<int64_t>(k0) * ldk, ldk, min(kKT, t.k_len - k0));
            load_rows(sV[buf ^ 1], vh + static_cast<int64_t>(k0) * ldv, ldv, min(kKT, t.k_len - k0));
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        if (kt == 0) {
            // Q fragments (A operand, 16 x 80 as 5 k-steps)
#pragma unroll
            for (int ks = 0; ks < 5; ++ks) {
                const int r = warp * 16 + (lane & 15);
                const int c = ks * 16 + (lane >> 4) * 8;
                ldmatrix_x4(qa[ks], sQ + r * kRowH + c);
            }
        }
        // S = Q K^T for 64 keys: 8 n-tiles of 8 keys
        float s[8][4];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
#pragma unroll
            for (int ks = 0; ks < 5; ++ks) {
                uint32_t kb[2];
                const int r = nt * 8 + (lane & 7);
                const int c = ks * 16 + ((lane >> 3) & 1) * 8;
                ldmatrix_x2(kb, sK[buf] + r * kRowH + c);
                mma_16816(s[nt], qa[ks], kb);
            }
        }
        // mask keys past the sequence end, scale, online softmax (rows r0 = lane/4, r1 = r0 + 8)
        const int kbase = kt * kKT;
        float mx[2] = {m_run[0], m_run[1]};
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = kbase + nt * 8 + (lane & 3) * 2 + (e & 1);
                float val = s[nt][e] * scale_log2;
                if (key >= t.k_len) val = -INFINITY;
                s[nt][e] = val;
                mx[e >> 1] = fmaxf(mx[e >> 1], val);
            }
        }
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
            mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
        }
        float corr[2], rowsum[2] = {0.0f, 0.0f};
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) corr[rr] = exp2f(m_run[rr] - mx[rr]);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float pv = exp2f(s[nt][e] - mx[e >> 1]);
                s[nt][e] = pv;
                rowsum[e >> 1] += pv;
            }
        }
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            rowsum[rr] += __shfl_xor_sync(0xffffffffu, rowsum[rr], 1);
            rowsum[rr] += __shfl_xor_sync(0xffffffffu, rowsum[rr], 2);
            l_run[rr] = l_run[rr] * corr[rr] + rowsum[rr];
            m_run[rr] = mx[rr];
        }
#pragma unroll
        for (int i = 0; i < 9; ++i) {
            o[i][0] *= corr[0];
            o[i][1] *= corr[0];
            o[i][2] *= corr[1];
            o[i][3] *= corr[1];
        }
        // O += P V: P (16 x 64) as 4 k-steps of A fragments built from the
        // score tiles.  P is split into an fp16 head and the fp16 rounding of
        // its remainder (two products per fragment), so the probabilities
        // keep ~22 bits instead of fp16's 11 and agree with the fp32 row
        // sums; the padded output columns 72..79 are not computed.
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            uint32_t pa[4], pl[4];
            split_half2(s[2 * ks][0], s[2 * ks][1], pa[0], pl[0]);
            split_half2(s[2 * ks][2], s[2 * ks][3], pa[1], pl[1]);
            split_half2(s[2 * ks + 1][0], s[2 * ks + 1][1], pa[2], pl[2]);
            split_half2(s[2 * ks + 1][2], s[2 * ks + 1][3], pa[3], pl[3]);
#pragma unroll
            for (int nt = 0; nt < 9; ++nt) {
                uint32_t vb[2];
                const int r = ks * 16 + (lane & 15);
                ldmatrix_x2_trans(vb, sV[buf] + r * kRowH + nt * 8);
                mma_16816(o[nt], pa, vb);
                mma_16816(o[nt], pl, vb);
            }
        }
        __syncthreads();
    }

    // normalise and store rows r0, r1 (72 of the 80 columns)
    const float inv0 = l_run[0] > 0.0f ? 1.0f / l_run[0] : 0.0f;
    const float inv1 = l_run[1] > 0.0f ? 1.0f / l_run[1] : 0.0f;
    const int r0 = warp * 16 + (lane >> 2), r1 = r0 + 8;
#pragma unroll
    for (int nt = 0; nt < 9; ++nt) {
        const int c = nt * 8 + (lane & 3) * 2;
        if (r0 < t.q_rows) {
            float* dst = out + static_cast<int64_t>(t.o_row0 + r0) * ldo + head * kDH + c;
            *reinterpret_cast<float2*>(dst) = make_float2(o[nt][0] * inv0, o[nt][1] * inv0);
        }
        if (r1 < t.q_rows) {
            float* dst = out + static_cast<int64_t>(t.o_row0 + r1) * ldo + head * kDH + c;
            *reinterpret_cast<float2*>(dst) = make_float2(o[nt][2] * inv1, o[nt][3] * inv1);
        }
    }
}

// Exact mode: the fixed fp32 evaluation order of the CPU checker (one thread
// per query row; fma chain over d for each score, scale, max; own exp;
// sum of p over keys ascending; fma chain over keys for each output dim; one
// division), so the whole tower can be verified bit for bit.  Scores are
// recomputed in each of the three passes instead of rescaled online, which
// would change the arithmetic.  A verification mode: ~3x the attention work.
constexpr int kExactThreads = 64;
constexpr int kExactKeys = 64;

__global__ void __launch_bounds__(kExactThreads)
attention_exact_kernel(const __half* __restrict__ q, int64_t ldq, const __half* __restrict__ k, int64_t ldk,
                       const __half* __restrict__ v, int64_t ldv, const AttnTile* __restrict__ tiles,
                       float* __restrict__ out, int64_t ldo, float scale) {
    __shared__ float sK[kExactKeys * kDH];
    __shared__ float sV[kExactKeys * kDH];
    const AttnTile t = tiles[blockIdx.x];
    const int head = blockIdx.y;
    const int r = threadIdx.x;
    const bool active = r < t.q_rows;
    float qv[kDH];
    const __half* qrow = q + static_cast<int64_t>(t.q_row0 + (active ? r : 0)) * ldq + head * kDH;
#pragma unroll
    for (int d = 0; d < kDH; ++d) qv[d] = __half2float(qrow[d]);
    const __half* kh = k + static_cast<int64_t>(t.k_row0) * ldk + head * kDH;
    const __half* vh = v + static_cast<int64_t>(t.k_row0) * ldv + head * kDH;

    float m = -INFINITY, l = 0.0f;
    float acc[kDH];
#pragma unroll
    for (int d = 0; d < kDH; ++d) acc[d] = 0.0f;

    for (int pass = 0; pass < 3; ++pass) {
        for (int k0 = 0; k0 < t.k_len; k0 += kExactKeys) {
            const int nk = min(kExactKeys, t.k_len - k0);
            __syncthreads();
            for (int i = threadIdx.x; i < nk * kDH; i += kExactThreads) {
                const int kk = i / kDH, d = i % kDH;
                sK[i] = __half2float(kh[static_cast<int64_t>(k0 + kk) * ldk + d]);
                if (pass == 2) sV[i] = __half2float(vh[static_cast<int64_t>(k0 + kk) * ldv + d]);
            }
            __syncthreads();
            for (int kk = 0; kk < nk; ++kk) {
                float dot = 0.0f;
#pragma unroll
                for (int d = 0; d < kDH; ++d) dot = __fmaf_rn(qv[d], sK[kk * kDH + d], dot);
                const float sc = __fmul_rn(dot, scale);
                if (pass == 0) {
                    m = fmaxf(m, sc);
                } else {
                    const float pv = own_expf(__fsub_rn(sc, m));
                    if (pass == 1) {
                        l = __fadd_rn(l, pv);
                    } else {
#pragma unroll
                        for (int d = 0; d < kDH; ++d) acc[d] = __fmaf_rn(pv, sV[kk * kDH + d], acc[d]);
                    }
                }
            }
        }
    }
    if (active) {
        float* o = out + static_cast<int64_t>(t.o_row0 + r) * ldo + head * kDH;
#pragma unroll
        for (int d = 0; d < kDH; ++d) o[d] = __fdiv_rn(acc[d], l);
    }
}

}  // namespace

size_t attn_tiles_bytes(int n_tiles) { return static_cast<size_t>(n_tiles) * sizeof(AttnTile); }

// Build the tile table for n_seq sequences: sequence s has q_len[s] query rows
// starting at q_off[s], k_len[s] keys starting at k_off[s], and writes its
// outputs from row o_off[s].  Returns the number of tiles written to `tiles`
// (host memory, capacity max_tiles), or -1 when it does not fit.
int attn_build_tiles(const int* q_off, const int* q_len, const int* k_off, const int* k_len, const int* o_off,
                     int n_seq, void* tiles, int max_tiles) {
    AttnTile* t = static_cast<AttnTile*>(tiles);
    int n = 0;
    for (int s = 0; s < n_seq; ++s) {
        for (int q0 = 0; q0 < q_len[s]; q0 += kQT) {
            if (n >= max_tiles) return -1;
            t[n].q_row0 = q_off[s] + q0;
            t[n].q_rows = q_len[s] - q0 < kQT ? q_len[s] - q0 : kQT;
            t[n].k_row0 = k_off[s];
            t[n].k_len = k_len[s];
            t[n].o_row0 = o_off[s] + q0;
            t[n].pad[0] = t[n].pad[1] = t[n].pad[2] = 0;
            ++n;
        }
    }
    return n;
}

cudaError_t launch_attention(const __half* q, int64_t ldq, const __half* k, int64_t ldk, const __half* v,
                             int64_t ldv, const void* tiles_dev, int n_tiles, int n_head, float* out, int64_t ldo,
                             cudaStream_t s, bool force_exact) {
    if (n_tiles <= 0) return cudaSuccess;
    DeviceState* ds = state();
    if (force_exact || (ds && ds->attn_exact)) {
        const float scale = 1.0f / sqrtf(static_cast<float>(kDH));
        dim3 grid(static_cast<unsigned>(n_tiles), static_cast<unsigned>(n_head));
        attention_exact_kernel<<<grid, kExactThreads, 0, s>>>(q, ldq, k, ldk, v, ldv,
                                                              static_cast<const AttnTile*>(tiles_dev), out, ldo,
                                                              scale);
        count_launch();
        return cudaGetLastError();
    }
    constexpr int smem = (kQT + 4 * kKT) * kRowH * 2;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(kDH));
    dim3 grid(static_cast<unsigned>(n_tiles), static_cast<unsigned>(n_head));
    attention_kernel<<<grid, kWarps * 32, smem, s>>>(q, ldq, k, ldk, v, ldv, static_cast<const AttnTile*>(tiles_dev),
                                                  out, ldo, scale_log2);
    count_launch();
    return cudaGetLastError();
}

}  // namespace b2q
