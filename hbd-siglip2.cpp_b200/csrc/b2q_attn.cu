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
// The default kernel (attention_tc_kernel) is built on the fifth-generation
// tensor cores: one CTA = 128 query rows of one head of one sequence, one
// thread per query row and TMEM lane.  Per 64-key tile, S = Q K^T goes to TMEM
// (tcgen05.mma, kind::f16), each thread runs the online softmax on its own row
// in registers, writes its probabilities to shared memory as the A operand of
// P V, and adds the P V tile (TMEM) into its fp32 output registers.  The
// score MMA of the next tile and the P V MMA of this one overlap the softmax.
// A second kernel (attention_kernel: 64-row halves of a tile, mma.sync
// m16n8k16 fragments, FlashAttention-2 form) and the exact checker kernel
// stay selectable.  Every image of a batch is its own sequence, so no padding
// or masking across images is needed; keys past a sequence's end are masked.
#include "b2q_internal.h"
#include "b2q_numerics.cuh"
#include "b2q_ptx.cuh"

#include <cuda_fp16.h>

namespace b2q {

namespace {

constexpr int kDH = 72;           // head dim
constexpr int kTileRows = 128;    // query rows per tile-table entry
constexpr int kRowH = 88;         // smem row stride in halves (176 B: conflict-free ldmatrix)
constexpr int kQT = 64;           // query rows per CTA of the 64-row kernels (half a tile)
constexpr int kKT = 64;           // key rows per tile
constexpr int kWarps = 4;

struct AttnTile {
    int q_row0;     // first query row (in Q's row space)
    int q_rows;     // valid query rows in this tile (<= 128)
    int k_row0;     // first key row of the sequence
    int k_len;      // keys in the sequence
    int o_row0;     // output row of the tile's first query
    int pad[3];
};

// The 64-row kernels run each 128-row table entry as two CTAs: half h covers
// query rows 64h .. 64h + 63 of the entry (none when the entry is shorter).
__device__ __forceinline__ AttnTile half_tile(AttnTile t, int h) {
    t.q_row0 += kQT * h;
    t.o_row0 += kQT * h;
    t.q_rows = min(kQT, t.q_rows - kQT * h);
    return t;
}

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

    const AttnTile t = half_tile(tiles[blockIdx.x >> 1], blockIdx.x & 1);
    if (t.q_rows <= 0) return;
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
// per query row; fma chain over d for each score, scale, max; own exp; sum
// of p over keys ascending; fma chain over keys for each output dim; one
// division), so the whole tower can be verified bit for bit.  Two passes over
// the keys: the first finds the row maximum, the second recomputes each
// score, takes p = exp(s - max) and feeds both the running sum l and the 72
// output chains (both ascending over keys, as in the checker; the sum is only
// used at the end, so one pass serves both).  Scores are recomputed rather
// than rescaled online, which would change the arithmetic.  Four keys' score
// chains are evaluated side by side (each its own chain over d), so the
// thread is not waiting on one FMA at a time.
constexpr int kExactThreads = 64;
constexpr int kExactKeys = 64;

// Key rows are read four dimensions at a time (16-byte shared loads; a row
// is 288 bytes, so every row starts 16-byte aligned), the products still
// accumulated one dimension after the other.
template <int kN>
__device__ __forceinline__ void exact_scores(const float (&qv)[kDH], const float* sk, float scale, float (&sc)[kN]) {
    float dot[kN];
#pragma unroll
    for (int j = 0; j < kN; ++j) dot[j] = 0.0f;
#pragma unroll
    for (int d4 = 0; d4 < kDH / 4; ++d4)
#pragma unroll
        for (int j = 0; j < kN; ++j) {
            const float4 kv = *reinterpret_cast<const float4*>(sk + j * kDH + 4 * d4);
            dot[j] = __fmaf_rn(qv[4 * d4 + 0], kv.x, dot[j]);
            dot[j] = __fmaf_rn(qv[4 * d4 + 1], kv.y, dot[j]);
            dot[j] = __fmaf_rn(qv[4 * d4 + 2], kv.z, dot[j]);
            dot[j] = __fmaf_rn(qv[4 * d4 + 3], kv.w, dot[j]);
        }
#pragma unroll
    for (int j = 0; j < kN; ++j) sc[j] = __fmul_rn(dot[j], scale);
}

__device__ __forceinline__ void store_halves8(float* dst, uint4 r) {
    const __half2* h = reinterpret_cast<const __half2*>(&r);
    const float2 a = __half22float2(h[0]), b = __half22float2(h[1]), c = __half22float2(h[2]),
                 d = __half22float2(h[3]);
    reinterpret_cast<float4*>(dst)[0] = make_float4(a.x, a.y, b.x, b.y);
    reinterpret_cast<float4*>(dst)[1] = make_float4(c.x, c.y, d.x, d.y);
}

__device__ __forceinline__ void exact_accumulate(float (&acc)[kDH], float pv, const float* sv) {
#pragma unroll
    for (int d4 = 0; d4 < kDH / 4; ++d4) {
        const float4 vv = *reinterpret_cast<const float4*>(sv + 4 * d4);
        acc[4 * d4 + 0] = __fmaf_rn(pv, vv.x, acc[4 * d4 + 0]);
        acc[4 * d4 + 1] = __fmaf_rn(pv, vv.y, acc[4 * d4 + 1]);
        acc[4 * d4 + 2] = __fmaf_rn(pv, vv.z, acc[4 * d4 + 2]);
        acc[4 * d4 + 3] = __fmaf_rn(pv, vv.w, acc[4 * d4 + 3]);
    }
}

__global__ void __launch_bounds__(kExactThreads)
attention_exact_kernel(const __half* __restrict__ q, int64_t ldq, const __half* __restrict__ k, int64_t ldk,
                       const __half* __restrict__ v, int64_t ldv, const AttnTile* __restrict__ tiles,
                       float* __restrict__ out, int64_t ldo, float scale) {
    __shared__ __align__(16) float sK[kExactKeys * kDH];
    __shared__ __align__(16) float sV[kExactKeys * kDH];
    const AttnTile t = half_tile(tiles[blockIdx.x >> 1], blockIdx.x & 1);
    if (t.q_rows <= 0) return;
    const int head = blockIdx.y;
    const int r = threadIdx.x;
    const bool active = r < t.q_rows;
    float qv[kDH];
    const __half* qrow = q + static_cast<int64_t>(t.q_row0 + (active ? r : 0)) * ldq + head * kDH;
#pragma unroll
    for (int d = 0; d < kDH; ++d) qv[d] = __half2float(qrow[d]);
    const __half* kh = k + static_cast<int64_t>(t.k_row0) * ldk + head * kDH;
    const __half* vh = v + static_cast<int64_t>(t.k_row0) * ldv + head * kDH;
    // key and value rows that start on 16-byte boundaries are read 8 halves at a time
    const bool vec_rows = ((reinterpret_cast<uintptr_t>(kh) | reinterpret_cast<uintptr_t>(vh) |
                            static_cast<uintptr_t>(ldk * 2) | static_cast<uintptr_t>(ldv * 2)) & 15u) == 0;

    float m = -INFINITY, l = 0.0f;
    float acc[kDH];
#pragma unroll
    for (int d = 0; d < kDH; ++d) acc[d] = 0.0f;

    for (int pass = 0; pass < 2; ++pass) {
        for (int k0 = 0; k0 < t.k_len; k0 += kExactKeys) {
            const int nk = min(kExactKeys, t.k_len - k0);
            __syncthreads();
            if (vec_rows) {
                // 9 x 16-byte chunks of 8 halves per 72-dim row
                for (int i = threadIdx.x; i < nk * 9; i += kExactThreads) {
                    const int kk = i / 9, c = i - (i / 9) * 9;
                    const uint4 kr = *reinterpret_cast<const uint4*>(kh + static_cast<int64_t>(k0 + kk) * ldk + 8 * c);
                    store_halves8(sK + kk * kDH + 8 * c, kr);
                    if (pass == 1) {
                        const uint4 vr = *reinterpret_cast<const uint4*>(vh + static_cast<int64_t>(k0 + kk) * ldv + 8 * c);
                        store_halves8(sV + kk * kDH + 8 * c, vr);
                    }
                }
            } else {
                for (int i = threadIdx.x; i < nk * kDH; i += kExactThreads) {
                    const int kk = i / kDH, d = i % kDH;
                    sK[i] = __half2float(kh[static_cast<int64_t>(k0 + kk) * ldk + d]);
                    if (pass == 1) sV[i] = __half2float(vh[static_cast<int64_t>(k0 + kk) * ldv + d]);
                }
            }
            __syncthreads();
            int kk = 0;
            for (; kk + 4 <= nk; kk += 4) {
                float sc[4];
                exact_scores<4>(qv, sK + kk * kDH, scale, sc);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (pass == 0) {
                        m = fmaxf(m, sc[j]);
                    } else {
                        const float pv = own_expf(__fsub_rn(sc[j], m));
                        l = __fadd_rn(l, pv);
                        exact_accumulate(acc, pv, sV + (kk + j) * kDH);
                    }
                }
            }
            for (; kk < nk; ++kk) {
                float sc[1];
                exact_scores<1>(qv, sK + kk * kDH, scale, sc);
                if (pass == 0) {
                    m = fmaxf(m, sc[0]);
                } else {
                    const float pv = own_expf(__fsub_rn(sc[0], m));
                    l = __fadd_rn(l, pv);
                    exact_accumulate(acc, pv, sV + kk * kDH);
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

// ---------------------------------------------------------------------------
// tcgen05 kernel.  Shared memory (from a 1024-byte aligned base), every
// operand with the 128-byte swizzle (a 128-byte row's 16-byte chunk c stored
// at chunk c ^ (row % 8)), filled by cp.async, three key tiles in flight:
//   K[3]  K-major [2 atoms][64 rows][128 B]: dims 0..63 | 64..79 (72..79 zero)
//   V[3]  MN-major [2 atoms][64 keys][128 B]: dims 0..63 | 64..127 of each
//         key row as loaded (no transpose); in atom 1 only dims 64..79 are
//         read: 64..71 loaded, 72 = 1.0 (the row-sum column), 73..79 zero
// TMEM (256 columns): two 64-column buffers, each holding first the scores
// S(j) of key tile j (fp32) and then, over them, its probabilities as the A
// operand of P V: P_hi in columns 0..31 and P_lo in 32..63 (fp16 pairs);
// the output accumulator O (80 columns; column 72 = running row sum) at
// column 128; Q (the A operand of the scores: 80 dims as fp16 pairs, dims
// 72..79 zero) at column 208.
constexpr int kTcThreads = 224;   // warps 0-3: softmax (one query row each), 4: P V issue, 5: loads, 6: score issue
constexpr int kTcStages = 3;
constexpr uint32_t kTcK = 0, kTcKBuf = 16384, kTcV = 49152, kTcVBuf = 16384;
constexpr uint32_t kTcBar = 98304;
constexpr int kTcSmem = static_cast<int>(kTcBar) + 192 + 1024;   // 21 barriers, TMEM slot, abort flag
constexpr uint32_t kTcTmemCols = 256, kTcColO = 128, kTcColQ = 208;
constexpr uint32_t kTcOutPitch = 304;   // bytes per staged output row (76 floats)

__device__ __forceinline__ uint32_t sw128(uint32_t row, uint32_t chunk) {
    return row * 128u + (((chunk ^ row) & 7u) << 4);
}
__device__ __forceinline__ void sts_v4(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}
__device__ __forceinline__ void cp_async16_at(uint32_t dst, const void* gmem, bool valid) {
    const int bytes = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(gmem), "r"(bytes) : "memory");
}
// Writes of the generic proxy (st.shared, cp.async) are ordered before the
// tensor core's reads by this fence (with a barrier between writer and
// issuer).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Row r of a 72-wide fp16 operand in a two-atom region of 64 rows: chunks
// 0..7 (dims 0..63) in atom 0, chunk 8 (dims 64..71) as chunk 0 of atom 1.
// The same addresses serve the K-major (K) and MN-major (V) operands: only
// the descriptors differ.
__device__ __forceinline__ uint32_t tc_chunk_addr(uint32_t region, uint32_t r, uint32_t c) {
    return c < 8 ? region + sw128(r, c) : region + 64u * 128u + sw128(r, 0);
}

// A 64-row key tile (K or V) by the loader warp: lane l copies rows l and
// l + 32; rows >= valid are zeros (their scores are masked, their
// probabilities 0, and 0 x garbage could be NaN).
__device__ __forceinline__ void tc_load_tile(uint32_t buf, const __half* src, int64_t ld, int valid, uint32_t lane) {
#pragma unroll
    for (uint32_t h = 0; h < 2; ++h) {
        const uint32_t r = lane + 32u * h;
        const bool ok = static_cast<int>(r) < valid;
        const __half* g = src + (ok ? static_cast<int64_t>(r) * ld : 0);
#pragma unroll
        for (uint32_t c = 0; c < 9; ++c) cp_async16_at(tc_chunk_addr(buf, r, c), g + 8 * c, ok);
    }
}

// S(128 x 64) = Q K^T over the 80 padded dims: Q from TMEM (16 dims = 8
// columns per step), K K-major: four steps inside atom 0 (start address + 32
// bytes each) and one in atom 1.
__device__ __forceinline__ void tc_issue_scores(uint32_t tmem_s, uint32_t tmem_q, uint32_t k) {
    constexpr uint32_t idesc = idesc_f16_f32(128, 64);
#pragma unroll
    for (uint32_t ks = 0; ks < 5; ++ks) {
        const uint32_t kb = ks < 4 ? k + 32u * ks : k + 64u * 128u;
        mma_f16_ts(tmem_s, tmem_q + 8u * ks, smem_desc_k_sw128(kb), idesc, ks > 0 ? 1u : 0u);
    }
}
// O(128 x 80) (+)= P_hi V + P_lo V over the tile's 64 keys: P from TMEM
// (16 keys = 8 columns per step), V MN-major (16 keys = two 1024-byte
// atoms per step, dims 64..79 in the atom 8 KB on).
__device__ __forceinline__ void tc_issue_pv(uint32_t tmem_o, uint32_t tmem_p, uint32_t v, bool accumulate) {
    constexpr uint32_t idesc = idesc_f16_f32(128, 80) | kIdescBMajorMN;
#pragma unroll
    for (uint32_t ks = 0; ks < 4; ++ks)
        mma_f16_ts(tmem_o, tmem_p + 8u * ks, smem_desc_mn_sw128(v + 2048u * ks, 8192u), idesc,
                   (accumulate || ks > 0) ? 1u : 0u);
#pragma unroll
    for (uint32_t ks = 0; ks < 4; ++ks)
        mma_f16_ts(tmem_o, tmem_p + 32u + 8u * ks, smem_desc_mn_sw128(v + 2048u * ks, 8192u), idesc, 1u);
}

// Bounded wait taken by a whole warp: the warp goes on only if every lane's
// wait succeeded (an expiry records `code` and raises the CTA's abort flag).
__device__ __forceinline__ bool tc_warp_wait(uint32_t bar, uint32_t parity, volatile uint32_t* abort_flag,
                                             uint64_t timeout_ns, uint32_t* err, uint32_t code) {
    const bool ok = mbar_wait(bar, parity, abort_flag, timeout_ns);
    if (!ok) {
        *abort_flag = 1u;
        atomicCAS(err, 0u, code);
    }
    return __all_sync(0xffffffffu, ok);
}

// Multiplies this thread's row of O (80 columns) in TMEM by f, 16 columns
// at a time (the row's 64 scores stay live in registers meanwhile).
__device__ __forceinline__ void tc_scale_o(uint32_t taddr, float f) {
    uint32_t r[16];
#pragma unroll
    for (uint32_t h = 0; h < 5; ++h) {
        tmem_ld_32x32b_x16(taddr + 16u * h, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * f);
        tmem_st_32x32b_x16(taddr + 16u * h, r);
    }
    tmem_st_wait();
}

// Roles and hand-offs (mbarriers; no block-wide barrier inside the key loop).
// Key tile j uses TMEM buffer j % 2 and K / V buffers j % 3; every barrier
// named "[b]" exists once per buffer, so no waiter can be overtaken by the
// next phase of the barrier it waits on.
//   loader warp, per key tile j: once S(j-3) has read K buffer j % 3
//     (k_empty), issue the cp.async of K tile j (k_full completes when they
//     land); once P(j-3) V(j-3) has read V buffer j % 3 (v_empty), the same
//     for V tile j (v_full).  It never waits for its own copies.
//   P V issuer, per key tile j: wait for P(j) (p_full, four softmax warps)
//     and V tile j; issue O (+)= P(j) V(j) (commits o_done[j % 2], v_empty).
//   score issuer, per key tile j: once P(j-2) V(j-2) is done (o_done) and K
//     tile j has landed, issue S(j) into TMEM buffer j % 2 (commits s_full,
//     k_empty).  Two issuing threads keep the tensor core fed faster than
//     one: a single thread issues about one MMA per 64 cycles.
//   softmax warps (thread = query row = TMEM lane), per key tile j:
//     wait for S(j), read the row, mask, row max, probabilities
//     p = exp2(s * scale_log2 - m) against a reference m that moves only
//     when the row's maximum exceeds it by more than 8 (so p <= 256, exact
//     in the fp16 split); if m moved, wait for P(j-1) V(j-1) and rescale the
//     row of O in TMEM; write P_hi / P_lo over S(j); signal p_full.
// The softmax warps never wait for a P V product in the steady state, so
// the score tiles stream through them while the tensor core runs behind; a
// softmax warp can be one key tile ahead of the slowest one (tile j+2 needs
// S(j+2), which waits for P(j) V(j)).
// Barrier phases: every waiter on a per-buffer barrier has itself seen the
// phase before the one it waits for (k-th wait of a waiter = k-th phase),
// and the next phase needs an arrival that follows its own, so a parity
// wait always names the intended phase.
// Every wait is bounded; an expired wait records its code, raises the CTA's
// abort flag (every other wait then gives up too), and the roles unwind.
// Two CTAs per SM (14 warps, 117 registers per thread).
__global__ void __launch_bounds__(kTcThreads, 2)
attention_tc_kernel(const __half* __restrict__ q, int64_t ldq, const __half* __restrict__ k, int64_t ldk,
                    const __half* __restrict__ v, int64_t ldv, const AttnTile* __restrict__ tiles,
                    float* __restrict__ out, int64_t ldo, float scale_log2, uint32_t* err, uint64_t timeout_ns,
                    int stall) {
    extern __shared__ __align__(1024) uint8_t tc_smem[];
    const uint32_t raw = smem_u32(tc_smem);
    const uint32_t base = (raw + 1023u) & ~1023u;
    const uint32_t sK = base + kTcK, sV = base + kTcV;
    // per-buffer barriers: bar + 8 * buffer
    const uint32_t bar_s = base + kTcBar, bar_p = bar_s + 16, bar_kf = bar_s + 32, bar_vf = bar_s + 56,
                   bar_ke = bar_s + 80, bar_ve = bar_s + 104, bar_o = bar_s + 128, bar_last = bar_s + 144,
                   bar_q = bar_s + 152, bar_fin = bar_s + 160;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tc_smem + (base - raw) + kTcBar + 168);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const AttnTile t = tiles[blockIdx.x];
    const int head = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5;
    const uint32_t lane = tid & 31;
    const __half* qh = q + static_cast<int64_t>(t.q_row0) * ldq + head * kDH;
    const __half* kh = k + static_cast<int64_t>(t.k_row0) * ldk + head * kDH;
    const __half* vh = v + static_cast<int64_t>(t.k_row0) * ldv + head * kDH;
    const int n_kt = (t.k_len + kKT - 1) / kKT;

    if (tid == 0) {
        for (uint32_t b = 0; b < 2; ++b) {
            mbar_init(bar_s + 8 * b, 1);
            mbar_init(bar_p + 8 * b, 4);
        }
        for (uint32_t b = 0; b < kTcStages; ++b) {
            mbar_init(bar_kf + 8 * b, 32);   // one cp.async arrival per loader lane
            mbar_init(bar_vf + 8 * b, 32);
            mbar_init(bar_ke + 8 * b, 1);
            mbar_init(bar_ve + 8 * b, 1);
        }
        mbar_init(bar_o, 1);
        mbar_init(bar_o + 8, 1);
        mbar_init(bar_last, 1);
        mbar_init(bar_q, 4);
        mbar_init(bar_fin, 2);
        *abort_flag = 0u;
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, kTcTmemCols);
        tc_fence_before();
    }
    uint4 qv[9];
    if (warp < 4) {
        // this thread's query row (zeros past the tile), into TMEM below;
        // the loads are in flight during the constant stores
        const bool ok = tid < t.q_rows;
        const uint4* g = reinterpret_cast<const uint4*>(qh + (ok ? static_cast<int64_t>(tid) * ldq : 0));
#pragma unroll
        for (int c = 0; c < 9; ++c) qv[c] = ok ? __ldg(g + c) : make_uint4(0, 0, 0, 0);
        // constant parts: dims 72..79 (chunk 1 of atom 1) are zero in every
        // K buffer and hold 1.0 at dim 72 in every V buffer
        for (uint32_t i = tid; i < kTcStages * 64u; i += 128u) {
            const uint32_t r = i & 63u, b = i >> 6;
            sts_v4(sK + b * kTcKBuf + 64u * 128u + sw128(r, 1), 0, 0, 0, 0);
            sts_v4(sV + b * kTcVBuf + 64u * 128u + sw128(r, 1), 0x00003C00u, 0, 0, 0);
        }
        fence_proxy_async_smem();
    } else if (warp == 5 && n_kt > 0) {
        // key tile 0 (its arrival follows the barrier below)
        tc_load_tile(sK, kh, ldk, min(kKT, t.k_len), lane);
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < 4) {
        // ---------------------------------------------------------- softmax
        const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
        {   // Q row into TMEM: column c holds dims 2c, 2c+1
            uint32_t r0[32], r1[16];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                r0[4 * c] = qv[c].x;
                r0[4 * c + 1] = qv[c].y;
                r0[4 * c + 2] = qv[c].z;
                r0[4 * c + 3] = qv[c].w;
            }
            r1[0] = qv[8].x;
            r1[1] = qv[8].y;
            r1[2] = qv[8].z;
            r1[3] = qv[8].w;
#pragma unroll
            for (int c = 4; c < 16; ++c) r1[c] = 0u;
            tmem_st_32x32b_x32(tmem + lane_base + kTcColQ, r0);
            tmem_st_32x32b_x16(tmem + lane_base + kTcColQ + 32u, r1);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_q);
        }
        float m_ref = -INFINITY;
        bool done = false;
        for (int j = 0; j < n_kt; ++j) {
            const uint32_t b = j & 1;
            const uint32_t tbuf = tmem + lane_base + 64u * b;
            if (!tc_warp_wait(bar_s + 8u * b, (j >> 1) & 1, abort_flag, timeout_ns, err, kDevTimeoutTmemFull)) break;
            tc_fence_after();
            float s[64];
            {
                uint32_t r0[32], r1[32];
                tmem_ld_32x32b_x32(tbuf, r0);
                tmem_ld_32x32b_x32(tbuf + 32u, r1);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    s[i] = __uint_as_float(r0[i]);
                    s[32 + i] = __uint_as_float(r1[i]);
                }
            }
            const int valid = t.k_len - j * kKT;   // keys of this tile that exist (>= 1)
            if (valid < kKT) {
#pragma unroll
                for (int i = 0; i < 64; ++i)
                    if (i >= valid) s[i] = -INFINITY;
            }
            float mx;
            {   // row maximum of the raw scores (a tree, not a 64-deep chain)
                float m8[8];
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    m8[i] = fmaxf(fmaxf(fmaxf(s[i], s[i + 8]), fmaxf(s[i + 16], s[i + 24])),
                                  fmaxf(fmaxf(s[i + 32], s[i + 40]), fmaxf(s[i + 48], s[i + 56])));
                mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                           fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
            }
            const float m_new = mx * scale_log2;
            const bool move = m_new > m_ref + 8.0f;
            float corr = 1.0f;
            if (move) {
                corr = ex2_approx(m_ref - m_new);   // 0 on the first tile
                m_ref = m_new;
            }
            if (j > 0 && __any_sync(0xffffffffu, move)) {
                // O holds P(0..j-1) V against the old reference: wait for the
                // last of those products.  S(j-1) and S(j) were issued after
                // P(j-3) V and P(j-2) V completed, so o_done[(j-1) % 2] has
                // passed P(j-3) V and this parity names P(j-1) V(j-1)
                if (!tc_warp_wait(bar_o + 8u * ((j - 1) & 1), ((j - 1) >> 1) & 1, abort_flag, timeout_ns, err,
                                  kDevTimeoutTmemFull))
                    break;
                tc_fence_after();
                tc_scale_o(tmem + lane_base + kTcColO, corr);
            }
            {   // P over S(j): column c of P_hi / P_lo holds keys 2c, 2c+1
                uint32_t hi[32], lo[32];
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const float p0 = ex2_approx(__fmaf_rn(s[2 * c], scale_log2, -m_ref));
                    const float p1 = ex2_approx(__fmaf_rn(s[2 * c + 1], scale_log2, -m_ref));
                    split_half2(p0, p1, hi[c], lo[c]);
                }
                tmem_st_32x32b_x32(tbuf, hi);
                tmem_st_32x32b_x32(tbuf + 32u, lo);
                tmem_st_wait();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_p + 8u * b);
            done = j + 1 == n_kt;
        }
        if (done && tc_warp_wait(bar_last, 0, abort_flag, timeout_ns, err, kDevTimeoutTmemFull)) {
            tc_fence_after();
            uint32_t r0[32], r1[32], r2[16];
            tmem_ld_32x32b_x32(tmem + lane_base + kTcColO, r0);
            tmem_ld_32x32b_x32(tmem + lane_base + kTcColO + 32u, r1);
            tmem_ld_32x32b_x16(tmem + lane_base + kTcColO + 64u, r2);
            tmem_ld_wait();
            // Every MMA has completed, so the K buffers are free: stage the
            // normalised rows there ([128][76] floats: conflict-free 16-byte
            // stores) and let each warp write its 32 rows whole, 128
            // contiguous bytes per store instruction.
            const float l = __uint_as_float(r2[8]);
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            const uint32_t row = sK + static_cast<uint32_t>(tid) * kTcOutPitch;
#pragma unroll
            for (int d = 0; d < 32; d += 4) {
                sts_v4(row + 4u * d, __float_as_uint(__uint_as_float(r0[d]) * inv),
                       __float_as_uint(__uint_as_float(r0[d + 1]) * inv),
                       __float_as_uint(__uint_as_float(r0[d + 2]) * inv),
                       __float_as_uint(__uint_as_float(r0[d + 3]) * inv));
                sts_v4(row + 128u + 4u * d, __float_as_uint(__uint_as_float(r1[d]) * inv),
                       __float_as_uint(__uint_as_float(r1[d + 1]) * inv),
                       __float_as_uint(__uint_as_float(r1[d + 2]) * inv),
                       __float_as_uint(__uint_as_float(r1[d + 3]) * inv));
            }
#pragma unroll
            for (int d = 0; d < 8; d += 4)
                sts_v4(row + 256u + 4u * d, __float_as_uint(__uint_as_float(r2[d]) * inv),
                       __float_as_uint(__uint_as_float(r2[d + 1]) * inv),
                       __float_as_uint(__uint_as_float(r2[d + 2]) * inv),
                       __float_as_uint(__uint_as_float(r2[d + 3]) * inv));
            __syncwarp();
            const int rows = min(32, t.q_rows - warp * 32);
#pragma unroll 4
            for (int r = 0; r < rows; ++r) {
                const int rr = warp * 32 + r;
                float* dst = out + static_cast<int64_t>(t.o_row0 + rr) * ldo + head * kDH;
                const uint32_t src = sK + static_cast<uint32_t>(rr) * kTcOutPitch;
                dst[lane] = lds_f32(src + 4u * lane);
                dst[32 + lane] = lds_f32(src + 128u + 4u * lane);
                if (lane < 8) dst[64 + lane] = lds_f32(src + 256u + 4u * lane);
            }
        }
    } else if (warp == 4) {
        // ------------------------------------------------------ P V issue
        const bool issuer = lane == 0 && !stall;
        int b3 = 0, u3 = 0;   // j % 3 and j / 3
        for (int j = 0; j < n_kt; ++j) {
            const uint32_t b = j & 1;
            if (!tc_warp_wait(bar_p + 8u * b, (j >> 1) & 1, abort_flag, timeout_ns, err, kDevTimeoutEmpty)) break;
            if (!tc_warp_wait(bar_vf + 8u * b3, u3 & 1, abort_flag, timeout_ns, err, kDevTimeoutFull)) break;
            fence_proxy_async_smem();
            tc_fence_after();
            if (issuer) {
                tc_issue_pv(tmem + kTcColO, tmem + 64u * b, sV + kTcVBuf * b3, j > 0);
                mma_commit(bar_o + 8u * b);
                mma_commit(bar_ve + 8u * b3);
                if (j + 1 == n_kt) mma_commit(bar_last);
            }
            __syncwarp();
            if (++b3 == kTcStages) {
                b3 = 0;
                ++u3;
            }
        }
    } else if (warp == 6) {
        // --------------------------------------------------- score issue
        const bool issuer = lane == 0 && !stall;
        const uint32_t tq = tmem + kTcColQ;
        bool ok = tc_warp_wait(bar_q, 0, abort_flag, timeout_ns, err, kDevTimeoutFull);
        int b3 = 0, u3 = 0;   // j % 3 and j / 3
        for (int j = 0; ok && j < n_kt; ++j) {
            const uint32_t b = j & 1;
            // S(j) overwrites P(j-2) in TMEM buffer b: P(j-2) V(j-2) must
            // have read it
            if (j >= 2 &&
                !tc_warp_wait(bar_o + 8u * b, ((j - 2) >> 1) & 1, abort_flag, timeout_ns, err, kDevTimeoutTmemFull))
                break;
            if (!tc_warp_wait(bar_kf + 8u * b3, u3 & 1, abort_flag, timeout_ns, err, kDevTimeoutFull)) break;
            fence_proxy_async_smem();
            tc_fence_after();
            if (issuer) {
                tc_issue_scores(tmem + 64u * b, tq, sK + kTcKBuf * b3);
                mma_commit(bar_s + 8u * b);
                mma_commit(bar_ke + 8u * b3);
            }
            __syncwarp();
            if (++b3 == kTcStages) {
                b3 = 0;
                ++u3;
            }
        }
    } else if (warp == 5) {
        // ----------------------------------------------------------- loader
        // k_full / v_full [j % 3] phase j / 3 carries tile j; k_empty /
        // v_empty [j % 3] phase j / 3 is S(j) / P(j) V(j).
        // Tiles 0..2 go in the order the MMAs take them: K0 K1 V0 K2 V1 V2.
        // An arrival completes once every earlier copy of its lane has
        // landed, so each one follows its own tile and no later tile.
        for (int i = 0; i < 2 * kTcStages; ++i) {
            const bool is_v = (0x34u >> i) & 1u;                        // K K V K V V
            const int j = static_cast<int>((0x212010u >> (4 * i)) & 0xFu);   // 0 1 0 2 1 2
            if (j >= n_kt) continue;
            if (i > 0) {
                const int k0 = j * kKT, valid = min(kKT, t.k_len - k0);
                if (is_v)
                    tc_load_tile(sV + kTcVBuf * j, vh + static_cast<int64_t>(k0) * ldv, ldv, valid, lane);
                else
                    tc_load_tile(sK + kTcKBuf * j, kh + static_cast<int64_t>(k0) * ldk, ldk, valid, lane);
            }
            cp_async_arrive_noinc((is_v ? bar_vf : bar_kf) + 8u * j);
        }
        int b3 = 0, u3 = 0;   // (j - 3) % 3 == j % 3 and (j - 3) / 3
        for (int j = kTcStages; j < n_kt; ++j) {
            const int k0 = j * kKT, valid = min(kKT, t.k_len - k0);
            if (!tc_warp_wait(bar_ke + 8u * b3, u3 & 1, abort_flag, timeout_ns, err, kDevTimeoutEmpty)) break;
            tc_load_tile(sK + kTcKBuf * b3, kh + static_cast<int64_t>(k0) * ldk, ldk, valid, lane);
            cp_async_arrive_noinc(bar_kf + 8u * b3);
            if (!tc_warp_wait(bar_ve + 8u * b3, u3 & 1, abort_flag, timeout_ns, err, kDevTimeoutEmpty)) break;
            tc_load_tile(sV + kTcVBuf * b3, vh + static_cast<int64_t>(k0) * ldv, ldv, valid, lane);
            cp_async_arrive_noinc(bar_vf + 8u * b3);
            if (++b3 == kTcStages) {
                b3 = 0;
                ++u3;
            }
        }
    }

    // Release: no copy in flight into shared memory, every MMA this CTA
    // issued retired (the issuer's commit below arrives once they all have),
    // every TMEM access landed.
    cp_async_wait<0>();
    tmem_ld_wait();
    tmem_st_wait();
    tc_fence_before();
    __syncthreads();
    if (tid == 128 || tid == 192) {   // the MMA issuers
        tc_fence_after();
        mma_commit(bar_fin);
        if (tid == 128) {
            volatile uint32_t no_abort = 0;
            mbar_wait(bar_fin, 0, &no_abort, 100000000ull);
        }
    }
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTcTmemCols);
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
        for (int q0 = 0; q0 < q_len[s]; q0 += kTileRows) {
            if (n >= max_tiles) return -1;
            t[n].q_row0 = q_off[s] + q0;
            t[n].q_rows = q_len[s] - q0 < kTileRows ? q_len[s] - q0 : kTileRows;
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
    const AttnTile* tiles = static_cast<const AttnTile*>(tiles_dev);
    if (force_exact || (ds && ds->attn_exact)) {
        const float scale = 1.0f / sqrtf(static_cast<float>(kDH));
        dim3 grid(static_cast<unsigned>(2 * n_tiles), static_cast<unsigned>(n_head));
        attention_exact_kernel<<<grid, kExactThreads, 0, s>>>(q, ldq, k, ldk, v, ldv, tiles, out, ldo, scale);
        count_launch();
        return cudaGetLastError();
    }
    const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(kDH));
    if (ds && ds->attn_kernel == 0) {
        static bool tc_configured = false;
        if (!tc_configured) {
            cudaError_t e =
                cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
            if (e != cudaSuccess) return e;
            tc_configured = true;
        }
        dim3 grid(static_cast<unsigned>(n_tiles), static_cast<unsigned>(n_head));
        attention_tc_kernel<<<grid, kTcThreads, kTcSmem, s>>>(q, ldq, k, ldk, v, ldv, tiles, out, ldo, scale_log2,
                                                             ds->err, ds->timeout_ns, ds->test_stall);
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
    dim3 grid(static_cast<unsigned>(2 * n_tiles), static_cast<unsigned>(n_head));
    attention_kernel<<<grid, kWarps * 32, smem, s>>>(q, ldq, k, ldk, v, ldv, tiles, out, ldo, scale_log2);
    count_launch();
    return cudaGetLastError();
}

}  // namespace b2q
