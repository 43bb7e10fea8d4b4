// b2q_gemm.cu — Q8_0 x q8_1 block-scaled GEMM on sm_100a tensor cores.
//
// Semantics (ggml_mul_mat of a Q8_0 weight; restated in the reference at
// src/cuda/siglip2_custom_mmq.cu:229-266):
//     y[m][n] = sum_kb  dW[n,kb] * dX[m,kb] * S[m,n,kb]
//     S[m,n,kb] = sum_{j<32} qX[m,32kb+j] * qW[n,32kb+j]         (int32, exact)
// accumulated over ascending kb as acc = fma((float)S * dW, dX, acc).
//
// Because every 32-wide K block carries its own pair of scales, the int32
// block dot must leave the tensor core once per block.  Each CTA therefore
// computes one 128 x BN output tile as a stream of single-K-block MMAs
// (kind::i8: one K=32 instruction; kind::f16: two K=16 instructions on fp16
// carriers of the same int8 values, exact because every partial sum is an
// integer below 2^24) into a ring of TMEM accumulators (512 columns / BN
// deep), and the epilogue warps rescale-and-accumulate each block in
// registers with packed f32x2 math while the tensor core runs ahead.  That
// rescale (two fp32 operations per output element per K block) bounds the
// kernel, so the epilogue loop carries almost nothing else: ring positions
// advance without divisions, the K-block loop is unrolled per stage, and each
// thread's 32-column TMEM load for the next chunk is in flight while it
// computes the current one.
//
// Warp roles: warpgroup 0 holds the TMA producer (warp 0) and the TMEM owner
// / MMA issuer (warp 1) and gives most of its registers to the epilogue
// warps.  Layouts (GemmCfg): one CTA per SM with eight epilogue warps (two
// per 32-lane TMEM quadrant, each owning half of a 256- or 128-column tile's
// columns), or two CTAs per SM with four epilogue warps each (one per
// quadrant, all of a 128- or 64-column tile's columns).
#include "b2q_internal.h"
#include "b2q_numerics.cuh"
#include "b2q_ptx.cuh"

namespace b2q {

template <int kOps, int kBN, int kCtas>
struct GemmCfg {
    static constexpr int BM = 128;
    static constexpr int BN = kBN;
    static constexpr int CTAS = kCtas;                     // resident CTAs per SM (1 or 2)
    static constexpr int ES = kOps == kOpsF16 ? 2 : 1;
    static constexpr int KROW = 128;                       // bytes of K per smem row per stage
    static constexpr int KBS = KROW / (32 * ES);           // K blocks per stage: 4 (i8) or 2 (f16)
    static constexpr int A_BYTES = BM * KROW;
    static constexpr int B_BYTES = BN * KROW;
    static constexpr int DX_BYTES = KBS * BM * 4;
    static constexpr int DW_BYTES = KBS * BN * 4;
    static constexpr int LOAD_BYTES = A_BYTES + B_BYTES + DX_BYTES + DW_BYTES;   // TMA bytes per stage
    static constexpr int STAGE_BYTES = (LOAD_BYTES + 1023) / 1024 * 1024;      // the swizzle needs 1024-byte stages
    static constexpr int BAR_BYTES = 256;
    // two CTAs share the SM's 228 KB: four stages where they fit in half of it
    static constexpr int STAGES = kCtas == 1 ? 4 : (4 * STAGE_BYTES + BAR_BYTES + 1024 <= 113 * 1024 ? 4 : 3);
    static constexpr int SMEM = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
    // One CTA per SM: eight epilogue warps, two per TMEM lane quadrant, each
    // owning half of the tile's columns.  Two CTAs per SM: four epilogue warps
    // per CTA, one per quadrant, each owning all of its 32 rows' columns; the
    // SM's two CTAs interleave, so one CTA's tile-end epilogue overlaps the
    // other's K-block loop.
    // 192-column tiles: twelve epilogue warps, three per TMEM lane quadrant
    // (and SMSP), each owning 64 of the tile's columns (run_epilogue_w12).
    static constexpr bool W12 = kCtas == 1 && kBN == 192;
    static constexpr int EPI_WARPS = W12 ? 12 : (kCtas == 1 ? 8 : 4);
    static constexpr int THREADS = 128 + EPI_WARPS * 32;   // 512, 384 or 256
    static constexpr int LAUNCH_REGS = kCtas == 1 && !W12 ? 168 : 128;
    static constexpr int WG0_REGS = W12 ? 32 : (kCtas == 1 ? 40 : 24);   // producer / MMA warpgroup after setmaxnreg
    static constexpr int EPI_REGS = W12 ? 160 : 232;
    static constexpr int COLS = BN * 4 / EPI_WARPS;        // columns per epilogue thread
    static constexpr int CC = COLS / 64;                   // 64-column chunks per epilogue thread
    static constexpr int CH = 2 * CC;                      // 16x256b.x8 TMEM loads per K block (2 slabs)
    static constexpr int TMEM_COLS = 512 / kCtas;
    static constexpr int NBUF = TMEM_COLS / BN;            // accumulator ring depth (192 columns: two, 128 unused)
    static_assert(STAGE_BYTES % 1024 == 0, "stage must keep 1024-byte alignment for the swizzle");
    static_assert(CH % 2 == 0, "register double-buffer parity must repeat every K block");
    static_assert(NBUF >= 2, "the accumulator ring needs two buffers");
    static_assert(SMEM * kCtas <= 227 * 1024, "shared memory budget");
    static_assert(LAUNCH_REGS * THREADS * kCtas <= 65536, "launch register budget");
    static_assert(WG0_REGS * 128 + EPI_REGS * EPI_WARPS * 32 <= THREADS * LAUNCH_REGS,
                  "register split exceeds the launch");
};

struct GemmParams {
    int M, N, Kb;
    int m_tiles, n_tiles;
    int nb_off;         // first column tile of this launch (tiles cover columns (nb_off + nb) * BN)
    int epi;
    const float* bias;
    const float* residual;
    void* out;
    int64_t ld_out;
    void* q_out;        // GELU_Q8: values [M][Kp_out]
    float* d_out;       // GELU_Q8: scales [Kp_out/32][d_ld]
    int64_t Kp_out;
    int64_t d_ld;
    int32_t* dump;
    uint32_t* err;
    uint64_t timeout_ns;
    int stall;          // failure-path test: the producer issues nothing, so waits expire
};

__device__ __forceinline__ void raise_error(uint32_t* err, volatile uint32_t* abort_flag, uint32_t code) {
    *abort_flag = 1u;
    atomicCAS(err, 0u, code);
}

template <int kOps>
__device__ __forceinline__ float carrier_to_float(uint32_t r) {
    if constexpr (kOps == kOpsF16) {
        return __uint_as_float(r);              // fp32 accumulator holding an exact integer
    } else {
        return __int2float_rn(static_cast<int32_t>(r));
    }
}

// One 16x256b.x8 chunk: 2 rows (lane t/4 and t/4 + 8 of a 16-lane slab) x
// 8 column pairs.  acc[2g + h] += ((float)S * dW) * dX for row h, pair g.
// w4[i] holds the weight scales of pairs 2i (x, y) and 2i + 1 (z, w).
template <int kOps>
__device__ __forceinline__ void rescale_chunk(float2* acc, const uint32_t (&r)[32], const float4 (&w4)[4], float2 dx0,
                                              float2 dx1) {
#pragma unroll
    for (int g = 0; g < 8; ++g) {
        const float4 wq = w4[g >> 1];
        const float2 w = (g & 1) ? make_float2(wq.z, wq.w) : make_float2(wq.x, wq.y);
        const float2 f0 = make_float2(carrier_to_float<kOps>(r[4 * g + 0]), carrier_to_float<kOps>(r[4 * g + 1]));
        const float2 f1 = make_float2(carrier_to_float<kOps>(r[4 * g + 2]), carrier_to_float<kOps>(r[4 * g + 3]));
        acc[2 * g] = __ffma2_rn(__fmul2_rn(f0, w), dx0, acc[2 * g]);
        acc[2 * g + 1] = __ffma2_rn(__fmul2_rn(f1, w), dx1, acc[2 * g + 1]);
    }
}

// Ring position: index and phase bit, advanced without divisions.
template <int N>
struct Ring {
    uint32_t idx = 0, phase = 0;
    __device__ __forceinline__ void next() {
        if (++idx == N) {
            idx = 0;
            phase ^= 1u;
        }
    }
};

// Shared-memory layout, as 32-bit shared-window addresses: the stages, then
// the barrier arrays (8 bytes per barrier).
struct Smem {
    uint32_t base;
    uint32_t full;      // [STAGES] TMA landed
    uint32_t empty;     // [STAGES] MMA + epilogue done with the stage
    uint32_t tfull;     // [NBUF]   accumulator ready
    uint32_t tempty;    // [NBUF]   accumulator drained
    volatile uint32_t* abort_flag;
};

__device__ __forceinline__ uint32_t bar_at(uint32_t arr, uint32_t i) { return arr + 8u * i; }

// ---------------------------------------------------------------- producer
template <int kOps, int kBN, int kCtas>
__device__ bool run_producer(const Smem& sm, const CUtensorMap* tmA, const CUtensorMap* tmB, const CUtensorMap* tmDX,
                             const CUtensorMap* tmDW, const GemmParams& p, uint32_t& issued) {
    using Cfg = GemmCfg<kOps, kBN, kCtas>;
    const int num_tiles = p.m_tiles * p.n_tiles;
    const int nst = (p.Kb + Cfg::KBS - 1) / Cfg::KBS;
    if (p.stall) return true;   // nothing issued: the consumers' bounded waits run out
    Ring<Cfg::STAGES> st_ring;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        const int mb = tile / p.n_tiles, nb = tile - (tile / p.n_tiles) * p.n_tiles + p.nb_off;
        for (int st = 0; st < nst; ++st) {
            const uint32_t s = st_ring.idx;
            if (!mbar_wait(bar_at(sm.empty, s), st_ring.phase ^ 1u, sm.abort_flag, p.timeout_ns)) {
                raise_error(p.err, sm.abort_flag, kDevTimeoutEmpty);
                return false;
            }
            const uint32_t sbase = sm.base + s * Cfg::STAGE_BYTES;
            const uint32_t fb = bar_at(sm.full, s);
            mbar_arrive_expect_tx(fb, Cfg::LOAD_BYTES);
            const int kx = st * (Cfg::KROW / Cfg::ES);
            tma_load_2d(sbase, tmA, fb, kx, mb * Cfg::BM);
            tma_load_2d(sbase + Cfg::A_BYTES, tmB, fb, kx, nb * Cfg::BN);
            tma_load_2d(sbase + Cfg::A_BYTES + Cfg::B_BYTES, tmDX, fb, mb * Cfg::BM, st * Cfg::KBS);
            tma_load_2d(sbase + Cfg::A_BYTES + Cfg::B_BYTES + Cfg::DX_BYTES, tmDW, fb, nb * Cfg::BN, st * Cfg::KBS);
            ++issued;
            st_ring.next();
        }
    }
    return true;
}

// ---------------------------------------------------------------- MMA issuer
template <int kOps, int kBN, int kCtas>
__device__ bool run_mma(const Smem& sm, uint32_t tmem_base, const GemmParams& p, uint32_t& issued) {
    using Cfg = GemmCfg<kOps, kBN, kCtas>;
    const uint32_t idesc = kOps == kOpsF16 ? idesc_f16_f32(Cfg::BM, Cfg::BN) : idesc_i8_s32(Cfg::BM, Cfg::BN);
    const int num_tiles = p.m_tiles * p.n_tiles;
    const int nst = (p.Kb + Cfg::KBS - 1) / Cfg::KBS;
    Ring<Cfg::STAGES> st_ring;
    Ring<Cfg::NBUF> acc_ring;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        for (int st = 0; st < nst; ++st) {
            const uint32_t s = st_ring.idx;
            if (!mbar_wait(bar_at(sm.full, s), st_ring.phase, sm.abort_flag, p.timeout_ns)) {
                raise_error(p.err, sm.abort_flag, kDevTimeoutFull);
                return false;
            }
            tc_fence_after();
            const uint32_t a_base = sm.base + s * Cfg::STAGE_BYTES;
            const uint32_t b_base = a_base + Cfg::A_BYTES;
            const int nkb = min(Cfg::KBS, p.Kb - st * Cfg::KBS);
            for (int j = 0; j < nkb; ++j) {
                const uint32_t b = acc_ring.idx;
                if (!mbar_wait(bar_at(sm.tempty, b), acc_ring.phase ^ 1u, sm.abort_flag, p.timeout_ns)) {
                    raise_error(p.err, sm.abort_flag, kDevTimeoutTmemEmpty);
                    return false;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + b * Cfg::BN;
                if constexpr (kOps == kOpsF16) {
                    mma_f16(d, smem_desc_k_sw128(a_base + j * 64), smem_desc_k_sw128(b_base + j * 64), idesc, 0u);
                    mma_f16(d, smem_desc_k_sw128(a_base + j * 64 + 32), smem_desc_k_sw128(b_base + j * 64 + 32), idesc,
                            1u);
                } else {
                    mma_i8(d, smem_desc_k_sw128(a_base + j * 32), smem_desc_k_sw128(b_base + j * 32), idesc, 0u);
                }
                mma_commit(bar_at(sm.tfull, b));
                ++issued;
                acc_ring.next();
            }
            mma_commit(bar_at(sm.empty, s));
            st_ring.next();
        }
    }
    return true;
}

// ---------------------------------------------------------------- epilogue
//
// Thread geometry.  Epilogue warp ew (0..7) reads TMEM lane quadrant
// quad = warp % 4 (the only lanes a warp may access) and column half
// ew / 4 of the tile, through 16x256b loads: lane t holds rows
// quad*32 + 16s + t/4 + 8h (slab s, h in {0,1}) and the column pairs
// 64cc + 8g + 2(t%4) + {0,1} of its half (64-column chunk cc, pair g < 8).
// Chunk c = 2cc + s is one 32-register load; acc[16c + 2g + h] is the pair
// (g, h).  Holding four rows and 32 columns (instead of one row and all 128
// columns) makes each shared-memory scale load serve four rows, which keeps
// the per-block rescale off the shared-memory pipe.

constexpr int kResBatch = 4;   // column groups (of 8) per batch of residual loads in store_tile

template <int kOps, int kBN, int kCtas>
__device__ __forceinline__ void store_tile(const GemmParams& p, float2* acc, int mrow0, int nblk0, int q) {
    using Cfg = GemmCfg<kOps, kBN, kCtas>;
    if (p.epi == B2Q_EPI_BIAS_GELU_Q8) {
        // In phases over the whole tile, so that the independent element
        // chains overlap: bias + GELU in place for all 64 pairs, then each
        // (row, 32-column block)'s absmax and scales, then rounding and
        // stores.  Per element the operations are those of the q8_1 rule.
#pragma unroll
        for (int cc = 0; cc < Cfg::CC; ++cc)
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                const int n = nblk0 + cc * 64 + 8 * g + 2 * q;
                const float2 b = (p.bias && n < p.N) ? *reinterpret_cast<const float2*>(p.bias + n) : make_float2(0.0f, 0.0f);
#pragma unroll
                for (int s = 0; s < 2; ++s)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        float2& a = acc[16 * (2 * cc + s) + 2 * g + h];
                        a = gelu2(__fadd2_rn(a, b));
                    }
            }
        // absmax of each (row, block): this thread's 8 values, then the 4 lanes sharing t/4
        float amax[Cfg::CC][2][2][2];
#pragma unroll
        for (int cc = 0; cc < Cfg::CC; ++cc)
#pragma unroll
            for (int bl = 0; bl < 2; ++bl)
#pragma unroll
                for (int s = 0; s < 2; ++s)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        float m = 0.0f;
#pragma unroll
                        for (int gg = 0; gg < 4; ++gg) {
                            const float2 v = acc[16 * (2 * cc + s) + 2 * (4 * bl + gg) + h];
                            m = fmaxf(m, fmaxf(fabsf(v.x), fabsf(v.y)));
                        }
                        amax[cc][bl][s][h] = m;
                    }
#pragma unroll
        for (int cc = 0; cc < Cfg::CC; ++cc)
#pragma unroll
            for (int bl = 0; bl < 2; ++bl)
#pragma unroll
                for (int s = 0; s < 2; ++s)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        float& m = amax[cc][bl][s][h];
                        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
                        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
                    }
#pragma unroll
        for (int cc = 0; cc < Cfg::CC; ++cc) {
#pragma unroll
            for (int bl = 0; bl < 2; ++bl) {
                const int n0 = nblk0 + cc * 64 + bl * 32;        // q8_1 block start (warp-uniform)
                if (n0 >= p.Kp_out) continue;
#pragma unroll
                for (int s = 0; s < 2; ++s) {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int m = mrow0 + 16 * s + 8 * h;
                        if (m >= p.M) continue;
                        const float a = amax[cc][bl][s][h];
                        if (q == 0) p.d_out[static_cast<int64_t>(n0 / 32) * p.d_ld + m] = q8_scale(a);
                        const float inv = q8_inv_scale(a);
#pragma unroll
                        for (int gg = 0; gg < 4; ++gg) {
                            const float2 v = acc[16 * (2 * cc + s) + 2 * (4 * bl + gg) + h];
                            const int64_t off = static_cast<int64_t>(m) * p.Kp_out + n0 + 8 * gg + 2 * q;
                            if constexpr (kOps == kOpsF16) {
                                // q = rint(x * inv) on the fp32 adder (q8_round_adder2); |x| <= a
                                // bounds |x * inv| below 127.5, so q needs no clamp, and the
                                // integer packs into its fp16 carrier exactly
                                const float2 qf = q8_round_adder2(v, inv);
                                reinterpret_cast<__half2*>(reinterpret_cast<__half*>(p.q_out) + off)[0] =
                                    __floats2half2_rn(qf.x, qf.y);
                            } else {
                                const int32_t q0 = q8_round(v.x, inv), q1 = q8_round(v.y, inv);
                                const uint32_t lo = static_cast<uint32_t>(q0) & 0xFFu;
                                const uint32_t hi = static_cast<uint32_t>(q1) & 0xFFu;
                                reinterpret_cast<uint16_t*>(reinterpret_cast<int8_t*>(p.q_out) + off)[0] =
                                    static_cast<uint16_t>(lo | (hi << 8));
                            }
                        }
                    }
                }
            }
        }
    } else if (p.epi == B2Q_EPI_BIAS_F16) {
        __half* out = reinterpret_cast<__half*>(p.out);
#pragma unroll
        for (int cc = 0; cc < Cfg::CC; ++cc) {
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                const int n = nblk0 + cc * 64 + 8 * g + 2 * q;
                if (n >= p.N) continue;
                const float2 b = p.bias ? *reinterpret_cast<const float2*>(p.bias + n) : make_float2(0.0f, 0.0f);
#pragma unroll
                for (int s = 0; s < 2; ++s) {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int m = mrow0 + 16 * s + 8 * h;
                        if (m >= p.M) continue;
                        const float2 a = acc[16 * (2 * cc + s) + 2 * g + h];
                        *reinterpret_cast<__half2*>(out + static_cast<int64_t>(m) * p.ld_out + n) =
                            __floats2half2_rn(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y));
                    }
                }
            }
        }
    } else {
        float* out = reinterpret_cast<float*>(p.out);
        const bool add_bias = p.epi != B2Q_EPI_NONE && p.bias;
        const bool add_res = p.epi == B2Q_EPI_BIAS_RESIDUAL;
        // In batches of kResBatch column groups: the batch's residual values are all
        // loaded before any of its outputs is stored.  Each thread reads
        // exactly the elements it writes (the residual may be the output
        // itself), so the early loads are safe, and one memory latency per
        // batch replaces one per element pair.
#pragma unroll
        for (int cc = 0; cc < Cfg::CC; ++cc) {
#pragma unroll
            for (int g0 = 0; g0 < 8; g0 += kResBatch) {
                float2 r[kResBatch][2][2];
#pragma unroll
                for (int g = 0; g < kResBatch; ++g)
#pragma unroll
                    for (int s = 0; s < 2; ++s)
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int n = nblk0 + cc * 64 + 8 * (g0 + g) + 2 * q;
                            const int m = mrow0 + 16 * s + 8 * h;
                            r[g][s][h] = (add_res && n < p.N && m < p.M)
                                             ? *reinterpret_cast<const float2*>(p.residual +
                                                                                static_cast<int64_t>(m) * p.ld_out + n)
                                             : make_float2(0.0f, 0.0f);
                        }
#pragma unroll
                for (int g = 0; g < kResBatch; ++g) {
                    const int n = nblk0 + cc * 64 + 8 * (g0 + g) + 2 * q;
                    if (n >= p.N) continue;
                    const float2 b = add_bias ? *reinterpret_cast<const float2*>(p.bias + n) : make_float2(0.0f, 0.0f);
#pragma unroll
                    for (int s = 0; s < 2; ++s) {
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int m = mrow0 + 16 * s + 8 * h;
                            if (m >= p.M) continue;
                            float2 v = acc[16 * (2 * cc + s) + 2 * (g0 + g) + h];
                            if (add_bias) {
                                v.x = __fadd_rn(v.x, b.x);
                                v.y = __fadd_rn(v.y, b.y);
                            }
                            if (add_res) {
                                v.x = __fadd_rn(v.x, r[g][s][h].x);
                                v.y = __fadd_rn(v.y, r[g][s][h].y);
                            }
                            *reinterpret_cast<float2*>(out + static_cast<int64_t>(m) * p.ld_out + n) = v;
                        }
                    }
                }
            }
        }
    }
}

template <int kOps, int kBN, int kCtas, bool kDump>
__device__ bool run_epilogue(const Smem& sm, uint32_t tmem_base, const GemmParams& p, int warp, int lane) {
    using Cfg = GemmCfg<kOps, kBN, kCtas>;
    const int ew = warp - 4;
    const int quad = warp & 3;                  // TMEM lane quadrant this warp may access
    const int col0 = (ew >> 2) * Cfg::COLS;     // first column of this warp's half of the tile
    const int q = lane & 3;
    const int rloc = quad * 32 + (lane >> 2);   // tile row of (slab 0, h 0)
    const uint32_t taddr0 = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + col0;
    const int num_tiles = p.m_tiles * p.n_tiles;
    const int nst = (p.Kb + Cfg::KBS - 1) / Cfg::KBS;
    Ring<Cfg::STAGES> st_ring;
    Ring<Cfg::NBUF> acc_ring;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        const int mb = tile / p.n_tiles, nb = tile - (tile / p.n_tiles) * p.n_tiles + p.nb_off;
        const int mrow0 = mb * Cfg::BM + rloc;
        const int nblk0 = nb * Cfg::BN + col0;
        float2 acc[Cfg::COLS / 2];
#pragma unroll
        for (int i = 0; i < Cfg::COLS / 2; ++i) acc[i] = make_float2(0.0f, 0.0f);
        uint32_t ra[32], rb[32];
        if (!mbar_wait(bar_at(sm.tfull, acc_ring.idx), acc_ring.phase, sm.abort_flag, p.timeout_ns)) {
            raise_error(p.err, sm.abort_flag, kDevTimeoutTmemFull);
            return false;
        }
        tc_fence_after();
        tmem_ld_16x256b_x8(taddr0 + acc_ring.idx * Cfg::BN, ra);
        int kb = 0;
        bool stage_ready = false;   // set by an early probe of the next stage's barrier
        for (int st = 0; st < nst; ++st) {
            const uint32_t s = st_ring.idx;
            if (!stage_ready && !mbar_wait(bar_at(sm.full, s), st_ring.phase, sm.abort_flag, p.timeout_ns)) {
                raise_error(p.err, sm.abort_flag, kDevTimeoutFull);
                return false;
            }
            const uint32_t sbase = sm.base + s * Cfg::STAGE_BYTES;
            const uint32_t sdx = sbase + Cfg::A_BYTES + Cfg::B_BYTES + rloc * 4;             // dX[j][row]
            // dW[j][slot]: this thread's 16-byte vectors sit at slots 16i + 4q of each 64-column chunk
            const uint32_t sdw = sbase + Cfg::A_BYTES + Cfg::B_BYTES + Cfg::DX_BYTES + (col0 + 4 * q) * 4;
            const int nkb = min(Cfg::KBS, p.Kb - st * Cfg::KBS);
            stage_ready = false;
#pragma unroll
            for (int j = 0; j < Cfg::KBS; ++j) {
                if (j < nkb) {
                    float2 dx[2][2];
#pragma unroll
                    for (int sl = 0; sl < 2; ++sl)
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const float v = lds_f32(sdx + (j * Cfg::BM + 16 * sl + 8 * h) * 4);
                            dx[sl][h] = make_float2(v, v);
                        }
                    const uint32_t w2 = sdw + j * Cfg::BN * 4;
                    float4 wv[Cfg::CC][4];
#pragma unroll
                    for (int cc = 0; cc < Cfg::CC; ++cc)
#pragma unroll
                        for (int i = 0; i < 4; ++i) wv[cc][i] = lds_v4_f32(w2 + (cc * 64 + 16 * i) * 4);
                    const bool has_next = kb + 1 < p.Kb;
                    // the next accumulator's barrier is probed one chunk before its first
                    // load, so the probe's round trip overlaps this chunk's arithmetic
                    bool next_ready = false;
#pragma unroll
                    for (int c = 0; c < Cfg::CH; ++c) {
                        uint32_t(&cur)[32] = (c & 1) ? rb : ra;
                        uint32_t(&nxt)[32] = (c & 1) ? ra : rb;
                        tmem_ld_wait_regs(cur);
                        if (c == Cfg::CH - 1) {
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(bar_at(sm.tempty, acc_ring.idx));
                            acc_ring.next();
                            if (has_next) {
                                if (!next_ready &&
                                    !mbar_wait(bar_at(sm.tfull, acc_ring.idx), acc_ring.phase, sm.abort_flag, p.timeout_ns)) {
                                    raise_error(p.err, sm.abort_flag, kDevTimeoutTmemFull);
                                    return false;
                                }
                                tc_fence_after();
                                tmem_ld_16x256b_x8(taddr0 + acc_ring.idx * Cfg::BN, nxt);
                            }
                        } else {
                            const int c1 = c + 1;
                            tmem_ld_16x256b_x8(taddr0 + acc_ring.idx * Cfg::BN +
                                                   (static_cast<uint32_t>((c1 & 1) * 16) << 16) + (c1 >> 1) * 64,
                                               nxt);
                            if (c == Cfg::CH - 2 && has_next) {
                                Ring<Cfg::NBUF> nb = acc_ring;
                                nb.next();
                                next_ready = mbar_test_wait(bar_at(sm.tfull, nb.idx), nb.phase);
                                if (j == nkb - 1) {   // the next block starts the next stage
                                    Ring<Cfg::STAGES> ns = st_ring;
                                    ns.next();
                                    stage_ready = mbar_test_wait(bar_at(sm.full, ns.idx), ns.phase);
                                }
                            }
                        }
                        if constexpr (kDump) {
                            const int sl = c & 1, cc = c >> 1;
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const int m = mrow0 + 16 * sl + 8 * h;
                                if (m >= p.M) continue;
                                int32_t* drow = p.dump + (static_cast<int64_t>(kb) * p.M + m) * p.N;
#pragma unroll
                                for (int g = 0; g < 8; ++g) {
                                    const int n = nblk0 + cc * 64 + 8 * g + 2 * q;
                                    if (n >= p.N) continue;
                                    drow[n] = static_cast<int32_t>(carrier_to_float<kOps>(cur[4 * g + 2 * h]));
                                    drow[n + 1] = static_cast<int32_t>(carrier_to_float<kOps>(cur[4 * g + 2 * h + 1]));
                                }
                            }
                        } else {
                            rescale_chunk<kOps>(acc + 16 * c, cur, wv[c >> 1], dx[c & 1][0], dx[c & 1][1]);
                        }
                    }
                    ++kb;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_at(sm.empty, s));
            st_ring.next();
        }
        if constexpr (!kDump) store_tile<kOps, kBN, kCtas>(p, acc, mrow0, nblk0, q);
    }
    return true;
}


// 192-column tiles, twelve epilogue warps (three per SMSP): each thread holds
// 4 rows x 16 columns, and a K block is one short chain per warp: wait for
// the accumulator, both 16-lane slabs' loads and the block's scales issued
// together, one wait, the buffer released at once (before the arithmetic),
// then 64 packed rescale instructions.  The SMSP's other two epilogue warps
// cover the chain's latencies, so the loop carries no intra-warp double
// buffering and no early probes, which leaves about 85 other instructions
// per block (against ~180 in the two-warp loop above); the stage is released
// once every lane has used its scales.
template <int kOps>
__device__ bool run_epilogue_w12(const Smem& sm, uint32_t tmem_base, const GemmParams& p, int warp, int lane) {
    using Cfg = GemmCfg<kOps, 192, 1>;
    const int ew = warp - 4;
    const int quad = warp & 3;                  // TMEM lane quadrant this warp may access
    const int col0 = (ew >> 2) * 64;            // first of this warp's 64 columns
    const int q = lane & 3;
    const int rloc = quad * 32 + (lane >> 2);
    const uint32_t taddr0 = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + col0;
    const uint32_t dx_off = Cfg::A_BYTES + Cfg::B_BYTES + rloc * 4;
    // dW[j][slot]: this thread's 16-byte vectors sit at slots 16i + 4q of its 64-column group
    const uint32_t dw_off = Cfg::A_BYTES + Cfg::B_BYTES + Cfg::DX_BYTES + (col0 + 4 * q) * 4;
    const int num_tiles = p.m_tiles * p.n_tiles;
    Ring<Cfg::NBUF> acc_ring;
    Ring<Cfg::STAGES> st_ring;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        const int mb = tile / p.n_tiles, nb = tile - (tile / p.n_tiles) * p.n_tiles + p.nb_off;
        const int mrow0 = mb * Cfg::BM + rloc;
        const int nblk0 = nb * Cfg::BN + col0;
        float2 acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = make_float2(0.0f, 0.0f);
        int j = 0;   // K block inside the current stage
        for (int kb = 0; kb < p.Kb; ++kb) {
            if (j == 0 && !mbar_wait(bar_at(sm.full, st_ring.idx), st_ring.phase, sm.abort_flag, p.timeout_ns)) {
                raise_error(p.err, sm.abort_flag, kDevTimeoutFull);
                return false;
            }
            if (!mbar_wait(bar_at(sm.tfull, acc_ring.idx), acc_ring.phase, sm.abort_flag, p.timeout_ns)) {
                raise_error(p.err, sm.abort_flag, kDevTimeoutTmemFull);
                return false;
            }
            tc_fence_after();
            uint32_t r0[32], r1[32];
            const uint32_t ta = taddr0 + acc_ring.idx * Cfg::BN;
            tmem_ld_16x256b_x8(ta, r0);
            tmem_ld_16x256b_x8(ta + (16u << 16), r1);
            const uint32_t sb = sm.base + st_ring.idx * Cfg::STAGE_BYTES;
            const uint32_t sdx = sb + dx_off + j * Cfg::BM * 4;   // rows +0, +8, +16, +24
            const float d00 = lds_f32(sdx), d01 = lds_f32(sdx + 32), d10 = lds_f32(sdx + 64), d11 = lds_f32(sdx + 96);
            const uint32_t sdw = sb + dw_off + j * Cfg::BN * 4;
            float4 wv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) wv[i] = lds_v4_f32(sdw + 64 * i);
            tmem_ld_wait_regs(r0);
            tmem_ld_wait_regs(r1);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_at(sm.tempty, acc_ring.idx));
            acc_ring.next();
            rescale_chunk<kOps>(acc, r0, wv, make_float2(d00, d00), make_float2(d01, d01));
            rescale_chunk<kOps>(acc + 16, r1, wv, make_float2(d10, d10), make_float2(d11, d11));
            if (++j == Cfg::KBS || kb + 1 == p.Kb) {   // every lane has used this stage's scales
                __syncwarp();
                if (lane == 0) mbar_arrive(bar_at(sm.empty, st_ring.idx));
                st_ring.next();
                j = 0;
            }
        }
        store_tile<kOps, 192, 1>(p, acc, mrow0, nblk0, q);
    }
    return true;
}

template <int kOps, int kBN, int kCtas, bool kDump>
__global__ void __launch_bounds__(GemmCfg<kOps, kBN, kCtas>::THREADS, kCtas)
gemm_q8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmDX, const __grid_constant__ CUtensorMap tmDW,
               const GemmParams p) {
    using Cfg = GemmCfg<kOps, kBN, kCtas>;
    extern __shared__ uint8_t smem_raw[];
    Smem sm;
    // the 128-byte swizzle needs 1024-byte aligned stages
    uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* bars = base + Cfg::STAGES * Cfg::STAGE_BYTES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8 * (2 * Cfg::STAGES + 2 * Cfg::NBUF));
    sm.base = smem_u32(base);
    sm.full = smem_u32(bars);
    sm.empty = sm.full + 8 * Cfg::STAGES;
    sm.tfull = sm.empty + 8 * Cfg::STAGES;
    sm.tempty = sm.tfull + 8 * Cfg::NBUF;
    sm.abort_flag = tmem_slot + 1;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::STAGES; ++s) {
            mbar_init(bar_at(sm.full, s), 1);
            mbar_init(bar_at(sm.empty, s), 1 + Cfg::EPI_WARPS);
        }
        for (int b = 0; b < Cfg::NBUF; ++b) {
            mbar_init(bar_at(sm.tfull, b), 1);
            mbar_init(bar_at(sm.tempty, b), Cfg::EPI_WARPS);
        }
        *sm.abort_flag = 0u;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp < 4) {
        warpgroup_reg_dealloc<Cfg::WG0_REGS>();
        if (warp == 0 && lane == 0) {
            tma_prefetch_desc(&tmA);
            tma_prefetch_desc(&tmB);
            tma_prefetch_desc(&tmDX);
            tma_prefetch_desc(&tmDW);
            uint32_t issued = 0;
            run_producer<kOps, kBN, kCtas>(sm, &tmA, &tmB, &tmDX, &tmDW, p, issued);
            // drain: never leave a copy in flight into this CTA's shared memory
            const uint32_t n_drain = issued < Cfg::STAGES ? issued : Cfg::STAGES;
            for (uint32_t i = 0; i < n_drain; ++i) {
                const uint32_t g = issued - 1 - i;
                volatile uint32_t no_abort = 0;
                mbar_wait(bar_at(sm.full, g % Cfg::STAGES), (g / Cfg::STAGES) & 1u, &no_abort, 100000000ull);
            }
        } else if (warp == 1 && lane == 0) {
            uint32_t issued = 0;
            run_mma<kOps, kBN, kCtas>(sm, tmem_base, p, issued);
            // every issued MMA must have retired before TMEM is released
            if (issued > 0) {
                volatile uint32_t no_abort = 0;
                const uint32_t g = issued - 1;
                mbar_wait(bar_at(sm.tfull, g % Cfg::NBUF), (g / Cfg::NBUF) & 1u, &no_abort, 100000000ull);
            }
        }
    } else {
        warpgroup_reg_alloc<Cfg::EPI_REGS>();
        if constexpr (Cfg::W12 && !kDump)
            run_epilogue_w12<kOps>(sm, tmem_base, p, warp, lane);
        else
            run_epilogue<kOps, kBN, kCtas, kDump>(sm, tmem_base, p, warp, lane);
        // an epilogue that gave up on an expired wait may still have a TMEM
        // load in flight: let it land before TMEM is released
        tmem_ld_wait();
        tc_fence_before();
    }

    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
    }
}

// ------------------------------------------------------------------ host side

template <int kOps, int kBN, int kCtas, bool kDump>
static cudaError_t configure_once() {
    static bool done = false;
    if (done) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(gemm_q8_kernel<kOps, kBN, kCtas, kDump>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         GemmCfg<kOps, kBN, kCtas>::SMEM);
    if (e == cudaSuccess) done = true;
    return e;
}

// Output columns [n_base, n_base + n_cols) of the GEMM, in kBN-column tiles
// (n_base a multiple of kBN).
template <int kOps, int kBN, int kCtas, bool kDump>
static b2q_status run_gemm(const GemmArgs& a, cudaStream_t s, int64_t n_base, int64_t n_cols) {
    using Cfg = GemmCfg<kOps, kBN, kCtas>;
    DeviceState* ds = state();
    const b2q_weight* w = a.w;
    const ActLayout L = act_layout(a.M, w->K, kOps);
    const CUtensorMapDataType dt = kOps == kOpsF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
    CUtensorMap tmA, tmDX;
    const uint8_t* act = static_cast<const uint8_t*>(a.act);
    if (!make_tmap_2d(&tmA, dt, act, L.Kp, L.M, L.Kp * L.es, Cfg::KROW / Cfg::ES, Cfg::BM, true) ||
        !make_tmap_2d(&tmDX, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, act + L.d_offset, L.M, L.Kb, L.ld * 4, Cfg::BM,
                      Cfg::KBS, false))
        return set_error(B2Q_ERR_CUDA, "cuTensorMapEncodeTiled failed for the activation planes");
    const CUtensorMap* tmB = kBN == 256 ? &w->tm_q256 : kBN == 192 ? &w->tm_q192 : kBN == 128 ? &w->tm_q128 : &w->tm_q64;
    const CUtensorMap* tmDW = kBN == 256 ? &w->tm_d256 : kBN == 192 ? &w->tm_d192 : kBN == 128 ? &w->tm_d128 : &w->tm_d64;

    GemmParams p{};
    p.M = static_cast<int>(a.M);
    p.N = static_cast<int>(w->N);
    p.Kb = static_cast<int>(w->Kb);
    p.m_tiles = static_cast<int>((a.M + Cfg::BM - 1) / Cfg::BM);
    p.n_tiles = static_cast<int>((n_cols + Cfg::BN - 1) / Cfg::BN);
    p.nb_off = static_cast<int>(n_base / Cfg::BN);
    p.epi = a.epi;
    p.bias = a.bias;
    p.residual = a.residual;
    p.out = a.out;
    p.ld_out = a.ld_out > 0 ? a.ld_out : w->N;
    p.dump = a.dump;
    p.err = ds->err;
    p.timeout_ns = ds->timeout_ns;
    p.stall = ds->test_stall;
    if (a.epi == B2Q_EPI_BIAS_GELU_Q8) {
        const ActLayout O = act_layout(a.M, w->N, kOps);
        p.q_out = a.act_out;
        p.d_out = reinterpret_cast<float*>(static_cast<uint8_t*>(a.act_out) + O.d_offset);
        p.Kp_out = O.Kp;
        p.d_ld = O.ld;
    }
    cudaError_t e = configure_once<kOps, kBN, kCtas, kDump>();
    if (e != cudaSuccess) return cuda_check(e, "cudaFuncSetAttribute(gemm)");
    const int tiles = p.m_tiles * p.n_tiles;
    const int slots = ds->num_sms * kCtas;
    const int grid = tiles < slots ? tiles : slots;
    gemm_q8_kernel<kOps, kBN, kCtas, kDump><<<grid, Cfg::THREADS, Cfg::SMEM, s>>>(tmA, *tmB, tmDX, *tmDW, p);
    count_launch();
    return cuda_check(cudaGetLastError(), "gemm launch");
}

// 256-column tiles leave the last tile of N part empty when N is not a
// multiple of 256 (N = 1152: five tiles for 4.5 tiles of work, and the
// epilogue costs the same for the empty half).  When the remainder fits one
// 128-column tile, the columns are covered by two launches instead: 256-wide
// tiles up to the last multiple of 256, then 128-wide tiles for the rest.
// Every output element is computed exactly as in a single launch.
static int64_t split_remainder(int64_t N) {
    const int64_t rem = N % 256;
    return (N > 256 && rem != 0 && rem <= 128) ? rem : 0;
}

template <int kOps>
static b2q_status dispatch_bn(const GemmArgs& a, cudaStream_t s, int bn, int ctas, bool split) {
    const int64_t N = a.w->N;
    if (a.dump) return run_gemm<kOps, 128, 1, true>(a, s, 0, N);
    if (bn == 64) return run_gemm<kOps, 64, 2, false>(a, s, 0, N);   // 64-column tiles exist in the two-CTA form
    if (bn == 192) return run_gemm<kOps, 192, 1, false>(a, s, 0, N);  // 192-column tiles: one CTA, twelve epilogue warps
    if (ctas == 2) return run_gemm<kOps, 128, 2, false>(a, s, 0, N);
    if (bn != 256) return run_gemm<kOps, 128, 1, false>(a, s, 0, N);
    const int64_t rem = split ? split_remainder(N) : 0;
    if (rem == 0) return run_gemm<kOps, 256, 1, false>(a, s, 0, N);
    b2q_status st = run_gemm<kOps, 256, 1, false>(a, s, 0, N - rem);
    if (st != B2Q_OK) return st;
    return run_gemm<kOps, 128, 1, false>(a, s, N - rem, rem);
}

// Tile width when not forced by B2Q_TUNE_GEMM_BN: whichever of 256 and 128
// columns finishes the persistent grid's tile rounds sooner, with a
// 128-column tile costing about 0.6 of a 256-column one (it carries the same
// per-K-block synchronisation for half the columns), and the 256 option
// counting its split remainder launch.  Large M keeps 256; small M (few
// tiles, or a last round that is mostly empty) takes 128.
static int auto_bn(int64_t M, int64_t N, int num_sms) {
    const int64_t mt = (M + 127) / 128;
    const int64_t rem = split_remainder(N);
    const double r256 = rem ? static_cast<double>((mt * (N / 256) + num_sms - 1) / num_sms) +
                                  0.6 * static_cast<double>((mt + num_sms - 1) / num_sms)
                            : static_cast<double>((mt * ((N + 255) / 256) + num_sms - 1) / num_sms);
    const int64_t r128 = (mt * ((N + 127) / 128) + num_sms - 1) / num_sms;
    return 0.6 * static_cast<double>(r128) < 0.95 * r256 ? 128 : 256;
}

// Two CTAs per SM (128-column tiles, four epilogue warps each) when the
// 128-column tiles give every SM at least one, except for the GELU -> q8_1
// epilogue.  Measured at 65,536 and 313,755 tokens: QKV (fp16 out) +5%, O
// projection and fc2 (bias + residual) +8%, fc1 with fp32 output +1-3%; the
// GELU tile end, whose cost per thread is the same in both layouts, runs 3%
// slower as two 128-column tiles.  At 54 tiles (729 tokens, N = 1152) the
// eight-warp single CTA is faster.
static int auto_ctas(int64_t M, int64_t N, int epi, int num_sms) {
    if (epi == B2Q_EPI_BIAS_GELU_Q8) return 1;
    const int64_t tiles128 = ((M + 127) / 128) * ((N + 127) / 128);
    return tiles128 >= num_sms ? 2 : 1;
}

// Fewer 128-column tiles than SMs (small M): 64-column tiles, two CTAs per
// SM, double the tiles.  Measured at M = 320-2,048: the N = 1152 projections
// (O, fc2) gain 12-22% (fc2 at M = 729: 104 -> 126 TOPS), the wider ones are
// within 2% of the best layout.
static bool small_tiles(int64_t M, int64_t N, int num_sms) {
    return ((M + 127) / 128) * ((N + 127) / 128) < num_sms;
}

// 192-column tiles (one CTA per SM, twelve epilogue warps) against the
// layout chosen otherwise, by the tile rounds each needs: at large M a
// 192-column tile takes about 0.714 of the time of a pair of co-resident
// 128-column tiles (measured: +3 to +8% over the two-CTA and 256-column
// layouts at 65,536 and 313,755 tokens, bit-identical), so they win unless
// their last round is mostly empty; with fewer 128-column tiles than SMs
// (the 64-column regime) they win when one round of them replaces two or
// more rounds of 64-column tiles (QKV and fc1 at 729 tokens: +23%).
static bool use_w12(int64_t M, int64_t N, int epi, int num_sms) {
    const int64_t mt = (M + 127) / 128;
    const int64_t t192 = mt * ((N + 191) / 192);
    const double r192 = 0.714 * static_cast<double>((t192 + num_sms - 1) / num_sms);
    if (small_tiles(M, N, num_sms)) {
        const int64_t t64 = mt * ((N + 63) / 64);
        return t192 <= num_sms && t64 > 2 * num_sms;
    }
    double other;
    if (epi == B2Q_EPI_BIAS_GELU_Q8) {
        other = static_cast<double>((mt * ((N + 255) / 256) + num_sms - 1) / num_sms);
    } else {
        other = static_cast<double>((mt * ((N + 127) / 128) + 2 * num_sms - 1) / (2 * num_sms));
    }
    return r192 < 0.98 * other;
}

b2q_status launch_gemm(const GemmArgs& a, cudaStream_t s) {
    DeviceState* ds = state();
    const bool forced = ds->gemm_bn == 64 || ds->gemm_bn == 128 || ds->gemm_bn == 192 || ds->gemm_bn == 256;
    if (!forced && ds->gemm_ctas == 0 && use_w12(a.M, a.w->N, a.epi, ds->num_sms))
        return a.w->mode == kOpsF16 ? dispatch_bn<kOpsF16>(a, s, 192, 1, false) : dispatch_bn<kOpsI8>(a, s, 192, 1, false);
    if (!forced && ds->gemm_ctas == 0 && small_tiles(a.M, a.w->N, ds->num_sms))
        return a.w->mode == kOpsF16 ? dispatch_bn<kOpsF16>(a, s, 64, 2, false) : dispatch_bn<kOpsI8>(a, s, 64, 2, false);
    const int bn = forced ? ds->gemm_bn : auto_bn(a.M, a.w->N, ds->num_sms);
    const int ctas = ds->gemm_ctas == 1 || ds->gemm_ctas == 2
                         ? ds->gemm_ctas
                         : (forced ? 1 : auto_ctas(a.M, a.w->N, a.epi, ds->num_sms));
    return a.w->mode == kOpsF16 ? dispatch_bn<kOpsF16>(a, s, bn, ctas, !forced)
                                : dispatch_bn<kOpsI8>(a, s, bn, ctas, !forced);
}

// Weight tensor maps are built once at registration (box = 128 bytes of K by
// BN rows, 128-byte swizzle; scales BN x blocks-per-stage), for every width.
bool make_weight_maps(b2q_weight* w) {
    const int es = ops_elem_bytes(w->mode);
    const uint32_t kbs = 128 / (32 * es);
    const CUtensorMapDataType dt = w->mode == kOpsF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
    return make_tmap_2d(&w->tm_q256, dt, w->q, w->K, w->N, w->K * es, 128 / es, 256, true) &&
           make_tmap_2d(&w->tm_q192, dt, w->q, w->K, w->N, w->K * es, 128 / es, 192, true) &&
           make_tmap_2d(&w->tm_q128, dt, w->q, w->K, w->N, w->K * es, 128 / es, 128, true) &&
           make_tmap_2d(&w->tm_q64, dt, w->q, w->K, w->N, w->K * es, 128 / es, 64, true) &&
           make_tmap_2d(&w->tm_d64, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w->d, w->Nd, w->Kb, w->Nd * 4, 64, kbs, false) &&
           make_tmap_2d(&w->tm_d256, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w->d, w->Nd, w->Kb, w->Nd * 4, 256, kbs, false) &&
           make_tmap_2d(&w->tm_d192, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w->d, w->Nd, w->Kb, w->Nd * 4, 192, kbs, false) &&
           make_tmap_2d(&w->tm_d128, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w->d, w->Nd, w->Kb, w->Nd * 4, 128, kbs, false);
}

}  // namespace b2q
