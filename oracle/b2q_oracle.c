/*
 * b2q_oracle.c — CPU restatement of the SigLIP2 Q8_0 x q8_1 hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see b2q_oracle.h): the checker for the CUDA path
 * and the timed CPU baseline ("port").  Built with -ffp-contract=off so that
 * every rounding step below is exactly the one written.
 */
#include "b2q_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#if defined(__x86_64__)
#include <immintrin.h>
#endif
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* threading                                                                 */
/* ------------------------------------------------------------------------ */
int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void) n;
#endif
}

/* ------------------------------------------------------------------------ */
/* Element-rule variants (orc_set_rules).  The default (0) is the canonical  */
/* order the CUDA kernels reproduce bit for bit.  The other bits switch the  */
/* towers to the reference's own element rules, so that the distance        */
/* between two faithful implementations of the same tower can be measured:  */
/*   ORC_RULE_LN    LayerNorm as fused_layernorm_affine_kernel<1024>         */
/*                  (src/cuda/siglip2_megakernel.cu:81-121): thread t of    */
/*                  1024 sums elements t, t+1024, ...; xor butterflies      */
/*                  16..1 inside each warp, then across the 32 warp sums;    */
/*                  var = fma(-mean, mean, ss/H); inv = correctly rounded    */
/*                  1/sqrt (the kernel's rsqrtf is approximate; its exact    */
/*                  rounding is not reproducible on the CPU, and this        */
/*                  stands in for it as another last-bit choice).            */
/*   ORC_RULE_GELU  0.5*x*(1+tanhf(sqrt(2/pi)*x*(1+0.044715*x*x))) with the  */
/*                  C library's tanhf (siglip2_megakernel.cu:276-280).       */
/*   ORC_RULE_Q8    q8_1 with x*(127/a) rounded half away from zero.         */
/*   ORC_RULE_GEMM  per-block accumulate acc += (dw*dx)*(float)S.            */
/* ------------------------------------------------------------------------ */
static int g_rules = 0;
void orc_set_rules(int rules) { g_rules = rules; }
int  orc_get_rules(void) { return g_rules; }

/* ------------------------------------------------------------------------ */
/* fp16 <-> fp32 (IEEE binary16, round-to-nearest-even)                      */
/* ggml block_q8_0::d is an fp16 (ggml-common.h block_q8_0; gguf quants.py:389) */
/* ------------------------------------------------------------------------ */
float orc_fp16_to_fp32(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float) v;
}

uint16_t orc_fp32_to_fp16(float f) {
    _Float16 v = (_Float16) f;
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}

/* ------------------------------------------------------------------------ */
/* exp / reciprocal / GELU                                                   */
/*                                                                           */
/* The reference's GELU (src/cuda/siglip2_megakernel.cu:276-280) is the      */
/* tanh form 0.5*x*(1+tanh(y)), y = sqrt(2/pi)*x*(1+0.044715*x^2), with the  */
/* platform tanhf.  CPU and GPU math libraries differ in the last bits, so   */
/* this library evaluates the same function its own way on both sides, with */
/* the same operations in the same order (every step an IEEE-exact +,*,fma): */
/* 0.5*(1+tanh(y)) = 1/(1+e^{-2y}), hence gelu(x) = x / (1 + e^{-2y}); one   */
/* exponential and one division, no cancellation for negative x.             */
/*   exp: Cody-Waite reduction x = n ln2 + r (ln2 split into a 16-bit head   */
/*        and its tail), degree-8 Taylor polynomial of e^r on |r| <= ln2/2,  */
/*        2^n through the exponent field.                                    */
/*   a/b: reciprocal seed from the integer bit pattern (the "magic constant" */
/*        method: 0x7EF311C7 - bits(b), relative error below 1/8), three     */
/*        Newton-Raphson steps y += y*(1 - b*y), then one Markstein          */
/*        correction q = q0 + y*(a - b*q0) of the quotient q0 = a*y.         */
/* Error vs. the float64 tanh form is tested in tests/test_oracle.py.        */
/* ------------------------------------------------------------------------ */
#define ORC_LOG2E   1.44269504088896340736f
#define ORC_LN2_HI  0.693145751953125f          /* 0x3F317200 */
#define ORC_LN2_LO  1.42860682030941723212e-6f  /* ln2 - LN2_HI */

float orc_expf(float x) {
    /* valid for |x| <= 80 (callers clamp) */
    float n = rintf(x * ORC_LOG2E);
    float r = fmaf(n, -ORC_LN2_HI, x);
    r = fmaf(n, -ORC_LN2_LO, r);
    float p = 2.48015873015873015873e-5f;            /* 1/8! */
    p = fmaf(p, r, 1.98412698412698412698e-4f);      /* 1/7! */
    p = fmaf(p, r, 1.38888888888888888889e-3f);      /* 1/6! */
    p = fmaf(p, r, 8.33333333333333333333e-3f);      /* 1/5! */
    p = fmaf(p, r, 4.16666666666666666667e-2f);      /* 1/4! */
    p = fmaf(p, r, 1.66666666666666666667e-1f);      /* 1/3! */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    /* scale by 2^n through the exponent field */
    int32_t ni = (int32_t) n;
    union { float f; int32_t i; } s;
    s.i = (ni + 127) << 23;
    return p * s.f;
}

float orc_div(float a, float b) {
    /* b normal and positive (callers: b = 1 + e^z >= 1) */
    union { float f; int32_t i; } u;
    u.f = b;
    u.i = 0x7EF311C7 - u.i;
    float y = u.f;
    for (int it = 0; it < 3; ++it) {
        float e = fmaf(-b, y, 1.0f);
        y = fmaf(y, e, y);
    }
    float q0 = a * y;
    float r = fmaf(-b, q0, a);
    return fmaf(r, y, q0);
}

float orc_gelu(float x) {
    const float GELU_COEF_A = 0.044715f;
    const float M2_SQRT_2_OVER_PI = -1.59576912160573071175978423973752f;   /* -2*sqrt(2/pi) */
    float x2 = x * x;
    float inner = fmaf(GELU_COEF_A, x2, 1.0f);
    float z = (M2_SQRT_2_OVER_PI * x) * inner;     /* -2y */
    z = fminf(fmaxf(z, -80.0f), 80.0f);
    float d = 1.0f + orc_expf(z);
    return orc_div(x, d);
}

void orc_gelu_n(const float *x, int64_t n, float *y) {
    for (int64_t i = 0; i < n; ++i) y[i] = orc_gelu(x[i]);
}

/* The reference's own GELU expression with the C library's tanhf
 * (ORC_RULE_GELU). */
static float gelu_tanh_ref(float x) {
    const float a = 0.044715f * x;
    const float inner = fmaf(a, x, 1.0f);
    const float y = (0.79788456080286535587989211986876f * x) * inner;
    return (0.5f * x) * (1.0f + tanhf(y));
}

static inline float tower_gelu(float x) { return (g_rules & ORC_RULE_GELU) ? gelu_tanh_ref(x) : orc_gelu(x); }

/* ------------------------------------------------------------------------ */
/* Q8_0 weight codec — gguf-py quants.py:381-401 (bit-exact with            */
/* ggml-quants.c quantize_row_q8_0_ref): d = max|x|/127 in fp32,             */
/* id = d ? 1/d : 0, q = roundf(x*id) (half away from zero), d stored fp16.  */
/* ------------------------------------------------------------------------ */
void orc_quantize_q8_0(const float *x, int64_t N, int64_t K, int64_t Kp, uint8_t *out) {
    const int64_t Kb = Kp / 32;
    #pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t kb = 0; kb < Kb; ++kb) {
            float v[32];
            for (int j = 0; j < 32; ++j) {
                int64_t k = kb * 32 + j;
                v[j] = (k < K) ? x[n * K + k] : 0.0f;
            }
            float amax = 0.0f;
            for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
            float d  = amax / 127.0f;
            float id = (d != 0.0f) ? 1.0f / d : 0.0f;
            uint8_t *blk = out + (n * Kb + kb) * 34;
            uint16_t dh = orc_fp32_to_fp16(d);
            memcpy(blk, &dh, 2);
            for (int j = 0; j < 32; ++j) {
                float q = roundf(v[j] * id);
                blk[2 + j] = (uint8_t) (int8_t) q;
            }
        }
    }
}

void orc_dequantize_q8_0(const uint8_t *w, int64_t N, int64_t Kp, float *out) {
    const int64_t Kb = Kp / 32;
    #pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t kb = 0; kb < Kb; ++kb) {
            const uint8_t *blk = w + (n * Kb + kb) * 34;
            uint16_t dh;
            memcpy(&dh, blk, 2);
            float d = orc_fp16_to_fp32(dh);
            for (int j = 0; j < 32; ++j)
                out[n * Kp + kb * 32 + j] = (float) (int8_t) blk[2 + j] * d;
        }
    }
}

/* ------------------------------------------------------------------------ */
/* q8_1 activation quantize — src/cuda/siglip2_custom_mmq.cu:51-82:          */
/* a = max|x| over the 32-block, d = a/127, q = rint(x * 127/a) (round half  */
/* to even, __float2int_rn) clamped to [-128,127]; a == 0 gives q = 0.       */
/* Columns K..Kp-1 are zero (pad_x_to_w, siglip2_vision.cpp:99-107).         */
/* ------------------------------------------------------------------------ */
static inline void q8_1_block(const float *v, int8_t *q, float *d) {
    float a = 0.0f;
    for (int j = 0; j < 32; ++j) a = fmaxf(a, fabsf(v[j]));
    float inv = (a == 0.0f) ? 0.0f : 127.0f / a;
    *d = a / 127.0f;
    for (int j = 0; j < 32; ++j) {
        float r = rintf(v[j] * inv);
        if (r > 127.0f) r = 127.0f;
        if (r < -128.0f) r = -128.0f;
        q[j] = (int8_t) r;
    }
}

/* Alternative activation rules (ggml-CUDA's own q8_1 source is absent here,
 * so the conventions it might use are kept selectable for a later check
 * against it): 0 = the rule above (x * (127/a), half to even; what the GPU
 * kernels do), 1 = x * (127/a) rounded half away from zero, 2 = x / d
 * (d = a/127) half to even, 3 = x * (1/d) half away from zero (the ggml CPU
 * Q8_0 convention applied to activations). */
static inline int8_t q8_1_round(float v, float a, float d, int rule) {
    float r;
    if (a == 0.0f) return 0;
    switch (rule) {
        case 1:  r = roundf(v * (127.0f / a)); break;
        case 2:  r = rintf(v / d); break;
        case 3:  r = roundf(v * (1.0f / d)); break;
        default: r = rintf(v * (127.0f / a)); break;
    }
    if (r > 127.0f) r = 127.0f;
    if (r < -128.0f) r = -128.0f;
    return (int8_t) r;
}

void orc_quantize_q8_1_rule(const float *x, int64_t M, int64_t K, int64_t ldx, int64_t Kp,
                            int8_t *qs, float *d, int rule) {
    const int64_t Kb = Kp / 32;
    for (int64_t m = 0; m < M; ++m)
        for (int64_t kb = 0; kb < Kb; ++kb) {
            float v[32], a = 0.0f;
            for (int j = 0; j < 32; ++j) {
                int64_t k = kb * 32 + j;
                v[j] = (k < K) ? x[m * ldx + k] : 0.0f;
                a = fmaxf(a, fabsf(v[j]));
            }
            const float dd = a / 127.0f;
            d[m * Kb + kb] = dd;
            for (int j = 0; j < 32; ++j) qs[m * Kp + kb * 32 + j] = q8_1_round(v[j], a, dd, rule);
        }
}

void orc_quantize_q8_1(const float *x, int64_t M, int64_t K, int64_t ldx, int64_t Kp,
                       int8_t *qs, float *d) {
    const int64_t Kb = Kp / 32;
    #pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t kb = 0; kb < Kb; ++kb) {
            float v[32];
            for (int j = 0; j < 32; ++j) {
                int64_t k = kb * 32 + j;
                v[j] = (k < K) ? x[m * ldx + k] : 0.0f;
            }
            q8_1_block(v, qs + m * Kp + kb * 32, d + m * Kb + kb);
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Block GEMM — ggml_mul_mat(W Q8_0, X) semantics as restated by            */
/* src/cuda/siglip2_custom_mmq.cu:229-266: per K-block int32 dot, then       */
/* Cf += (float)Cint * dw * dx, evaluated as fma((float)S*dw, dx, acc).      */
/* ------------------------------------------------------------------------ */
__attribute__((target_clones("arch=x86-64-v4", "arch=x86-64-v3", "default")))
static int32_t dot32_i8(const int8_t *a, const int8_t *b) {
    int32_t s = 0;
    for (int j = 0; j < 32; ++j) s += (int32_t) a[j] * (int32_t) b[j];
    return s;
}

#if defined(__x86_64__)
/* AVX512-VNNI form of the same GEMM, bit-identical to the scalar loop below:
 * vpdpbusd multiplies unsigned by signed bytes, so the activation bytes are
 * biased by +128 and the exact int32 correction 128*sum_j(w) is subtracted;
 * then, per block, vcvtdq2ps (exact: |S| < 2^20), vmulps by the weight
 * scales and vfmadd231ps with the activation scale, kb ascending: the same
 * fp32 operations as (float)S*dw then fmaf(t, dx, acc).  Weights are packed
 * per 16 output columns as [kb][j/4][16 columns][4 bytes], so one 64-byte
 * load feeds 16 columns and the bias-corrected activation dword is
 * broadcast; four rows share each weight load. */
#define ORC_VNNI_TARGET __attribute__((target("avx512f,avx512bw,avx512vnni")))

typedef struct {
    int64_t N, Kb, NT;          /* NT = 16-column tiles */
    int8_t *w;                  /* [NT][Kb][8][16][4] */
    int32_t *wsum;              /* [NT][Kb][16] 128 * sum_j w */
    float *wd;                  /* [NT][Kb][16] */
} vnni_pack;

static void vnni_pack_weights(const uint8_t *w, int64_t N, int64_t Kp, vnni_pack *P) {
    const int64_t Kb = Kp / 32, NT = (N + 15) / 16;
    P->N = N; P->Kb = Kb; P->NT = NT;
    P->w = (int8_t *) calloc((size_t) (NT * Kb * 512), 1);
    P->wsum = (int32_t *) calloc((size_t) (NT * Kb * 16), sizeof(int32_t));
    P->wd = (float *) calloc((size_t) (NT * Kb * 16), sizeof(float));
    #pragma omp parallel for schedule(static)
    for (int64_t nt = 0; nt < NT; ++nt)
        for (int64_t kb = 0; kb < Kb; ++kb)
            for (int c = 0; c < 16; ++c) {
                const int64_t n = nt * 16 + c;
                if (n >= N) continue;
                const uint8_t *blk = w + (n * Kb + kb) * 34;
                uint16_t dh;
                memcpy(&dh, blk, 2);
                P->wd[(nt * Kb + kb) * 16 + c] = orc_fp16_to_fp32(dh);
                int32_t sum = 0;
                for (int j = 0; j < 32; ++j) {
                    const int8_t v = (int8_t) blk[2 + j];
                    P->w[(nt * Kb + kb) * 512 + (j / 4) * 64 + c * 4 + (j % 4)] = v;
                    sum += v;
                }
                P->wsum[(nt * Kb + kb) * 16 + c] = 128 * sum;
            }
}

ORC_VNNI_TARGET
static void vnni_rows(const vnni_pack *P, const uint8_t *xu, const float *dx, int64_t Kp, int64_t m0, int R,
                      int64_t nt, float *y, int64_t N) {
    const int64_t Kb = P->Kb;
    __m512 acc[4];
    for (int r = 0; r < 4; ++r) acc[r] = _mm512_setzero_ps();
    for (int64_t kb = 0; kb < Kb; ++kb) {
        const int8_t *wb = P->w + (nt * Kb + kb) * 512;
        __m512i S[4];
        for (int r = 0; r < 4; ++r) S[r] = _mm512_setzero_si512();
        for (int g = 0; g < 8; ++g) {
            const __m512i wv = _mm512_loadu_si512((const void *) (wb + g * 64));
            for (int r = 0; r < R; ++r) {
                int32_t xd4;
                memcpy(&xd4, xu + (m0 + r) * Kp + kb * 32 + g * 4, 4);
                S[r] = _mm512_dpbusd_epi32(S[r], _mm512_set1_epi32(xd4), wv);
            }
        }
        const __m512i corr = _mm512_loadu_si512((const void *) (P->wsum + (nt * Kb + kb) * 16));
        const __m512 wd = _mm512_loadu_ps(P->wd + (nt * Kb + kb) * 16);
        for (int r = 0; r < R; ++r) {
            const __m512 t = _mm512_mul_ps(_mm512_cvtepi32_ps(_mm512_sub_epi32(S[r], corr)), wd);
            acc[r] = _mm512_fmadd_ps(t, _mm512_set1_ps(dx[(m0 + r) * Kb + kb]), acc[r]);
        }
    }
    const int64_t n0 = nt * 16;
    const __mmask16 mask = (N - n0 >= 16) ? (__mmask16) 0xFFFF : (__mmask16) ((1u << (N - n0)) - 1u);
    for (int r = 0; r < R; ++r) _mm512_mask_storeu_ps(y + (m0 + r) * N + n0, mask, acc[r]);
}

static int vnni_available(void) {
    static int cached = -1;
    if (cached < 0) {
        __builtin_cpu_init();
        cached = __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
                 __builtin_cpu_supports("avx512vnni");
        if (getenv("ORC_NO_VNNI")) cached = 0;
    }
    return cached;
}

static void gemm_q8_vnni(const uint8_t *w, int64_t N, int64_t Kp, const int8_t *qs, const float *dx, int64_t M,
                         float *y) {
    vnni_pack P;
    vnni_pack_weights(w, N, Kp, &P);
    uint8_t *xu = (uint8_t *) malloc((size_t) M * (size_t) Kp);
    #pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < M * Kp; ++i) xu[i] = (uint8_t) ((int32_t) qs[i] + 128);
    const int64_t MT = (M + 3) / 4;
    #pragma omp parallel for schedule(dynamic, 1) collapse(2)
    for (int64_t mt = 0; mt < MT; ++mt)
        for (int64_t nt = 0; nt < P.NT; ++nt) {
            const int64_t m0 = mt * 4;
            const int R = (int) ((M - m0) < 4 ? (M - m0) : 4);
            vnni_rows(&P, xu, dx, Kp, m0, R, nt, y, N);
        }
    free(xu);
    free(P.w);
    free(P.wsum);
    free(P.wd);
}
#endif

int orc_gemm_uses_vnni(void) {
#if defined(__x86_64__)
    return vnni_available();
#else
    return 0;
#endif
}

void orc_gemm_q8(const uint8_t *w, int64_t N, int64_t Kp,
                 const int8_t *qs, const float *dx, int64_t M,
                 float *y, int32_t *block_sums) {
#if defined(__x86_64__)
    if (!block_sums && vnni_available() && (g_rules & ORC_RULE_GEMM) == 0) {
        gemm_q8_vnni(w, N, Kp, qs, dx, M, y);
        return;
    }
#endif
    const int64_t Kb = Kp / 32;
    /* unpack weights once: int8 plane + fp32 scales (exact fp16 widening) */
    int8_t *wq = (int8_t *) malloc((size_t) N * (size_t) Kp);
    float  *wd = (float *) malloc((size_t) N * (size_t) Kb * sizeof(float));
    #pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t kb = 0; kb < Kb; ++kb) {
            const uint8_t *blk = w + (n * Kb + kb) * 34;
            uint16_t dh;
            memcpy(&dh, blk, 2);
            wd[n * Kb + kb] = orc_fp16_to_fp32(dh);
            memcpy(wq + n * Kp + kb * 32, blk + 2, 32);
        }
    }
    const int gemm_alt = (g_rules & ORC_RULE_GEMM) != 0;
    #pragma omp parallel for schedule(dynamic, 4)
    for (int64_t m = 0; m < M; ++m) {
        const int8_t *xr = qs + m * Kp;
        const float  *xd = dx + m * Kb;
        for (int64_t n = 0; n < N; ++n) {
            const int8_t *wr = wq + n * Kp;
            const float  *wdr = wd + n * Kb;
            float acc = 0.0f;
            for (int64_t kb = 0; kb < Kb; ++kb) {
                int32_t S = dot32_i8(xr + kb * 32, wr + kb * 32);
                if (block_sums) block_sums[(m * N + n) * Kb + kb] = S;
                if (gemm_alt) {
                    acc = fmaf(wdr[kb] * xd[kb], (float) S, acc);
                } else {
                    float t = (float) S * wdr[kb];
                    acc = fmaf(t, xd[kb], acc);
                }
            }
            y[m * N + n] = acc;
        }
    }
    free(wq);
    free(wd);
}

/* ------------------------------------------------------------------------ */
/* LayerNorm + affine — src/cuda/siglip2_megakernel.cu:81-121.               */
/* One-pass sums.  Summation order (shared with the CUDA row kernel): lane   */
/* l in 0..31 accumulates elements (c*32 + l)*4 + j for c ascending, j in    */
/* 0..3, s += v and ss = fma(v, v, ss); the 32 lane partials are combined by */
/* an xor butterfly with offsets 16, 8, 4, 2, 1.  H must be a multiple of    */
/* 128.  mean = s/H, var = ss/H - mean*mean, inv = 1/sqrt(var + eps).        */
/* y = ((x - mean) * inv) * w + b with separately rounded steps.             */
/* ------------------------------------------------------------------------ */
static void row_moments(const float *x, int64_t H, float *mean_out, float *inv_unused, float *s_out, float *ss_out) {
    (void) inv_unused;
    float ps[32], pss[32];
    const int64_t chunks = H / 128;
    for (int l = 0; l < 32; ++l) {
        float s = 0.0f, ss = 0.0f;
        for (int64_t c = 0; c < chunks; ++c) {
            for (int j = 0; j < 4; ++j) {
                float v = x[(c * 32 + l) * 4 + j];
                s  = s + v;
                ss = fmaf(v, v, ss);
            }
        }
        ps[l] = s;
        pss[l] = ss;
    }
    for (int off = 16; off >= 1; off >>= 1) {
        float ns[32], nss[32];
        for (int l = 0; l < 32; ++l) {
            ns[l]  = ps[l] + ps[l ^ off];
            nss[l] = pss[l] + pss[l ^ off];
        }
        memcpy(ps, ns, sizeof ps);
        memcpy(pss, nss, sizeof pss);
    }
    *s_out = ps[0];
    *ss_out = pss[0];
    *mean_out = ps[0] / (float) H;
}

/* LayerNorm in the reference kernel's own order (ORC_RULE_LN, see above). */
static void layernorm_ref_order(const float *xr, const float *w, const float *b, float eps, int64_t H, float *yr) {
    float s[1024], ss[1024];
    for (int t = 0; t < 1024; ++t) {
        float a = 0.0f, q = 0.0f;
        for (int64_t i = t; i < H; i += 1024) {
            const float v = xr[i];
            a = a + v;
            q = fmaf(v, v, q);
        }
        s[t] = a;
        ss[t] = q;
    }
    float ws[32], wss[32];
    for (int wp = 0; wp < 32; ++wp) {
        float ps[32], pss[32];
        memcpy(ps, s + 32 * wp, sizeof ps);
        memcpy(pss, ss + 32 * wp, sizeof pss);
        for (int off = 16; off >= 1; off >>= 1) {
            float ns[32], nss[32];
            for (int l = 0; l < 32; ++l) { ns[l] = ps[l] + ps[l ^ off]; nss[l] = pss[l] + pss[l ^ off]; }
            memcpy(ps, ns, sizeof ps);
            memcpy(pss, nss, sizeof pss);
        }
        ws[wp] = ps[0];
        wss[wp] = pss[0];
    }
    for (int off = 16; off >= 1; off >>= 1) {
        float ns[32], nss[32];
        for (int l = 0; l < 32; ++l) { ns[l] = ws[l] + ws[l ^ off]; nss[l] = wss[l] + wss[l ^ off]; }
        memcpy(ws, ns, sizeof ws);
        memcpy(wss, nss, sizeof wss);
    }
    const float mean = ws[0] / (float) H;
    const float var = fmaf(-mean, mean, wss[0] / (float) H);
    const float inv = (float) (1.0 / sqrt((double) (var + eps)));
    for (int64_t i = 0; i < H; ++i) {
        const float t = (xr[i] - mean) * inv;
        yr[i] = t * w[i] + b[i];
    }
}

void orc_layernorm(const float *x, const float *w, const float *b, float eps,
                   int64_t M, int64_t H, float *y) {
    if (g_rules & ORC_RULE_LN) {
        #pragma omp parallel for schedule(static)
        for (int64_t m = 0; m < M; ++m) layernorm_ref_order(x + m * H, w, b, eps, H, y + m * H);
        return;
    }
    #pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m) {
        const float *xr = x + m * H;
        float mean, s, ss;
        row_moments(xr, H, &mean, NULL, &s, &ss);
        float msq = ss / (float) H;
        float var = msq - mean * mean;
        float inv = 1.0f / sqrtf(var + eps);
        for (int64_t i = 0; i < H; ++i) {
            float t = (xr[i] - mean) * inv;
            y[m * H + i] = t * w[i] + b[i];
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Attention — flash_attn_ext with K/V cast to fp16 and F32 precision        */
/* (siglip2_vision.cpp:154-175), kq_scale = 1/sqrt(d_head) (:629-632).       */
/* ------------------------------------------------------------------------ */
/* Attention of the quantized (Q8) towers: one fixed fp32 evaluation order,
 * reproduced operation by operation by the GPU's exact attention mode.  Q, K
 * and V arrive as fp16 values (the QKV projection's output rounded to fp16;
 * K and V are cast to fp16 by the reference graph, siglip2_vision.cpp:
 * 164-165); with GGML_PREC_F32 (siglip2_vision.cpp:167) scores, softmax and
 * the weighted sum are fp32:
 *   s_k = fma-chain over d ascending of q_d*k_kd, times 1/sqrt(d_head)
 *   m = max_k s_k ; p_k = exp(s_k - m) (the library's own exp) ;
 *   l = sum_k p_k (keys ascending) ; o_d = fma-chain over k of p_k*v_kd, / l
 * q/k/v point at head 0 of row 0 with row strides ldq/ldk/ldv; Lq query rows
 * attend to Lk keys; out rows stride ldo. */
#if defined(__x86_64__)
/* orc_expf on 16 lanes: the same operations in the same order (rint by
 * vrndscaleps to nearest, the two-term reduction, the degree-8 polynomial,
 * 2^n through the exponent field), so every lane equals orc_expf. */
ORC_VNNI_TARGET
static inline __m512 orc_expf_x16(__m512 x) {
    const __m512 n = _mm512_roundscale_ps(_mm512_mul_ps(x, _mm512_set1_ps(ORC_LOG2E)),
                                          _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
    __m512 r = _mm512_fmadd_ps(n, _mm512_set1_ps(-ORC_LN2_HI), x);
    r = _mm512_fmadd_ps(n, _mm512_set1_ps(-ORC_LN2_LO), r);
    __m512 p = _mm512_set1_ps(2.48015873015873015873e-5f);
    p = _mm512_fmadd_ps(p, r, _mm512_set1_ps(1.98412698412698412698e-4f));
    p = _mm512_fmadd_ps(p, r, _mm512_set1_ps(1.38888888888888888889e-3f));
    p = _mm512_fmadd_ps(p, r, _mm512_set1_ps(8.33333333333333333333e-3f));
    p = _mm512_fmadd_ps(p, r, _mm512_set1_ps(4.16666666666666666667e-2f));
    p = _mm512_fmadd_ps(p, r, _mm512_set1_ps(1.66666666666666666667e-1f));
    p = _mm512_fmadd_ps(p, r, _mm512_set1_ps(0.5f));
    p = _mm512_fmadd_ps(p, r, _mm512_set1_ps(1.0f));
    p = _mm512_fmadd_ps(p, r, _mm512_set1_ps(1.0f));
    const __m512i ni = _mm512_cvtps_epi32(n);
    const __m512 sc = _mm512_castsi512_ps(_mm512_slli_epi32(_mm512_add_epi32(ni, _mm512_set1_epi32(127)), 23));
    return _mm512_mul_ps(p, sc);
}

/* attention_q8 on 16 lanes, bit-identical to the scalar loop: scores with one
 * key per lane (each lane's fma chain over d ascending, keys transposed to
 * [d][key] per head), the row maximum and the key-ascending sum of p as in
 * the scalar code, and the output with one dimension per lane (fma chain
 * over keys ascending), divided by the sum. */
ORC_VNNI_TARGET
static void attention_q8_avx512(const float *q, int64_t ldq, const float *k, int64_t ldk, const float *v,
                                int64_t ldv, int64_t Lq, int64_t Lk, int64_t n_head, int64_t dh, float *out,
                                int64_t ldo) {
    const float scale = 1.0f / sqrtf((float) dh);
    const int64_t Lk16 = (Lk + 15) / 16 * 16;
    const int64_t nd = (dh + 15) / 16;
    for (int64_t hd = 0; hd < n_head; ++hd) {
        float *kt = (float *) aligned_alloc(64, (size_t) (dh * Lk16) * sizeof(float));
        float *vh = (float *) aligned_alloc(64, (size_t) (Lk * nd * 16) * sizeof(float));
        for (int64_t d = 0; d < dh; ++d)
            for (int64_t kk = 0; kk < Lk16; ++kk) kt[d * Lk16 + kk] = kk < Lk ? k[kk * ldk + hd * dh + d] : 0.0f;
        for (int64_t kk = 0; kk < Lk; ++kk)
            for (int64_t d = 0; d < nd * 16; ++d) vh[kk * nd * 16 + d] = d < dh ? v[kk * ldv + hd * dh + d] : 0.0f;
        #pragma omp parallel for schedule(static)
        for (int64_t qi = 0; qi < Lq; ++qi) {
            const float *qr = q + qi * ldq + hd * dh;
            float *sc = (float *) aligned_alloc(64, (size_t) Lk16 * sizeof(float));
            for (int64_t k0 = 0; k0 < Lk16; k0 += 16) {
                __m512 dot = _mm512_setzero_ps();
                for (int64_t d = 0; d < dh; ++d)
                    dot = _mm512_fmadd_ps(_mm512_set1_ps(qr[d]), _mm512_load_ps(kt + d * Lk16 + k0), dot);
                _mm512_store_ps(sc + k0, _mm512_mul_ps(dot, _mm512_set1_ps(scale)));
            }
            float m = -INFINITY;
            for (int64_t kk = 0; kk < Lk; ++kk) m = fmaxf(m, sc[kk]);
            for (int64_t k0 = 0; k0 < Lk16; k0 += 16)
                _mm512_store_ps(sc + k0, orc_expf_x16(_mm512_sub_ps(_mm512_load_ps(sc + k0), _mm512_set1_ps(m))));
            float l = 0.0f;
            for (int64_t kk = 0; kk < Lk; ++kk) l = l + sc[kk];
            for (int64_t b = 0; b < nd; ++b) {
                __m512 acc = _mm512_setzero_ps();
                for (int64_t kk = 0; kk < Lk; ++kk)
                    acc = _mm512_fmadd_ps(_mm512_set1_ps(sc[kk]), _mm512_loadu_ps(vh + kk * nd * 16 + b * 16), acc);
                const __m512 o = _mm512_div_ps(acc, _mm512_set1_ps(l));
                const int64_t rem = dh - b * 16;
                const __mmask16 mk = rem >= 16 ? (__mmask16) 0xFFFF : (__mmask16) ((1u << rem) - 1u);
                _mm512_mask_storeu_ps(out + qi * ldo + hd * dh + b * 16, mk, o);
            }
            free(sc);
        }
        free(kt);
        free(vh);
    }
}
#endif

static void attention_q8(const float *q, int64_t ldq, const float *k, int64_t ldk, const float *v, int64_t ldv,
                         int64_t Lq, int64_t Lk, int64_t n_head, int64_t dh, float *out, int64_t ldo) {
#if defined(__x86_64__)
    if (vnni_available() && Lq > 1) {
        attention_q8_avx512(q, ldq, k, ldk, v, ldv, Lq, Lk, n_head, dh, out, ldo);
        return;
    }
#endif
    const float scale = 1.0f / sqrtf((float) dh);
    #pragma omp parallel for schedule(static) collapse(2)
    for (int64_t hd = 0; hd < n_head; ++hd) {
        for (int64_t qi = 0; qi < Lq; ++qi) {
            const float *qr = q + qi * ldq + hd * dh;
            float *s = (float *) malloc((size_t) Lk * sizeof(float));
            float m = -INFINITY;
            for (int64_t kk = 0; kk < Lk; ++kk) {
                const float *kr = k + kk * ldk + hd * dh;
                float dot = 0.0f;
                for (int64_t d = 0; d < dh; ++d) dot = fmaf(qr[d], kr[d], dot);
                s[kk] = dot * scale;
                m = fmaxf(m, s[kk]);
            }
            float l = 0.0f;
            for (int64_t kk = 0; kk < Lk; ++kk) {
                s[kk] = orc_expf(s[kk] - m);
                l = l + s[kk];
            }
            for (int64_t d = 0; d < dh; ++d) {
                float acc = 0.0f;
                for (int64_t kk = 0; kk < Lk; ++kk) acc = fmaf(s[kk], v[kk * ldv + hd * dh + d], acc);
                out[qi * ldo + hd * dh + d] = acc / l;
            }
            free(s);
        }
    }
}

static inline float half_of(float v) { return orc_fp16_to_fp32(orc_fp32_to_fp16(v)); }

void orc_attention(const float *qkv, int64_t T, int64_t H, int64_t n_head,
                   const int64_t *seq_off, const int64_t *seq_len, int64_t n_seq,
                   float *out) {
    (void) T;
    const int64_t dh = H / n_head;
    const float scale = 1.0f / sqrtf((float) dh);
    const int64_t ld = 3 * H;
    for (int64_t s = 0; s < n_seq; ++s) {
        const int64_t off = seq_off[s], L = seq_len[s];
        float *kh = (float *) malloc((size_t) L * (size_t) H * sizeof(float));
        float *vh = (float *) malloc((size_t) L * (size_t) H * sizeof(float));
        for (int64_t t = 0; t < L; ++t)
            for (int64_t i = 0; i < H; ++i) {
                kh[t * H + i] = orc_fp16_to_fp32(orc_fp32_to_fp16(qkv[(off + t) * ld + H + i]));
                vh[t * H + i] = orc_fp16_to_fp32(orc_fp32_to_fp16(qkv[(off + t) * ld + 2 * H + i]));
            }
        #pragma omp parallel for schedule(static) collapse(2)
        for (int64_t hd = 0; hd < n_head; ++hd) {
            for (int64_t q = 0; q < L; ++q) {
                const float *qr = qkv + (off + q) * ld + hd * dh;
                double *sc = (double *) malloc((size_t) L * sizeof(double));
                double mx = -INFINITY;
                for (int64_t k = 0; k < L; ++k) {
                    const float *kr = kh + k * H + hd * dh;
                    double dot = 0.0;
                    for (int64_t i = 0; i < dh; ++i) dot += (double) qr[i] * (double) kr[i];
                    sc[k] = dot * (double) scale;
                    if (sc[k] > mx) mx = sc[k];
                }
                double den = 0.0;
                for (int64_t k = 0; k < L; ++k) { sc[k] = exp(sc[k] - mx); den += sc[k]; }
                for (int64_t i = 0; i < dh; ++i) {
                    double acc = 0.0;
                    for (int64_t k = 0; k < L; ++k) acc += sc[k] * (double) vh[k * H + hd * dh + i];
                    out[(off + q) * H + hd * dh + i] = (float) (acc / den);
                }
                free(sc);
            }
        }
        free(kh);
        free(vh);
    }
}

/* ------------------------------------------------------------------------ */
/* Position-embedding resize: bilinear with antialias, align_corners=False  */
/* (ggml_interpolate BILINEAR|ANTIALIAS at siglip2_vision.cpp:680-691, the   */
/* counterpart of HF's F.interpolate(..., antialias=True)).  Separable       */
/* triangle filter of support max(1, in/out), weights normalised per output. */
/* Width pass first, then height.                                            */
/* ------------------------------------------------------------------------ */
static void aa_weights(int64_t in, int64_t out, int64_t i, int64_t *lo, int64_t *cnt, double *wt) {
    double scale = (double) in / (double) out;
    double support = scale >= 1.0 ? scale : 1.0;
    double center = scale * ((double) i + 0.5);
    double invs = scale >= 1.0 ? 1.0 / scale : 1.0;
    int64_t xmin = (int64_t) (center - support + 0.5);
    if (xmin < 0) xmin = 0;
    int64_t xmax = (int64_t) (center + support + 0.5);
    if (xmax > in) xmax = in;
    double tot = 0.0;
    int64_t n = xmax - xmin;
    for (int64_t j = 0; j < n; ++j) {
        double a = ((double) (j + xmin) - center + 0.5) * invs;
        double w = 1.0 - fabs(a);
        if (w < 0.0) w = 0.0;
        wt[j] = w;
        tot += w;
    }
    for (int64_t j = 0; j < n; ++j) wt[j] = tot != 0.0 ? wt[j] / tot : 0.0;
    *lo = xmin;
    *cnt = n;
}

void orc_pos_resize(const float *table, int64_t side, int64_t H,
                    int64_t h, int64_t w, float *out) {
    /* tmp: [side][w][H] */
    float *tmp = (float *) malloc((size_t) side * (size_t) w * (size_t) H * sizeof(float));
    double wt[256];
    for (int64_t c = 0; c < w; ++c) {
        int64_t lo, n;
        aa_weights(side, w, c, &lo, &n, wt);
        for (int64_t r = 0; r < side; ++r)
            for (int64_t i = 0; i < H; ++i) {
                double acc = 0.0;
                for (int64_t j = 0; j < n; ++j) acc += wt[j] * (double) table[(r * side + lo + j) * H + i];
                tmp[(r * w + c) * H + i] = (float) acc;
            }
    }
    for (int64_t r = 0; r < h; ++r) {
        int64_t lo, n;
        aa_weights(side, h, r, &lo, &n, wt);
        for (int64_t c = 0; c < w; ++c)
            for (int64_t i = 0; i < H; ++i) {
                double acc = 0.0;
                for (int64_t j = 0; j < n; ++j) acc += wt[j] * (double) tmp[((lo + j) * w + c) * H + i];
                out[(r * w + c) * H + i] = (float) acc;
            }
    }
    free(tmp);
}

/* ------------------------------------------------------------------------ */
/* Towers                                                                    */
/* ------------------------------------------------------------------------ */

/* y[M][N] = X[M][K] @ W^T (+ epilogue) with the q8_1 activation rule, or in  */
/* fp32 against dequantized weights when quant_act == 0.                     */
static void proj(const uint8_t *w, int64_t N, int64_t K, int64_t Kp, const float *x, int64_t M,
                 int quant_act, float *y) {
    if (quant_act) {
        int8_t *qs = (int8_t *) malloc((size_t) M * (size_t) Kp);
        float  *dx = (float *) malloc((size_t) M * (size_t) (Kp / 32) * sizeof(float));
        if (g_rules & ORC_RULE_Q8)
            orc_quantize_q8_1_rule(x, M, K, K, Kp, qs, dx, 1);
        else
            orc_quantize_q8_1(x, M, K, K, Kp, qs, dx);
        orc_gemm_q8(w, N, Kp, qs, dx, M, y, NULL);
        free(qs);
        free(dx);
    } else {
        float *wf = (float *) malloc((size_t) N * (size_t) Kp * sizeof(float));
        orc_dequantize_q8_0(w, N, Kp, wf);
        #pragma omp parallel for schedule(static)
        for (int64_t m = 0; m < M; ++m)
            for (int64_t n = 0; n < N; ++n) {
                double acc = 0.0;
                for (int64_t k = 0; k < K; ++k) acc += (double) x[m * K + k] * (double) wf[n * Kp + k];
                y[m * N + n] = (float) acc;
            }
        free(wf);
    }
}

static void add_bias(float *y, const float *b, int64_t M, int64_t N) {
    #pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n) y[m * N + n] = y[m * N + n] + b[n];
}

/* one pre-LN encoder block (siglip2_vision.cpp:181-244; siglip2_text.cpp:216-302) */
static void encoder_block(const orc_block *B, float *x, int64_t T, int64_t H, int64_t F, int64_t Fp,
                          int64_t n_head, float eps, const int64_t *seq_off, const int64_t *seq_len,
                          int64_t n_seq, int quant_act) {
    float *ln  = (float *) malloc((size_t) T * H * sizeof(float));
    float *qkv = (float *) malloc((size_t) T * 3 * H * sizeof(float));
    float *att = (float *) malloc((size_t) T * H * sizeof(float));
    float *o   = (float *) malloc((size_t) T * H * sizeof(float));
    float *up  = (float *) malloc((size_t) T * F * sizeof(float));

    orc_layernorm(x, B->ln1_w, B->ln1_b, eps, T, H, ln);
    proj(B->qkv_w, 3 * H, H, H, ln, T, quant_act, qkv);
    add_bias(qkv, B->qkv_b, T, 3 * H);
    if (quant_act) {
        #pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < T * 3 * H; ++i) qkv[i] = half_of(qkv[i]);
        for (int64_t sidx = 0; sidx < n_seq; ++sidx) {
            const float *base = qkv + seq_off[sidx] * 3 * H;
            attention_q8(base, 3 * H, base + H, 3 * H, base + 2 * H, 3 * H, seq_len[sidx], seq_len[sidx], n_head,
                         H / n_head, att + seq_off[sidx] * H, H);
        }
    } else {
        orc_attention(qkv, T, H, n_head, seq_off, seq_len, n_seq, att);
    }
    proj(B->o_w, H, H, H, att, T, quant_act, o);
    #pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t)
        for (int64_t i = 0; i < H; ++i)
            x[t * H + i] = (o[t * H + i] + B->o_b[i]) + x[t * H + i];

    orc_layernorm(x, B->ln2_w, B->ln2_b, eps, T, H, ln);
    proj(B->up_w, F, H, H, ln, T, quant_act, up);
    #pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t)
        for (int64_t i = 0; i < F; ++i)
            up[t * F + i] = tower_gelu(up[t * F + i] + B->up_b[i]);
    proj(B->down_w, H, F, Fp, up, T, quant_act, o);
    #pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t)
        for (int64_t i = 0; i < H; ++i)
            x[t * H + i] = (o[t * H + i] + B->down_b[i]) + x[t * H + i];

    free(ln); free(qkv); free(att); free(o); free(up);
}

int orc_vision_encode(const orc_vision_weights *W, const float *patches,
                      int64_t h, int64_t w, int pooling, int quant_act, float *out) {
    const int64_t H = W->H, T = h * w;

    float *x   = (float *) malloc((size_t) T * H * sizeof(float));
    float *pos = (float *) malloc((size_t) T * H * sizeof(float));

    /* patch embed + bias, then + resized position table (siglip2_vision.cpp:676-691) */
    proj(W->patch_w, H, W->patch_dim, W->patch_dim, patches, T, quant_act, x);
    if (h == W->pos_side && w == W->pos_side)
        memcpy(pos, W->pos_embd, (size_t) T * H * sizeof(float));
    else
        orc_pos_resize(W->pos_embd, W->pos_side, H, h, w, pos);
    for (int64_t t = 0; t < T; ++t)
        for (int64_t i = 0; i < H; ++i)
            x[t * H + i] = (x[t * H + i] + W->patch_b[i]) + pos[t * H + i];

    int64_t so = 0, sl = T;
    for (int64_t l = 0; l < W->n_layer; ++l)
        encoder_block(&W->blocks[l], x, T, H, W->F, W->Fp, W->n_head, W->eps, &so, &sl, 1, quant_act);

    orc_layernorm(x, W->post_ln_w, W->post_ln_b, W->eps, T, H, x);

    if (pooling == 0) {
        /* MEAN (siglip2_vision.cpp:699-701) */
        for (int64_t i = 0; i < H; ++i) {
            double acc = 0.0;
            for (int64_t t = 0; t < T; ++t) acc += x[t * H + i];
            out[i] = (float) (acc / (double) T);
        }
    } else {
        /* attention-pool head (siglip2_vision.cpp:249-314) */
        float *q   = (float *) malloc((size_t) H * sizeof(float));
        float *qkv = (float *) malloc((size_t) (T + 1) * 3 * H * sizeof(float));
        float *k   = (float *) malloc((size_t) T * H * sizeof(float));
        float *v   = (float *) malloc((size_t) T * H * sizeof(float));
        float *att = (float *) malloc((size_t) (T + 1) * H * sizeof(float));
        float *a   = (float *) malloc((size_t) H * sizeof(float));
        float *n1  = (float *) malloc((size_t) H * sizeof(float));
        float *up  = (float *) malloc((size_t) W->F * sizeof(float));
        float *dn  = (float *) malloc((size_t) H * sizeof(float));
        proj(W->hq_w, H, H, H, W->probe, 1, quant_act, q);
        add_bias(q, W->hq_b, 1, H);
        proj(W->hk_w, H, H, H, x, T, quant_act, k);
        add_bias(k, W->hk_b, T, H);
        proj(W->hv_w, H, H, H, x, T, quant_act, v);
        add_bias(v, W->hv_b, T, H);
        /* pack [probe q ; K ; V] rows: query row 0 attends to key rows 1..T */
        memset(qkv, 0, (size_t) (T + 1) * 3 * H * sizeof(float));
        memcpy(qkv, q, (size_t) H * sizeof(float));
        for (int64_t t = 0; t < T; ++t) {
            memcpy(qkv + (t + 1) * 3 * H + H, k + t * H, (size_t) H * sizeof(float));
            memcpy(qkv + (t + 1) * 3 * H + 2 * H, v + t * H, (size_t) H * sizeof(float));
        }
        /* single query against T keys */
        if (quant_act) {
            for (int64_t i = 0; i < H; ++i) q[i] = half_of(q[i]);
            for (int64_t i = 0; i < T * H; ++i) { k[i] = half_of(k[i]); v[i] = half_of(v[i]); }
            attention_q8(q, 0, k, H, v, H, 1, T, W->n_head, H / W->n_head, att, H);
        } else {
            const int64_t dh = H / W->n_head;
            const float scale = 1.0f / sqrtf((float) dh);
            for (int64_t hd = 0; hd < W->n_head; ++hd) {
                double *sc = (double *) malloc((size_t) T * sizeof(double));
                double mx = -INFINITY;
                for (int64_t t = 0; t < T; ++t) {
                    double dot = 0.0;
                    for (int64_t i = 0; i < dh; ++i)
                        dot += (double) q[hd * dh + i] * (double) half_of(k[t * H + hd * dh + i]);
                    sc[t] = dot * (double) scale;
                    if (sc[t] > mx) mx = sc[t];
                }
                double den = 0.0;
                for (int64_t t = 0; t < T; ++t) { sc[t] = exp(sc[t] - mx); den += sc[t]; }
                for (int64_t i = 0; i < dh; ++i) {
                    double acc = 0.0;
                    for (int64_t t = 0; t < T; ++t) acc += sc[t] * (double) half_of(v[t * H + hd * dh + i]);
                    att[hd * dh + i] = (float) (acc / den);
                }
                free(sc);
            }
        }
        proj(W->ho_w, H, H, H, att, 1, quant_act, a);
        add_bias(a, W->ho_b, 1, H);
        orc_layernorm(a, W->hln_w, W->hln_b, W->eps, 1, H, n1);
        proj(W->hup_w, W->F, H, H, n1, 1, quant_act, up);
        for (int64_t i = 0; i < W->F; ++i) up[i] = tower_gelu(up[i] + W->hup_b[i]);
        proj(W->hdown_w, H, W->F, W->Fp, up, 1, quant_act, dn);
        for (int64_t i = 0; i < H; ++i) out[i] = a[i] + (dn[i] + W->hdown_b[i]);
        free(q); free(qkv); free(k); free(v); free(att); free(a); free(n1); free(up); free(dn);
    }
    free(x);
    free(pos);
    return 0;
}

int orc_text_encode(const orc_text_weights *W, const int32_t *ids, int64_t n_prompts,
                    int quant_act, float *out) {
    const int64_t H = W->H, P = W->n_pos, T = n_prompts * P;

    const int64_t Kb = H / 32;
    float *x = (float *) malloc((size_t) T * H * sizeof(float));
    /* get_rows(token_embd Q8_0) dequantizes the row; + position row (siglip2_text.cpp:837-847) */
    for (int64_t t = 0; t < T; ++t) {
        int64_t id = ids[t];
        const uint8_t *row = W->tok_embd + id * Kb * 34;
        for (int64_t kb = 0; kb < Kb; ++kb) {
            uint16_t dh;
            memcpy(&dh, row + kb * 34, 2);
            float d = orc_fp16_to_fp32(dh);
            for (int j = 0; j < 32; ++j) {
                float e = (float) (int8_t) row[kb * 34 + 2 + j] * d;
                x[t * H + kb * 32 + j] = e + W->pos_embd[(t % P) * H + kb * 32 + j];
            }
        }
    }
    int64_t *so = (int64_t *) malloc((size_t) n_prompts * sizeof(int64_t));
    int64_t *sl = (int64_t *) malloc((size_t) n_prompts * sizeof(int64_t));
    for (int64_t p = 0; p < n_prompts; ++p) { so[p] = p * P; sl[p] = P; }
    for (int64_t l = 0; l < W->n_layer; ++l)
        encoder_block(&W->blocks[l], x, T, H, W->F, W->Fp, W->n_head, W->eps, so, sl, n_prompts, quant_act);
    orc_layernorm(x, W->final_ln_w, W->final_ln_b, W->eps, T, H, x);
    /* last-token pool (pool_idx = n_pos-1) then head (siglip2_text.cpp:857-865) */
    float *pooled = (float *) malloc((size_t) n_prompts * H * sizeof(float));
    for (int64_t p = 0; p < n_prompts; ++p)
        memcpy(pooled + p * H, x + (p * P + P - 1) * H, (size_t) H * sizeof(float));
    proj(W->head_w, H, H, H, pooled, n_prompts, quant_act, out);
    add_bias(out, W->head_b, n_prompts, H);
    free(x); free(so); free(sl); free(pooled);
    return 0;
}

void orc_score(const float *img, int64_t I, const float *txt, int64_t J, int64_t H,
               float logit_scale, float logit_bias, float *logits, float *out) {
    float *a = (float *) malloc((size_t) I * H * sizeof(float));
    float *b = (float *) malloc((size_t) J * H * sizeof(float));
    memcpy(a, img, (size_t) I * H * sizeof(float));
    memcpy(b, txt, (size_t) J * H * sizeof(float));
    float *rows[2] = { a, b };
    int64_t nr[2] = { I, J };
    for (int s = 0; s < 2; ++s)
        for (int64_t r = 0; r < nr[s]; ++r) {
            float *row = rows[s] + r * H;
            double sumsq = 0.0;
            for (int64_t c = 0; c < H; ++c) sumsq += (double) row[c] * (double) row[c];
            float inv = (float) (1.0 / (sqrt(sumsq) + 1e-12));
            for (int64_t c = 0; c < H; ++c) row[c] *= inv;
        }
    /* exp and the sigmoid's division are the library's own (orc_expf,
     * orc_div), the exponent clamped to 80 as in orc_gelu */
    const float scale = orc_expf(logit_scale);
    #pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < I; ++i)
        for (int64_t j = 0; j < J; ++j) {
            double dot = 0.0;
            for (int64_t c = 0; c < H; ++c) dot += (double) a[i * H + c] * (double) b[j * H + c];
            float logit = (float) (dot * (double) scale + (double) logit_bias);
            float p;
            if (logit >= 0.0f) { float e = orc_expf(logit < 80.0f ? -logit : -80.0f); p = orc_div(1.0f, 1.0f + e); }
            else               { float e = orc_expf(logit > -80.0f ? logit : -80.0f); p = orc_div(e, 1.0f + e); }
            if (logits) logits[i * J + j] = logit;
            out[i * J + j] = p;
        }
    free(a);
    free(b);
}
