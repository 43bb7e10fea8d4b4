/*
 * b2q_oracle.h — CPU restatement of the SigLIP2 Q8_0 x q8_1 hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path
 * and the timed CPU baseline; nothing in the product links, loads or calls
 * it.  Every function cites the reference source (paths relative to the
 * hbd-siglip2.cpp project root) whose behaviour it restates.
 *
 * Parity pins: the Q8_0 weight codec is pinned bit-exactly against gguf-py
 * 0.19.0 (the reference's own quantizer dependency, used at
 * scripts/convert_siglip2_to_gguf.py:263) through tests/golden fixtures; the
 * tower architecture is pinned at tolerance against HF transformers
 * Siglip2VisionModel/Siglip2TextModel run with the same dequantized weights.
 * ggml's own mul_mat/quantize_q8_1 (the empty `ggml` submodule) cannot be
 * built here, so the GEMM arithmetic follows the in-repo restatement in
 * src/cuda/siglip2_custom_mmq.cu and is otherwise unpinned against ggml.
 *
 * Canonical fp32 operation order (the GPU kernels follow the same order so
 * that, attention aside, results are bit-identical):
 *   q8_1 quantize  a = max|x| ; d = a/127 ; inv = a==0 ? 0 : 127/a ;
 *                  q = rint(x*inv) clamped to [-128,127]     (custom_mmq.cu:63-81)
 *   block GEMM     for kb ascending: t = (float)S_kb * dw ; acc = fma(t, dx, acc)
 *                                                            (custom_mmq.cu:263-266)
 *   LayerNorm      per-row sums in the 32-lane x float4 order described at
 *                  orc_layernorm; inv_std = 1/sqrt(var+eps) correctly rounded
 *                                                            (siglip2_megakernel.cu:81-121)
 *   GELU           the tanh form 0.5*x*(1+tanh(y)) evaluated as the equal
 *                  x / (1 + e^{-2y}) with the library's own exp and division
 *                  (orc_gelu)                                (siglip2_megakernel.cu:276-280)
 *   bias/residual  (mm + b) + r, two separately rounded adds (siglip2_megakernel.cu:287-300)
 */
#ifndef B2Q_ORACLE_H
#define B2Q_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- element-rule variants (default 0: the canonical order above) ------- */
/* The other rules are the reference's own element functions, used to
 * measure how far two faithful implementations of a tower drift apart
 * (b2q_oracle.c describes each). */
#define ORC_RULE_LN   1
#define ORC_RULE_GELU 2
#define ORC_RULE_Q8   4
#define ORC_RULE_GEMM 8
void orc_set_rules(int rules);
int  orc_get_rules(void);

/* ---- scalar numerics ---------------------------------------------------- */
float    orc_fp16_to_fp32(uint16_t h);
uint16_t orc_fp32_to_fp16(float f);
float    orc_expf(float x);
float    orc_div(float a, float b);
float    orc_gelu(float x);
void     orc_gelu_n(const float *x, int64_t n, float *y);
int      orc_num_threads(void);
void     orc_set_num_threads(int n);

/* ---- formats ------------------------------------------------------------ */
/* Q8_0 rows: x is [N][K] fp32, output [N][Kp/32] blocks of 34 bytes
 * ([fp16 d][32 x int8]).  Columns K..Kp-1 are zero (the K-padding rule of
 * tools/siglip2-quantize/main.cpp:174-186). */
void orc_quantize_q8_0(const float *x, int64_t N, int64_t K, int64_t Kp, uint8_t *out);
void orc_dequantize_q8_0(const uint8_t *w, int64_t N, int64_t Kp, float *out);

/* q8_1 activation planes: qs [M][Kp] int8, d [M][Kp/32] fp32. */
void orc_quantize_q8_1(const float *x, int64_t M, int64_t K, int64_t ldx, int64_t Kp,
                       int8_t *qs, float *d);
/* The same with a selectable rounding convention (0 = the default above;
 * 1 = half away from zero; 2 = x/d; 3 = x*(1/d) half away), see b2q_oracle.c. */
void orc_quantize_q8_1_rule(const float *x, int64_t M, int64_t K, int64_t ldx, int64_t Kp,
                            int8_t *qs, float *d, int rule);

/* ---- GEMM --------------------------------------------------------------- */
/* y[m][n] = sum_kb dw[n,kb]*dx[m,kb]*S[m,n,kb]  (canonical order above).
 * block_sums (optional, may be NULL) receives S as [M][N][Kb] int32. */
void orc_gemm_q8(const uint8_t *w, int64_t N, int64_t Kp,
                 const int8_t *qs, const float *dx, int64_t M,
                 float *y, int32_t *block_sums);
/* 1 when orc_gemm_q8 runs its AVX512-VNNI form on this host (bit-identical
 * to the scalar loop; ORC_NO_VNNI in the environment forces the scalar one). */
int orc_gemm_uses_vnni(void);

/* ---- row ops ------------------------------------------------------------ */
void orc_layernorm(const float *x, const float *w, const float *b, float eps,
                   int64_t M, int64_t H, float *y);

/* ---- attention ---------------------------------------------------------- */
/* qkv: [T][3H] fp32 rows laid out [Q | K | V], head h at offset h*dh inside
 * each (siglip2_vision.cpp:198-206).  K and V are rounded to fp16 before use
 * (siglip2_vision.cpp:164-165); scores, softmax and accumulation in double.
 * (The quantized towers use the fixed fp32 order documented at attention_q8
 * in b2q_oracle.c instead.)
 * key_len (may be NULL) limits the keys of each sequence; seq_off/seq_len
 * describe n_seq packed sequences.  out: [T][H]. */
void orc_attention(const float *qkv, int64_t T, int64_t H, int64_t n_head,
                   const int64_t *seq_off, const int64_t *seq_len, int64_t n_seq,
                   float *out);

/* ---- position embedding resize ----------------------------------------- */
/* table: [side*side][H] (row-major grid), out: [h*w][H]; bilinear with
 * antialias, align_corners=False (siglip2_vision.cpp:680-691). */
void orc_pos_resize(const float *table, int64_t side, int64_t H,
                    int64_t h, int64_t w, float *out);

/* ---- towers ------------------------------------------------------------- */
typedef struct orc_block {
    const float   *ln1_w, *ln1_b, *ln2_w, *ln2_b;
    const uint8_t *qkv_w; const float *qkv_b;    /* Q8_0 [3H][H]           */
    const uint8_t *o_w;   const float *o_b;      /* Q8_0 [H][H]            */
    const uint8_t *up_w;  const float *up_b;     /* Q8_0 [F][H]            */
    const uint8_t *down_w; const float *down_b;  /* Q8_0 [H][Fp] (K-padded) */
} orc_block;

typedef struct orc_vision_weights {
    int64_t H, F, Fp, n_head, n_layer, patch_dim, pos_side;
    float   eps;
    const uint8_t *patch_w; const float *patch_b;   /* Q8_0 [H][patch_dim] */
    const float   *pos_embd;                        /* [side*side][H]       */
    const orc_block *blocks;
    const float   *post_ln_w, *post_ln_b;
    /* attention-pool head (siglip2_vision.cpp:249-314) */
    const float   *probe;                           /* [H]                  */
    const uint8_t *hq_w, *hk_w, *hv_w, *ho_w;
    const float   *hq_b, *hk_b, *hv_b, *ho_b;
    const float   *hln_w, *hln_b;
    const uint8_t *hup_w; const float *hup_b;
    const uint8_t *hdown_w; const float *hdown_b;
} orc_vision_weights;

/* One image: patches [h*w][patch_dim]; pooling 0 = MEAN, 1 = PROBE.
 * out: [H].  quant_act = 0 runs every projection with fp32 activations
 * (dequantized weights) — the architecture check against HF. */
int orc_vision_encode(const orc_vision_weights *W, const float *patches,
                      int64_t h, int64_t w, int pooling, int quant_act, float *out);

typedef struct orc_text_weights {
    int64_t H, F, Fp, n_head, n_layer, vocab, n_pos;
    float   eps;
    const uint8_t *tok_embd;                        /* Q8_0 [vocab][H]      */
    const float   *pos_embd;                        /* [n_pos][H]           */
    const orc_block *blocks;
    const float   *final_ln_w, *final_ln_b;
    const uint8_t *head_w; const float *head_b;     /* Q8_0 [H][H]          */
} orc_text_weights;

/* n_prompts x n_pos token ids -> out [n_prompts][H] (siglip2_text.cpp:741-932) */
int orc_text_encode(const orc_text_weights *W, const int32_t *ids, int64_t n_prompts,
                    int quant_act, float *out);

/* Sigmoid scores (siglip2_score.cpp:78-134): img [I][H], txt [J][H] ->
 * out [I][J] = sigmoid(exp(logit_scale) * <img_i/|img_i|, txt_j/|txt_j|> + bias),
 * norms and dots in double; logits (may be NULL) receives the pre-sigmoid
 * values.  exp and the division are orc_expf / orc_div. */
void orc_score(const float *img, int64_t I, const float *txt, int64_t J, int64_t H,
               float logit_scale, float logit_bias, float *logits, float *out);

#ifdef __cplusplus
}
#endif
#endif
