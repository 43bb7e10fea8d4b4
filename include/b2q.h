/*
 * b2q.h — C ABI of the B200 (sm_100a) SigLIP2 Q8_0 x q8_1 hot path.
 *
 * Plain pointers and sizes only.  Device pointers are CUDA device addresses
 * on the calling thread's current device; `stream` is a cudaStream_t (NULL =
 * legacy default stream).  Every call returns a b2q_status (0 = OK); on
 * failure b2q_last_error() describes it.  No call traps or aborts, and no
 * launch call allocates device memory, so launches can be captured into CUDA
 * graphs (pointers are baked into the graph, as in the reference).
 *
 * Reference interfaces replaced (paths inside the hbd-siglip2.cpp project):
 *  - ggml_mul_mat(W Q8_0, X F32) executed by ggml-cuda's MMQ — call sites
 *    src/siglip2_vision.cpp:199,227,235,239,676 and src/siglip2_text.cpp:189,
 *    196,200,864; raw-pointer precedent src/cuda/siglip2_custom_mmq.cuh:96-103
 *  - quantize_q8_1 (src/cuda/siglip2_custom_mmq.cuh:63-67)
 *  - fused LayerNorm (src/cuda/siglip2_megakernel.cuh:49-57)
 *  - the bias+GELU / bias+residual tails (src/cuda/siglip2_megakernel.cuh:
 *    126-142) — here folded into the GEMM epilogue.
 */
#ifndef B2Q_H
#define B2Q_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int b2q_status;
enum {
    B2Q_OK = 0,
    B2Q_ERR_INVALID = -1,   /* null pointer, unknown enum value           */
    B2Q_ERR_SHAPE = -2,     /* unsupported or inconsistent shape          */
    B2Q_ERR_ALIGN = -3,     /* pointer or stride alignment                 */
    B2Q_ERR_CUDA = -4,      /* CUDA runtime / driver error                 */
    B2Q_ERR_DEVICE = -5,    /* a kernel's bounded wait expired             */
    B2Q_ERR_NOT_INIT = -6,  /* b2q_init not called on this thread/device   */
    B2Q_ERR_NOMEM = -7      /* allocation at init/registration failed      */
};

/* Operand carrier of the int8 values on the tensor cores. */
enum {
    B2Q_OPS_I8 = 0,   /* tcgen05 kind::i8, int32 accumulators              */
    B2Q_OPS_F16 = 1   /* int8 values carried exactly in fp16, kind::f16    */
};

/* Thread-local description of the last failure on this thread. */
const char *b2q_last_error(void);
int b2q_abi_version(void);
/* Kernel launches this library has issued in the process (all devices);
 * the kernels of a replayed encode graph count once per replay. */
uint64_t b2q_launch_count(void);
/* Tower encodes launched as one captured CUDA graph (B2Q_TUNE_GRAPHS). */
uint64_t b2q_graph_launch_count(void);

/* Per-device set-up (current device); allocates the device error word.
 * ops_mode: B2Q_OPS_I8 or B2Q_OPS_F16 (-1 = library default). */
b2q_status b2q_init(int device, int ops_mode);
/* Tuning knobs of the current device's state (reference precedent: the
 * SIGLIP2_* environment switches of src/cuda/siglip2_megakernel.cu:1378-1401).
 *   B2Q_TUNE_GEMM_BN:    GEMM tile width 64 (two CTAs per SM), 128, 192
 *                        (one CTA per SM, twelve epilogue warps) or 256
 *                        (0 = chosen per shape by the tile rounds each
 *                        layout needs: 192 at large M and for the wide
 *                        projections at small M, 64-column tiles when
 *                        128-column ones would not cover every SM, else 128
 *                        with two CTAs per SM, or 256 for the GELU epilogue)
 *   B2Q_TUNE_TIMEOUT_NS: bound of every in-kernel wait (default 2 s)
 *   B2Q_TUNE_ATTN_EXACT: 1 = attention in one fixed fp32 order (slow; makes
 *                        the tower bit-reproducible), 0 = tensor cores
 *   B2Q_TUNE_TEST_STALL: 1 = (tests only) the GEMM's TMA producer and the
 *                        attention's MMA issuer issue nothing, so the other
 *                        roles' bounded waits expire and the launch reports
 *                        B2Q_ERR_DEVICE through b2q_check_device without
 *                        faulting or hanging
 *   B2Q_TUNE_ATTN_KERNEL: tensor-core attention kernel: 0 = tcgen05 (TMEM
 *                        accumulators, 128 queries per CTA; default),
 *                        1 = mma.sync (64 queries per CTA)
 *   B2Q_TUNE_GEMM_CTAS:  GEMM CTAs resident per SM: 1 (eight epilogue warps
 *                        per CTA), 2 (128-column tiles, four epilogue warps
 *                        per CTA), 0 = chosen per shape and epilogue (2 when
 *                        the 128-column tiles cover every SM, except for the
 *                        GELU -> q8_1 epilogue).  Every setting gives
 *                        bit-identical results.
 *   B2Q_TUNE_GRAPHS:     1 (default) = a vision or text encode that repeats
 *                        the previous call's geometry, buffers and settings
 *                        is replayed as a CUDA graph (captured on the
 *                        second such call), 0 = kernels launched one by one.
 *                        Bit-identical either way. */
enum {
    B2Q_TUNE_GEMM_BN = 1,
    B2Q_TUNE_TIMEOUT_NS = 2,
    B2Q_TUNE_ATTN_EXACT = 3,
    B2Q_TUNE_TEST_STALL = 4,
    B2Q_TUNE_ATTN_KERNEL = 5,
    B2Q_TUNE_GEMM_CTAS = 6,
    B2Q_TUNE_GRAPHS = 7
};
b2q_status b2q_tune(int key, int64_t value);
/* Reads (and clears) the device error word after synchronising `stream`;
 * B2Q_ERR_DEVICE when it was set: codes 1-4 = an in-kernel wait expired
 * (1 TMA data, 2 stage release, 3 MMA commit, 4 accumulator release),
 * 5 = a token id outside the vocabulary. */
b2q_status b2q_check_device(void *stream, uint32_t *code_out);

/* ---- weights -------------------------------------------------------------
 * Registers a ggml Q8_0 tensor (block_q8_0 = fp16 d + 32 int8, 34 bytes):
 * N rows of K (ne[0], a multiple of 32; K-padded tensors pass the padded K),
 * row stride row_bytes (>= K/32*34).  `q8_0` is a device pointer, or a host
 * pointer when src_is_host != 0.  Repacks once into a 16-byte-aligned value
 * plane [N][K] and an fp32 scale plane [K/32][N rounded up to 64] (columns
 * permuted inside each 64-column group for the GEMM epilogue's loads); the
 * source is not retained.
 * Replaces the per-call raw read in src/cuda/siglip2_custom_mmq.cu:176-199. */
typedef struct b2q_weight b2q_weight;
b2q_status b2q_weight_register(const void *q8_0, int64_t N, int64_t K, int64_t row_bytes, int src_is_host,
                               void *stream, b2q_weight **out);
b2q_status b2q_weight_release(b2q_weight *w);
b2q_status b2q_weight_shape(const b2q_weight *w, int64_t *N, int64_t *K);

/* ---- activations ("q8_1 planes") -----------------------------------------
 * An activation buffer holds M rows of logical width K quantized per 32
 * columns (Kp = K rounded up to 32; columns K..Kp-1 are zero, the pad_x_to_w
 * rule of src/siglip2_vision.cpp:99-107):
 *   values: [M][Kp], 1 byte each (B2Q_OPS_I8) or fp16 carriers (B2Q_OPS_F16)
 *   scales: [Kp/32][ld] fp32, ld = M rounded up to 4, at byte offset
 *           scale_offset (256-aligned)
 * The caller allocates b2q_act_bytes(M, K) bytes (256-byte aligned). */
size_t b2q_act_bytes(int64_t M, int64_t K);
b2q_status b2q_act_layout(int64_t M, int64_t K, int64_t *Kp, int64_t *value_bytes, int64_t *scale_offset,
                          int64_t *scale_ld);

/* q8_1 quantize of fp32 rows x[M][ldx] (src/cuda/siglip2_custom_mmq.cu:51-97):
 * d = max|x|/127, q = rint(x*127/max|x|). */
b2q_status b2q_quantize_q8_1(const float *x, int64_t M, int64_t K, int64_t ldx, void *act, void *stream);

/* LayerNorm + affine then q8_1 quantize of the result, one pass
 * (src/cuda/siglip2_megakernel.cu:81-138 fused with the quantize step that
 * feeds the next mul_mat).  H must be a multiple of 128.  y_opt (may be
 * NULL) also receives the fp32 LayerNorm output. */
b2q_status b2q_ln_quantize_q8_1(const float *x, const float *w, const float *b, float eps, int64_t M, int64_t H,
                                void *act, float *y_opt, void *stream);

/* ---- GEMM ------------------------------------------------------------------
 * y[m][n] = sum_kb dW[n,kb] * dX[m,kb] * S[m,n,kb], S the int32 dot of the
 * 32 int8 pairs of block kb, accumulated in fp32 over ascending kb as
 * fma((float)S*dW, dX, acc) (src/cuda/siglip2_custom_mmq.cu:263-266),
 * followed by the epilogue below.  Output row stride ld_out (0 = N). */
enum {
    B2Q_EPI_NONE = 0,            /* y = acc                                  fp32  */
    B2Q_EPI_BIAS = 1,            /* y = acc + bias                           fp32  */
    B2Q_EPI_BIAS_RESIDUAL = 2,   /* y = (acc + bias) + residual              fp32  */
    B2Q_EPI_BIAS_GELU_Q8 = 3,    /* act_out <- q8_1(gelu(acc + bias)), K'=N        */
    B2Q_EPI_BIAS_F16 = 4         /* y = fp16(acc + bias)                     fp16  */
};
typedef struct b2q_epilogue {
    int kind;
    const float *bias;      /* [N] or NULL (treated as zeros)                 */
    const float *residual;  /* [M][ld_out] for BIAS_RESIDUAL; may equal y     */
    void *act_out;          /* activation buffer (M rows, K' = N) for GELU_Q8 */
    int64_t ld_out;         /* elements; 0 means N                            */
} b2q_epilogue;

b2q_status b2q_mul_mat_q8_0(const b2q_weight *w, const void *act, int64_t M, void *y, const b2q_epilogue *epi,
                            void *stream);

/* ggml_mul_mat(W Q8_0, X F32) -> Y F32 [M][N]: quantizes X (K = x_cols <= W's
 * K, zero-extended) into act_scratch (b2q_act_bytes(M, W's K) bytes), then
 * runs the GEMM. */
b2q_status b2q_mul_mat_q8_0_f32(const b2q_weight *w, const float *x, int64_t M, int64_t x_cols, float *y,
                                void *act_scratch, void *stream);

/* ggml_mul_mat like b2q_mul_mat_q8_0_f32, for callers that cannot allocate
 * device memory (no counterpart in the reference): an op hook inside another
 * framework's graph executor gets only the op's tensors and may not call
 * cudaMalloc mid-graph.  The q8_1 scratch is a fixed array of
 * B2Q_NOALLOC_MAX_SCRATCH_BYTES inside the library, reserved on every GPU
 * that loads it until the process exits; calls needing more
 * (b2q_act_bytes(M, K) > the maximum) fail with B2Q_ERR_SHAPE.  The first
 * call on a device looks up the array's device address
 * (cudaGetSymbolAddress), so make that first call before any stream capture.
 * All calls share the array: calls that overlap on the GPU race. */
#define B2Q_NOALLOC_MAX_SCRATCH_BYTES (32u << 20)
b2q_status b2q_mul_mat_q8_0_f32_noalloc(const b2q_weight *w, const float *x, int64_t M, int64_t x_cols, float *y,
                                        void *stream);

/* Debug: the int32 block dots S[kb][m][n] (Kb*M*N int32) of one GEMM. */
b2q_status b2q_block_sums(const b2q_weight *w, const void *act, int64_t M, int32_t *sums, void *stream);

/* ---- attention (head_dim 72) ---------------------------------------------
 * flash_attn_ext over packed sequences, replacing src/siglip2_vision.cpp:
 * 154-175 with the QKV-prep / post-FA copies of src/cuda/siglip2_megakernel.cu:
 * 166-267,358-394.  q, k, v: fp16 rows (row strides ldq/ldk/ldv elements),
 * head h at column h*72.  Sequence s (host arrays, n_seq entries) has q_len[s]
 * query rows from q_off[s], k_len[s] keys/values from k_off[s], and writes
 * out[o_off[s] + i][h*72 + d] (fp32, row stride ldo).  Softmax scale
 * 1/sqrt(72).  tiles_scratch: device memory of b2q_attention_scratch_bytes()
 * for the same sequence description (the tile table is copied into it).
 * Runs on the tcgen05 kernel unless B2Q_TUNE_ATTN_KERNEL (mma.sync) or
 * B2Q_TUNE_ATTN_EXACT (fixed fp32 order) selects another. */
size_t b2q_attention_scratch_bytes(const int32_t *q_len, int32_t n_seq);
b2q_status b2q_attention(const void *q, int64_t ldq, const void *k, int64_t ldk, const void *v, int64_t ldv,
                         const int32_t *q_off, const int32_t *q_len, const int32_t *k_off, const int32_t *k_len,
                         const int32_t *o_off, int32_t n_seq, int32_t n_head, int32_t d_head, float *out, int64_t ldo,
                         void *tiles_scratch, void *stream);

/* ---- vision tower ----------------------------------------------------------
 * Batched counterpart of siglip2::VisionEncoder (src/siglip2_vision.h:25-60;
 * load src/siglip2_vision.cpp:424-599, encode :601-758).  Tensors are handed
 * over by their GGUF names ("v.patch_embd.weight", "v.blk.N.attn_qkv.weight",
 * "v.head.probe", ... as loaded at src/siglip2_vision.cpp:496-556) with the
 * ggml type id (0 = F32, 8 = Q8_0) and ggml shape (ne0 innermost).  Q8_0 ffn_down
 * tensors carry the zero K-padding 4304 -> 4320 (tools/siglip2-quantize/
 * main.cpp:174-186).  A batch packs n_images images back to back: image i has
 * grid_hw[2i] x grid_hw[2i+1] patches of patch_dim fp32 values (row-major
 * over the grid); out receives n_images x hidden fp32 embeddings.  pooling
 * follows siglip2::Pooling: MEAN = 0, PROBE = 1. */
typedef struct b2q_vision b2q_vision;
typedef struct b2q_vision_config {
    int32_t hidden;     /* 1152 */
    int32_t ffn;        /* 4304 */
    int32_t n_head;     /* 16 (head_dim 72) */
    int32_t n_layer;    /* 27 */
    int32_t patch_dim;  /* 768 = 3 x 16 x 16 */
    int32_t pos_side;   /* 16: the learned 16 x 16 position table */
    float eps;          /* 1e-6 */
} b2q_vision_config;
enum { B2Q_POOL_MEAN = 0, B2Q_POOL_PROBE = 1 };
b2q_status b2q_vision_create(const b2q_vision_config *cfg, b2q_vision **out);
b2q_status b2q_vision_destroy(b2q_vision *v);
b2q_status b2q_vision_set_tensor(b2q_vision *v, const char *name, int32_t ggml_type, const void *host_data,
                                 int64_t ne0, int64_t ne1, void *stream);
/* Workspace for batches of up to max_tokens patches / max_images images
 * (allocates; encode calls with larger batches grow it). */
b2q_status b2q_vision_reserve(b2q_vision *v, int64_t max_tokens, int32_t max_images);
/* Device in, device out (patches [T][patch_dim], out [n_images][hidden]). */
b2q_status b2q_vision_encode(b2q_vision *v, const float *patches, const int32_t *grid_hw, int32_t n_images,
                             int32_t pooling, float *out, void *stream);
/* Host in, host out: uploads the patches, encodes, downloads the embeddings
 * and synchronises `stream`. */
b2q_status b2q_vision_encode_host(b2q_vision *v, const float *patches_host, const int32_t *grid_hw,
                                  int32_t n_images, int32_t pooling, float *out_host, void *stream);
/* Pipelined host entry point: queues the upload of the patches (on the
 * tower's own copy stream, into one of two device slots), the encode and the
 * download of the embeddings (on `stream`), and returns without waiting, so
 * the next call's upload runs while this call's encode does.  With pinned
 * host buffers the copies overlap the kernels; `out_host` must not be read,
 * nor `patches_host` rewritten, until b2q_vision_wait (or a synchronisation
 * of `stream`) returns.  Results are those of b2q_vision_encode_host. */
b2q_status b2q_vision_submit_host(b2q_vision *v, const float *patches_host, const int32_t *grid_hw,
                                  int32_t n_images, int32_t pooling, float *out_host, void *stream);
/* Waits for every encode submitted on `stream`. */
b2q_status b2q_vision_wait(b2q_vision *v, void *stream);
/* Waits for one submission's embeddings to be in its host buffer: back = 0
 * the latest b2q_vision_submit_host call, 1 the one before it.  A caller that
 * consumes each batch's embeddings (a gather across GPUs, a reply) submits
 * batch i + 1, waits with back = 1 and handles batch i while batch i + 1's
 * encode runs. */
b2q_status b2q_vision_wait_submitted(b2q_vision *v, int32_t back);

/* ---- text tower ------------------------------------------------------------
 * Batched counterpart of siglip2::TextEncoder::encode_batch
 * (src/siglip2_text.cpp:741-932; tensors by the GGUF names it loads at
 * :485-496 and "t.blk.N.*" at :38).  "t.token_embd.weight" is a Q8_0 table
 * [vocab][hidden] read row by row (get_rows); every other Q8_0 tensor is a
 * projection.  A batch is n_prompts rows of n_pos token ids (int32, each in
 * [0, vocab); an id outside it is replaced by 0 and reported through
 * b2q_check_device); out receives n_prompts x hidden fp32 embeddings: final
 * LayerNorm of each prompt's last token, then the head projection + bias.
 * Attention always runs in the fixed fp32 order of B2Q_TUNE_ATTN_EXACT, so
 * the embeddings are bit-reproducible. */
typedef struct b2q_text b2q_text;
typedef struct b2q_text_config {
    int32_t hidden;     /* 1152 */
    int32_t ffn;        /* 4304 */
    int32_t n_head;     /* 16 (head_dim 72) */
    int32_t n_layer;    /* 27 */
    int32_t vocab;      /* 256000 */
    int32_t n_pos;      /* 64 */
    float eps;          /* 1e-6 */
} b2q_text_config;
b2q_status b2q_text_create(const b2q_text_config *cfg, b2q_text **out);
b2q_status b2q_text_destroy(b2q_text *t);
b2q_status b2q_text_set_tensor(b2q_text *t, const char *name, int32_t ggml_type, const void *host_data, int64_t ne0,
                               int64_t ne1, void *stream);
b2q_status b2q_text_reserve(b2q_text *t, int32_t max_prompts);
/* Device in ([n_prompts][n_pos] int32), device out ([n_prompts][hidden]). */
b2q_status b2q_text_encode(b2q_text *t, const int32_t *ids, int32_t n_prompts, float *out, void *stream);
/* Host in, host out; synchronises `stream`. */
b2q_status b2q_text_encode_host(b2q_text *t, const int32_t *ids_host, int32_t n_prompts, float *out_host,
                                void *stream);

/* ---- image-text scoring -----------------------------------------------------
 * score_image_text (src/siglip2_score.cpp:90-134) on the device: both sets of
 * rows L2-normalised in double (+1e-12), logits[i][j] = dot(img_i, txt_j) *
 * e^{logit_scale} + logit_bias with the dot in double, probs = sigmoid(logits).
 * All pointers are device pointers; logits or probs may be NULL (not both).
 * scratch: b2q_score_scratch_bytes(n_image, n_text, hidden) bytes. */
size_t b2q_score_scratch_bytes(int32_t n_image, int32_t n_text, int32_t hidden);
b2q_status b2q_score(const float *img, int32_t n_image, const float *txt, int32_t n_text, int32_t hidden,
                     float logit_scale, float logit_bias, float *logits, float *probs, void *scratch, void *stream);

/* ---- GGUF checkpoints -------------------------------------------------------
 * Counterpart of GGUFLoader (src/gguf_loader.cpp:205-337).  b2q_gguf_open maps
 * a GGUF v2/v3 file read-only and parses its tensor table (no GPU needed);
 * tensor data pointers stay valid until b2q_gguf_close.  The tower loaders
 * hand every "v." / "t." tensor to b2q_vision_set_tensor / b2q_text_set_tensor:
 * biases, LayerNorm parameters, position tables and the probe as F32 (F16 and
 * BF16 widened), every other ".weight" as Q8_0 (stored Q8_0: as is; stored
 * F16/BF16/F32: quantized here with the ggml Q8_0 rule, K zero-padded to a
 * multiple of 32, as the reference converts F16 at load, gguf_loader.cpp:
 * 297-318).  Scoring parameters are [1]-shaped tensors ("mm.logit_scale",
 * "mm.logit_bias", src/siglip2_score.cpp:25-72): b2q_gguf_scalar_f32. */
typedef struct b2q_gguf b2q_gguf;
b2q_status b2q_gguf_open(const char *path, b2q_gguf **out);
b2q_status b2q_gguf_close(b2q_gguf *g);
int64_t b2q_gguf_n_tensors(const b2q_gguf *g);
/* ne: 4 entries (unused dimensions 1); data points into the mapped file. */
b2q_status b2q_gguf_tensor(const b2q_gguf *g, int64_t i, const char **name, int32_t *ggml_type, int32_t *n_dims,
                           int64_t *ne, const void **data);
b2q_status b2q_gguf_scalar_f32(const b2q_gguf *g, const char *name, float *out);
b2q_status b2q_vision_load_gguf(b2q_vision *v, const b2q_gguf *g, void *stream);
b2q_status b2q_text_load_gguf(b2q_text *t, const b2q_gguf *g, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* B2Q_H */
