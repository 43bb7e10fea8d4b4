// b2q_tower.cu — SigLIP2 vision tower driver over the Q8_0 hot path.
//
// Counterpart of VisionEncoder::load/encode (src/siglip2_vision.cpp:424-758)
// for batches: every image of a batch is packed into one token stream (its
// own grid, no padding), so each projection is one large GEMM over all
// tokens and attention runs per image on the packed rows.  Per layer
// (build_block, src/siglip2_vision.cpp:181-244):
//   LN1 -> q8_1            (LayerNorm fused with the activation quantize)
//   QKV GEMM + bias -> fp16 rows [Q | K | V]       (attention operands)
//   attention (head_dim 72) -> fp32 -> q8_1
//   O GEMM, epilogue (acc + b) + x -> x           (in place)
//   LN2 -> q8_1
//   fc1 GEMM, epilogue gelu(acc + b) -> q8_1 (K' = 4304 -> 4320)
//   fc2 GEMM, epilogue (acc + b) + x -> x
// then post-LN and MEAN pooling or the attention-pool head
// (build_probe_head, src/siglip2_vision.cpp:249-314).
#include "b2q_tower.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace b2q {

namespace {

// ---------------------------------------------------------------- kernels
// Position table [side*side][H] bilinearly resized (antialias, align_corners
// false) to each image's h x w grid (ggml_interpolate BILINEAR|ANTIALIAS at
// src/siglip2_vision.cpp:680-691; the counterpart of HF's F.interpolate with
// antialias=True): separable triangle filter of support max(1, in/out),
// weights normalised per output sample, accumulated in double.
struct ImageDesc {
    int t0, h, w, pad;
};

__device__ __forceinline__ int aa_taps(int in, int out, int i, int* lo, double* wt) {
    const double scale = static_cast<double>(in) / out;
    const double support = scale >= 1.0 ? scale : 1.0;
    const double center = scale * (i + 0.5);
    const double invs = scale >= 1.0 ? 1.0 / scale : 1.0;
    int xmin = static_cast<int>(center - support + 0.5);
    if (xmin < 0) xmin = 0;
    int xmax = static_cast<int>(center + support + 0.5);
    if (xmax > in) xmax = in;
    const int n = xmax - xmin;
    double tot = 0.0;
    for (int j = 0; j < n; ++j) {
        double w = 1.0 - fabs(((j + xmin) - center + 0.5) * invs);
        w = w < 0.0 ? 0.0 : w;
        wt[j] = w;
        tot += w;
    }
    for (int j = 0; j < n; ++j) wt[j] = tot != 0.0 ? wt[j] / tot : 0.0;
    *lo = xmin;
    return n;
}

// One block per kPosTok tokens of one image: the block's first threads
// compute each token's row and column taps once (shared memory), then all
// threads sweep the H channels, so the taps (double divisions) are not
// recomputed per channel and the table and output rows are read and written
// contiguously.  The per-element arithmetic and its order are those of the
// filter definition above.
constexpr int kPosTok = 8;
constexpr int kPosMaxTaps = 64;

__global__ void __launch_bounds__(128) pos_resize_kernel(const float* __restrict__ table, int side, int H,
                                                         const ImageDesc* __restrict__ imgs, float* __restrict__ out) {
    __shared__ double s_wy[kPosTok][kPosMaxTaps], s_wx[kPosTok][kPosMaxTaps];
    __shared__ int s_ny[kPosTok], s_nx[kPosTok], s_ly[kPosTok], s_lx[kPosTok];
    const ImageDesc im = imgs[blockIdx.y];
    const int n_tok = im.h * im.w;
    const int t_base = blockIdx.x * kPosTok;
    if (t_base >= n_tok) return;
    const bool same = im.h == side && im.w == side;
    if (!same && threadIdx.x < 2 * kPosTok) {
        const int k = threadIdx.x >> 1, t = t_base + k;
        if (t < n_tok) {
            if (threadIdx.x & 1)
                s_nx[k] = aa_taps(side, im.w, t % im.w, &s_lx[k], s_wx[k]);
            else
                s_ny[k] = aa_taps(side, im.h, t / im.w, &s_ly[k], s_wy[k]);
        }
    }
    __syncthreads();
    for (int k = 0; k < kPosTok && t_base + k < n_tok; ++k) {
        const int t = t_base + k;
        float* dst = out + static_cast<int64_t>(im.t0 + t) * H;
        if (same) {
            for (int i = threadIdx.x; i < H; i += blockDim.x) dst[i] = table[static_cast<int64_t>(t) * H + i];
            continue;
        }
        const int ny = s_ny[k], nx = s_nx[k], ly = s_ly[k], lx = s_lx[k];
        for (int i = threadIdx.x; i < H; i += blockDim.x) {
            double acc = 0.0;
            for (int a = 0; a < ny; ++a) {
                double row = 0.0;
                for (int b = 0; b < nx; ++b)
                    row = __dadd_rn(row, __dmul_rn(s_wx[k][b], table[static_cast<int64_t>((ly + a) * side + lx + b) * H + i]));
                acc = __dadd_rn(acc, __dmul_rn(s_wy[k][a], static_cast<double>(static_cast<float>(row))));
            }
            dst[i] = static_cast<float>(acc);
        }
    }
}

// MEAN pooling of each image's tokens (src/siglip2_vision.cpp:699-701).
__global__ void mean_pool_kernel(const float* __restrict__ x, int H, const ImageDesc* __restrict__ imgs,
                                 float* __restrict__ out) {
    const ImageDesc im = imgs[blockIdx.y];
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= H) return;
    const int n = im.h * im.w;
    double acc = 0.0;
    for (int t = 0; t < n; ++t) acc = __dadd_rn(acc, x[static_cast<int64_t>(im.t0 + t) * H + i]);
    out[static_cast<int64_t>(blockIdx.y) * H + i] = static_cast<float>(__ddiv_rn(acc, n));
}

}  // namespace

// ---------------------------------------------------------------- shared driver pieces
b2q_status TensorSet::put(const std::string& n, int32_t ggml_type, const void* host_data, int64_t ne0, int64_t ne1,
                          bool as_raw, cudaStream_t s) {
    if (ggml_type == 8) {   // GGML_TYPE_Q8_0: ne0 = K (innermost), ne1 = rows
        if (ne0 <= 0 || ne1 <= 0 || ne0 % 32) return set_error(B2Q_ERR_SHAPE, "Q8_0 tensor " + n + ": bad shape");
        if (as_raw) {
            const size_t bytes = static_cast<size_t>(ne1) * (ne0 / 32) * 34;
            DevBuf& b = raw_q8[n];
            B2Q_TRY(cuda_check(b.ensure(bytes), "cudaMalloc(table)"));
            B2Q_TRY(cuda_check(cudaMemcpyAsync(b.p, host_data, bytes, cudaMemcpyHostToDevice, s), "table upload"));
            return cuda_check(cudaStreamSynchronize(s), "table upload");
        }
        auto it = q8.find(n);
        if (it != q8.end()) {
            b2q_weight_release(it->second);
            q8.erase(it);
        }
        b2q_weight* w = nullptr;
        B2Q_TRY(b2q_weight_register(host_data, ne1, ne0, ne0 / 32 * 34, 1, s, &w));
        q8[n] = w;
        return B2Q_OK;
    }
    if (ggml_type == 0) {   // GGML_TYPE_F32
        const size_t bytes = static_cast<size_t>(ne0 * (ne1 > 0 ? ne1 : 1)) * 4;
        DevBuf& b = f32[n];
        B2Q_TRY(cuda_check(b.ensure(bytes), "cudaMalloc(tensor)"));
        B2Q_TRY(cuda_check(cudaMemcpyAsync(b.p, host_data, bytes, cudaMemcpyHostToDevice, s), "tensor upload"));
        return cuda_check(cudaStreamSynchronize(s), "tensor upload");
    }
    return set_error(B2Q_ERR_INVALID, "only GGML_TYPE_F32 (0) and GGML_TYPE_Q8_0 (8) tensors are accepted");
}

b2q_status gemm(const b2q_weight* w, const void* act, int64_t M, void* y, int kind, const float* bias,
                const float* residual, void* act_out, int64_t ld_out, cudaStream_t s) {
    b2q_epilogue e{kind, bias, residual, act_out, ld_out};
    return b2q_mul_mat_q8_0(w, act, M, y, &e, s);
}

static std::string blkname(const char* prefix, int l, const char* s) {
    return std::string(prefix) + "blk." + std::to_string(l) + "." + s;
}

b2q_status check_blocks(const TensorSet& ts, const char* prefix, int n_layer) {
    static const char* blk_q8[] = {"attn_qkv.weight", "attn_o.weight", "ffn_up.weight", "ffn_down.weight"};
    static const char* blk_f[] = {"ln1.weight", "ln1.bias", "attn_qkv.bias", "attn_o.bias", "ln2.weight",
                                  "ln2.bias", "ffn_up.bias", "ffn_down.bias"};
    for (int l = 0; l < n_layer; ++l) {
        for (const char* s : blk_q8)
            if (!ts.w(blkname(prefix, l, s))) return set_error(B2Q_ERR_INVALID, "missing " + blkname(prefix, l, s));
        for (const char* s : blk_f)
            if (!ts.f(blkname(prefix, l, s))) return set_error(B2Q_ERR_INVALID, "missing " + blkname(prefix, l, s));
    }
    return B2Q_OK;
}

b2q_status run_encoder_blocks(const TensorSet& ts, const char* prefix, int n_layer, int n_head, float eps, int64_t T,
                              int64_t H, float* x, __half* qkv, float* att, void* act_h, void* act_f,
                              const void* tiles, int n_tiles, bool exact_attention, cudaStream_t s) {
    for (int l = 0; l < n_layer; ++l) {
        auto W = [&](const char* n) { return ts.w(blkname(prefix, l, n)); };
        auto F = [&](const char* n) { return ts.f(blkname(prefix, l, n)); };
        B2Q_TRY(b2q_ln_quantize_q8_1(x, F("ln1.weight"), F("ln1.bias"), eps, T, H, act_h, nullptr, s));
        B2Q_TRY(gemm(W("attn_qkv.weight"), act_h, T, qkv, B2Q_EPI_BIAS_F16, F("attn_qkv.bias"), nullptr, nullptr, 0,
                     s));
        B2Q_TRY(cuda_check(launch_attention(qkv, 3 * H, qkv + H, 3 * H, qkv + 2 * H, 3 * H, tiles, n_tiles, n_head, att,
                                            H, s, exact_attention),
                           "attention launch"));
        B2Q_TRY(b2q_quantize_q8_1(att, T, H, H, act_h, s));
        B2Q_TRY(gemm(W("attn_o.weight"), act_h, T, x, B2Q_EPI_BIAS_RESIDUAL, F("attn_o.bias"), x, nullptr, 0, s));
        B2Q_TRY(b2q_ln_quantize_q8_1(x, F("ln2.weight"), F("ln2.bias"), eps, T, H, act_h, nullptr, s));
        B2Q_TRY(gemm(W("ffn_up.weight"), act_h, T, nullptr, B2Q_EPI_BIAS_GELU_Q8, F("ffn_up.bias"), nullptr, act_f, 0,
                     s));
        B2Q_TRY(gemm(W("ffn_down.weight"), act_f, T, x, B2Q_EPI_BIAS_RESIDUAL, F("ffn_down.bias"), x, nullptr, 0, s));
    }
    return B2Q_OK;
}

}  // namespace b2q

using namespace b2q;

struct b2q_vision {
    b2q_vision_config cfg{};
    int ffn_pad = 0;
    TensorSet ts;                                 // projections, biases, LN, tables, probe
    // workspace
    int64_t cap_tokens = 0;
    int32_t cap_images = 0;
    DevBuf x, pos, qkv16, attn, act_h, act_f, act_p, imgs, tiles, head_tiles, q16, ha, ha2, patches_in, out_dev;
    std::vector<uint8_t> host_tiles, host_head_tiles;
    bool probe_ready = false;
    // batch geometry whose tables are on the device (a repeated geometry
    // skips the upload and its stream synchronisation)
    std::vector<int32_t> tables_for;
    int n_tiles = 0, n_htiles = 0;
    // bumped whenever a tensor or a workspace buffer may have moved
    uint64_t gen = 0;
    EncodeGraph graph;
    // pipelined host entry point: two input / output slots, a copy stream,
    // and per slot the events "patches landed" and "encode done"
    DevBuf slot_in[2], slot_out[2];
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t landed[2] = {nullptr, nullptr}, done[2] = {nullptr, nullptr}, fetched[2] = {nullptr, nullptr};
    bool slot_busy[2] = {false, false};
    int next_slot = 0;
    ~b2q_vision() {
        for (int k = 0; k < 2; ++k) {
            if (landed[k]) cudaEventDestroy(landed[k]);
            if (done[k]) cudaEventDestroy(done[k]);
            if (fetched[k]) cudaEventDestroy(fetched[k]);
        }
        if (copy_stream) cudaStreamDestroy(copy_stream);
    }
    const float* f(const std::string& n) const { return ts.f(n); }
    const b2q_weight* w(const std::string& n) const { return ts.w(n); }
};

namespace {

b2q_status check_loaded(const b2q_vision* v) {
    if (!v->w("v.patch_embd.weight") || !v->f("v.patch_embd.bias") || !v->f("v.position_embd.weight") ||
        !v->f("v.post_ln.weight") || !v->f("v.post_ln.bias"))
        return set_error(B2Q_ERR_INVALID, "vision tower: stem / post-LN tensors missing");
    return check_blocks(v->ts, "v.", v->cfg.n_layer);
}

b2q_status check_head(const b2q_vision* v) {
    static const char* q8n[] = {"v.head.attn_q.weight", "v.head.attn_k.weight", "v.head.attn_v.weight",
                                "v.head.attn_o.weight", "v.head.ffn_up.weight", "v.head.ffn_down.weight"};
    static const char* fn[] = {"v.head.probe", "v.head.attn_q.bias", "v.head.attn_k.bias", "v.head.attn_v.bias",
                               "v.head.attn_o.bias", "v.head.ln.weight", "v.head.ln.bias", "v.head.ffn_up.bias",
                               "v.head.ffn_down.bias"};
    for (const char* n : q8n)
        if (!v->w(n)) return set_error(B2Q_ERR_INVALID, std::string("vision tower: missing ") + n);
    for (const char* n : fn)
        if (!v->f(n)) return set_error(B2Q_ERR_INVALID, std::string("vision tower: missing ") + n);
    return B2Q_OK;
}

}  // namespace

extern "C" {

b2q_status b2q_vision_create(const b2q_vision_config* cfg, b2q_vision** out) {
    B2Q_REQUIRE_STATE();
    (void) ds;
    if (!cfg || !out) return set_error(B2Q_ERR_INVALID, "null pointer");
    if (cfg->hidden != cfg->n_head * 72 || cfg->hidden % 128 || cfg->hidden / 128 != 9 || cfg->ffn <= 0 ||
        cfg->n_layer <= 0 || cfg->patch_dim % 32 || cfg->pos_side <= 0 ||
        cfg->pos_side > kPosMaxTaps)   // a resize tap count is at most the table side
        return set_error(B2Q_ERR_SHAPE,
                         "vision config: needs hidden 1152 = 16 heads x 72, patch_dim % 32 == 0, pos_side in 1..64");
    b2q_vision* v = new b2q_vision();
    v->cfg = *cfg;
    v->ffn_pad = static_cast<int>(round_up(cfg->ffn, 32));
    *out = v;
    return B2Q_OK;
}

b2q_status b2q_vision_destroy(b2q_vision* v) {
    delete v;
    return B2Q_OK;
}

b2q_status b2q_vision_set_tensor(b2q_vision* v, const char* name, int32_t ggml_type, const void* host_data,
                                 int64_t ne0, int64_t ne1, void* stream) {
    B2Q_REQUIRE_STATE();
    (void) ds;
    if (!v || !name || !host_data) return set_error(B2Q_ERR_INVALID, "null pointer");
    const std::string n(name);
    ++v->gen;
    B2Q_TRY(v->ts.put(n, ggml_type, host_data, ne0, ne1, false, static_cast<cudaStream_t>(stream)));
    if (n.rfind("v.head.", 0) == 0) v->probe_ready = false;
    return B2Q_OK;
}

b2q_status b2q_vision_reserve(b2q_vision* v, int64_t max_tokens, int32_t max_images) {
    B2Q_REQUIRE_STATE();
    (void) ds;
    if (!v || max_tokens <= 0 || max_images <= 0) return set_error(B2Q_ERR_INVALID, "bad reserve arguments");
    const int64_t T = max_tokens, H = v->cfg.hidden;
    const int64_t tiles = T / 64 + max_images;
    ++v->gen;
    B2Q_TRY(cuda_check(v->x.ensure(T * H * 4), "cudaMalloc(x)"));
    B2Q_TRY(cuda_check(v->pos.ensure(T * H * 4), "cudaMalloc(pos)"));
    B2Q_TRY(cuda_check(v->qkv16.ensure(T * 3 * H * 2), "cudaMalloc(qkv)"));
    B2Q_TRY(cuda_check(v->attn.ensure(T * H * 4), "cudaMalloc(attn)"));
    B2Q_TRY(cuda_check(v->act_h.ensure(b2q_act_bytes(T, H)), "cudaMalloc(act_h)"));
    B2Q_TRY(cuda_check(v->act_f.ensure(b2q_act_bytes(T, v->ffn_pad)), "cudaMalloc(act_f)"));
    B2Q_TRY(cuda_check(v->act_p.ensure(b2q_act_bytes(T, v->cfg.patch_dim)), "cudaMalloc(act_p)"));
    B2Q_TRY(cuda_check(v->imgs.ensure(static_cast<size_t>(max_images) * sizeof(ImageDesc)), "cudaMalloc(imgs)"));
    B2Q_TRY(cuda_check(v->tiles.ensure(attn_tiles_bytes(static_cast<int>(tiles))), "cudaMalloc(tiles)"));
    B2Q_TRY(cuda_check(v->head_tiles.ensure(attn_tiles_bytes(max_images)), "cudaMalloc(head tiles)"));
    B2Q_TRY(cuda_check(v->q16.ensure(H * 2), "cudaMalloc(q16)"));
    B2Q_TRY(cuda_check(v->ha.ensure(static_cast<size_t>(max_images) * H * 4), "cudaMalloc(head a)"));
    B2Q_TRY(cuda_check(v->ha2.ensure(static_cast<size_t>(max_images) * H * 4), "cudaMalloc(head a2)"));
    B2Q_TRY(cuda_check(v->patches_in.ensure(T * v->cfg.patch_dim * 4), "cudaMalloc(patches)"));
    B2Q_TRY(cuda_check(v->out_dev.ensure(static_cast<size_t>(max_images) * H * 4), "cudaMalloc(out)"));
    v->host_tiles.resize(attn_tiles_bytes(static_cast<int>(tiles)));
    v->host_head_tiles.resize(attn_tiles_bytes(max_images));
    v->tables_for.clear();   // device tables may have moved
    v->cap_tokens = T;
    v->cap_images = max_images;
    return B2Q_OK;
}

b2q_status b2q_vision_encode(b2q_vision* v, const float* patches, const int32_t* grid_hw, int32_t n_images,
                             int32_t pooling, float* out, void* stream) {
    B2Q_REQUIRE_STATE();
    (void) ds;
    if (!v || !patches || !grid_hw || !out) return set_error(B2Q_ERR_INVALID, "null pointer");
    if (n_images <= 0 || (pooling != B2Q_POOL_MEAN && pooling != B2Q_POOL_PROBE))
        return set_error(B2Q_ERR_INVALID, "bad n_images / pooling");
    B2Q_TRY(check_loaded(v));
    if (pooling == B2Q_POOL_PROBE) B2Q_TRY(check_head(v));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const b2q_vision_config& c = v->cfg;
    const int64_t H = c.hidden;

    // ---- batch geometry (host) ----
    std::vector<ImageDesc> imgs(n_images);
    std::vector<int> off(n_images), len(n_images), oidx(n_images), zero(n_images, 0), one(n_images, 1);
    int64_t T = 0;
    for (int i = 0; i < n_images; ++i) {
        const int h = grid_hw[2 * i], w = grid_hw[2 * i + 1];
        if (h <= 0 || w <= 0) return set_error(B2Q_ERR_SHAPE, "grid sides must be positive");
        imgs[i] = ImageDesc{static_cast<int>(T), h, w, 0};
        off[i] = static_cast<int>(T);
        len[i] = h * w;
        oidx[i] = i;
        T += h * w;
    }
    if (T > v->cap_tokens || n_images > v->cap_images)
        B2Q_TRY(b2q_vision_reserve(v, T > v->cap_tokens ? T : v->cap_tokens,
                                   n_images > v->cap_images ? n_images : v->cap_images));
    const bool same = v->tables_for.size() == static_cast<size_t>(2 * n_images) &&
                      std::memcmp(v->tables_for.data(), grid_hw, 2 * n_images * sizeof(int32_t)) == 0;
    if (!same) {
        v->n_tiles = attn_build_tiles(off.data(), len.data(), off.data(), len.data(), off.data(), n_images,
                                      v->host_tiles.data(),
                                      static_cast<int>(v->host_tiles.size() / attn_tiles_bytes(1)));
        v->n_htiles = attn_build_tiles(zero.data(), one.data(), off.data(), len.data(), oidx.data(), n_images,
                                       v->host_head_tiles.data(),
                                       static_cast<int>(v->host_head_tiles.size() / attn_tiles_bytes(1)));
        if (v->n_tiles < 0 || v->n_htiles < 0) {
            v->tables_for.clear();
            return set_error(B2Q_ERR_SHAPE, "attention tile table overflow");
        }
        B2Q_TRY(cuda_check(cudaMemcpyAsync(v->imgs.p, imgs.data(), n_images * sizeof(ImageDesc),
                                           cudaMemcpyHostToDevice, s),
                           "image table upload"));
        B2Q_TRY(cuda_check(cudaMemcpyAsync(v->tiles.p, v->host_tiles.data(), attn_tiles_bytes(v->n_tiles),
                                           cudaMemcpyHostToDevice, s),
                           "tile table upload"));
        B2Q_TRY(cuda_check(cudaMemcpyAsync(v->head_tiles.p, v->host_head_tiles.data(), attn_tiles_bytes(v->n_htiles),
                                           cudaMemcpyHostToDevice, s),
                           "head tile table upload"));
        // keep the host tables alive until the copies have been consumed
        B2Q_TRY(cuda_check(cudaStreamSynchronize(s), "table upload"));
        v->tables_for.assign(grid_hw, grid_hw + 2 * n_images);
    }
    const int n_tiles = v->n_tiles, n_htiles = v->n_htiles;

    if (pooling == B2Q_POOL_PROBE && !v->probe_ready) {
        // probe query q = probe . Wq + bq: one row shared by every image,
        // depends on weights only (src/siglip2_vision.cpp:259-265)
        B2Q_TRY(b2q_quantize_q8_1(v->f("v.head.probe"), 1, H, H, v->act_h.p, s));
        B2Q_TRY(gemm(v->w("v.head.attn_q.weight"), v->act_h.p, 1, v->q16.p, B2Q_EPI_BIAS_F16,
                     v->f("v.head.attn_q.bias"), nullptr, nullptr, 0, s));
        v->probe_ready = true;
    }

    // everything from here on is kernel launches only, so a repeated call
    // replays it as one CUDA graph (run_graphed)
    std::vector<int64_t> key = {static_cast<int64_t>(ds->tune_gen), static_cast<int64_t>(v->gen), n_images, pooling,
                                reinterpret_cast<int64_t>(patches), reinterpret_cast<int64_t>(out)};
    key.insert(key.end(), grid_hw, grid_hw + 2 * n_images);
    auto issue = [&](cudaStream_t s) -> b2q_status {
        float* x = v->x.as<float>();
        float* pos = v->pos.as<float>();
        __half* qkv = v->qkv16.as<__half>();
        float* att = v->attn.as<float>();

        // ---- stem: x = (patches . W + b) + pos  (src/siglip2_vision.cpp:676-691) ----
        {
            int max_tok = 1;
            for (int i = 0; i < n_images; ++i) max_tok = std::max(max_tok, grid_hw[2 * i] * grid_hw[2 * i + 1]);
            dim3 grid(static_cast<unsigned>((max_tok + kPosTok - 1) / kPosTok), static_cast<unsigned>(n_images));
            pos_resize_kernel<<<grid, 128, 0, s>>>(v->f("v.position_embd.weight"), c.pos_side, static_cast<int>(H),
                                                  v->imgs.as<ImageDesc>(), pos);
            count_launch();
            B2Q_TRY(cuda_check(cudaGetLastError(), "pos resize launch"));
        }
        B2Q_TRY(b2q_quantize_q8_1(patches, T, c.patch_dim, c.patch_dim, v->act_p.p, s));
        B2Q_TRY(gemm(v->w("v.patch_embd.weight"), v->act_p.p, T, x, B2Q_EPI_BIAS_RESIDUAL, v->f("v.patch_embd.bias"),
                     pos, nullptr, 0, s));

        // ---- encoder blocks ----
        B2Q_TRY(run_encoder_blocks(v->ts, "v.", c.n_layer, c.n_head, c.eps, T, H, x, qkv, att, v->act_h.p, v->act_f.p,
                                   v->tiles.p, n_tiles, false, s));

        // ---- post-LN (in place) and its q8_1 planes for the head ----
        B2Q_TRY(b2q_ln_quantize_q8_1(x, v->f("v.post_ln.weight"), v->f("v.post_ln.bias"), c.eps, T, H, v->act_h.p, x, s));

        if (pooling == B2Q_POOL_MEAN) {
            dim3 grid(static_cast<unsigned>((H + 127) / 128), static_cast<unsigned>(n_images));
            mean_pool_kernel<<<grid, 128, 0, s>>>(x, static_cast<int>(H), v->imgs.as<ImageDesc>(), out);
            count_launch();
            return cuda_check(cudaGetLastError(), "mean pool launch");
        }

        // ---- attention-pool head ----
        // K and V of every token: one [T][2H] fp16 block in the qkv buffer
        B2Q_TRY(gemm(v->w("v.head.attn_k.weight"), v->act_h.p, T, qkv, B2Q_EPI_BIAS_F16, v->f("v.head.attn_k.bias"),
                     nullptr, nullptr, 2 * H, s));
        B2Q_TRY(gemm(v->w("v.head.attn_v.weight"), v->act_h.p, T, qkv + H, B2Q_EPI_BIAS_F16, v->f("v.head.attn_v.bias"),
                     nullptr, nullptr, 2 * H, s));
        float* a = v->ha.as<float>();
        float* a2 = v->ha2.as<float>();
        B2Q_TRY(cuda_check(launch_attention(v->q16.as<__half>(), 0, qkv, 2 * H, qkv + H, 2 * H, v->head_tiles.p,
                                            n_htiles, c.n_head, a, H, s),
                           "head attention launch"));
        // attn = o_proj(a) + b; out = attn + (fc2(gelu(fc1(LN(attn)))) + b)
        B2Q_TRY(b2q_quantize_q8_1(a, n_images, H, H, v->act_h.p, s));
        B2Q_TRY(gemm(v->w("v.head.attn_o.weight"), v->act_h.p, n_images, a2, B2Q_EPI_BIAS, v->f("v.head.attn_o.bias"),
                     nullptr, nullptr, 0, s));
        B2Q_TRY(b2q_ln_quantize_q8_1(a2, v->f("v.head.ln.weight"), v->f("v.head.ln.bias"), c.eps, n_images, H,
                                     v->act_h.p, nullptr, s));
        B2Q_TRY(gemm(v->w("v.head.ffn_up.weight"), v->act_h.p, n_images, nullptr, B2Q_EPI_BIAS_GELU_Q8,
                     v->f("v.head.ffn_up.bias"), nullptr, v->act_f.p, 0, s));
        B2Q_TRY(gemm(v->w("v.head.ffn_down.weight"), v->act_f.p, n_images, out, B2Q_EPI_BIAS_RESIDUAL,
                     v->f("v.head.ffn_down.bias"), a2, nullptr, 0, s));
        return B2Q_OK;
    };
    return run_graphed(v->graph, key, s, issue);
}

b2q_status b2q_vision_encode_host(b2q_vision* v, const float* patches_host, const int32_t* grid_hw, int32_t n_images,
                                  int32_t pooling, float* out_host, void* stream) {
    B2Q_REQUIRE_STATE();
    (void) ds;
    if (!v || !patches_host || !grid_hw || !out_host) return set_error(B2Q_ERR_INVALID, "null pointer");
    int64_t T = 0;
    for (int i = 0; i < n_images; ++i) T += static_cast<int64_t>(grid_hw[2 * i]) * grid_hw[2 * i + 1];
    if (T <= 0) return set_error(B2Q_ERR_SHAPE, "empty batch");
    if (T > v->cap_tokens || n_images > v->cap_images)
        B2Q_TRY(b2q_vision_reserve(v, T > v->cap_tokens ? T : v->cap_tokens,
                                   n_images > v->cap_images ? n_images : v->cap_images));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    B2Q_TRY(cuda_check(cudaMemcpyAsync(v->patches_in.p, patches_host, static_cast<size_t>(T) * v->cfg.patch_dim * 4,
                                       cudaMemcpyHostToDevice, s),
                       "patch upload"));
    B2Q_TRY(b2q_vision_encode(v, v->patches_in.as<float>(), grid_hw, n_images, pooling, v->out_dev.as<float>(), stream));
    B2Q_TRY(cuda_check(cudaMemcpyAsync(out_host, v->out_dev.p, static_cast<size_t>(n_images) * v->cfg.hidden * 4,
                                       cudaMemcpyDeviceToHost, s),
                       "embedding download"));
    return cuda_check(cudaStreamSynchronize(s), "encode");
}

b2q_status b2q_vision_submit_host(b2q_vision* v, const float* patches_host, const int32_t* grid_hw, int32_t n_images,
                                  int32_t pooling, float* out_host, void* stream) {
    B2Q_REQUIRE_STATE();
    (void) ds;
    if (!v || !patches_host || !grid_hw || !out_host) return set_error(B2Q_ERR_INVALID, "null pointer");
    if (n_images <= 0) return set_error(B2Q_ERR_INVALID, "n_images must be positive");
    int64_t T = 0;
    for (int i = 0; i < n_images; ++i) T += static_cast<int64_t>(grid_hw[2 * i]) * grid_hw[2 * i + 1];
    if (T <= 0) return set_error(B2Q_ERR_SHAPE, "empty batch");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!v->copy_stream) {
        B2Q_TRY(cuda_check(cudaStreamCreateWithFlags(&v->copy_stream, cudaStreamNonBlocking), "copy stream"));
        for (int k = 0; k < 2; ++k) {
            B2Q_TRY(cuda_check(cudaEventCreateWithFlags(&v->landed[k], cudaEventDisableTiming), "event"));
            B2Q_TRY(cuda_check(cudaEventCreateWithFlags(&v->done[k], cudaEventDisableTiming), "event"));
            B2Q_TRY(cuda_check(cudaEventCreateWithFlags(&v->fetched[k], cudaEventDisableTiming), "event"));
        }
    }
    const int k = v->next_slot;
    const size_t in_bytes = static_cast<size_t>(T) * v->cfg.patch_dim * 4;
    const size_t out_bytes = static_cast<size_t>(n_images) * v->cfg.hidden * 4;
    if (in_bytes > v->slot_in[k].n || out_bytes > v->slot_out[k].n) {
        // growing a slot frees it: its previous encode must have finished
        if (v->slot_busy[k]) B2Q_TRY(cuda_check(cudaEventSynchronize(v->done[k]), "slot reuse"));
        B2Q_TRY(cuda_check(v->slot_in[k].ensure(in_bytes), "cudaMalloc(patch slot)"));
        B2Q_TRY(cuda_check(v->slot_out[k].ensure(out_bytes), "cudaMalloc(output slot)"));
    }
    // the upload may start once the encode that last read this slot is done;
    // it overlaps the encode of the other slot
    if (v->slot_busy[k]) B2Q_TRY(cuda_check(cudaStreamWaitEvent(v->copy_stream, v->done[k], 0), "slot wait"));
    B2Q_TRY(cuda_check(cudaMemcpyAsync(v->slot_in[k].p, patches_host, in_bytes, cudaMemcpyHostToDevice, v->copy_stream),
                       "patch upload"));
    B2Q_TRY(cuda_check(cudaEventRecord(v->landed[k], v->copy_stream), "event record"));
    B2Q_TRY(cuda_check(cudaStreamWaitEvent(s, v->landed[k], 0), "upload wait"));
    B2Q_TRY(b2q_vision_encode(v, v->slot_in[k].as<float>(), grid_hw, n_images, pooling, v->slot_out[k].as<float>(),
                              stream));
    B2Q_TRY(cuda_check(cudaEventRecord(v->done[k], s), "event record"));
    B2Q_TRY(cuda_check(cudaMemcpyAsync(out_host, v->slot_out[k].p, out_bytes, cudaMemcpyDeviceToHost, s),
                       "embedding download"));
    B2Q_TRY(cuda_check(cudaEventRecord(v->fetched[k], s), "event record"));
    v->slot_busy[k] = true;
    v->next_slot = k ^ 1;
    return B2Q_OK;
}

b2q_status b2q_vision_wait_submitted(b2q_vision* v, int32_t back) {
    B2Q_REQUIRE_STATE();
    (void) ds;
    if (!v) return set_error(B2Q_ERR_INVALID, "null pointer");
    if (back != 0 && back != 1) return set_error(B2Q_ERR_INVALID, "back must be 0 (latest) or 1 (the one before)");
    const int k = back == 0 ? (v->next_slot ^ 1) : v->next_slot;   // next_slot is the older of the two
    if (!v->slot_busy[k]) return set_error(B2Q_ERR_INVALID, "no such submission");
    return cuda_check(cudaEventSynchronize(v->fetched[k]), "submission wait");
}

b2q_status b2q_vision_wait(b2q_vision* v, void* stream) {
    B2Q_REQUIRE_STATE();
    (void) ds;
    if (!v) return set_error(B2Q_ERR_INVALID, "null pointer");
    return cuda_check(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "encode wait");
}

}  // extern "C"
