// b2q_capi.cu — the extern "C" boundary (include/b2q.h): argument checks,
// status codes, per-thread error text, per-device state, weight registry.
#include "b2q_internal.h"

#include <cudaTypedefs.h>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

namespace b2q {

bool make_weight_maps(b2q_weight* w);   // b2q_gemm.cu

namespace {
thread_local std::string t_last_error;
DeviceState g_states[64];
std::mutex g_init_mutex;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::atomic<uint64_t> g_launches{0};
}  // namespace

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
void add_launches(int64_t n) { g_launches.fetch_add(static_cast<uint64_t>(n), std::memory_order_relaxed); }
std::atomic<uint64_t> g_graph_launches{0};
void count_graph_launch() { g_graph_launches.fetch_add(1, std::memory_order_relaxed); }
uint64_t launches_now() { return g_launches.load(std::memory_order_relaxed); }

b2q_status set_error(b2q_status st, const std::string& msg) {
    t_last_error = msg;
    return st;
}

b2q_status cuda_check(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return B2Q_OK;
    return set_error(B2Q_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

DeviceState* state() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    DeviceState* s = &g_states[dev];
    return s->device == dev ? s : nullptr;
}

bool make_tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                  uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
    if (!g_encode) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t es[2] = {1, 1};
    CUresult r = g_encode(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

static bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace b2q

using namespace b2q;


extern "C" {

const char* b2q_last_error(void) { return t_last_error.c_str(); }

int b2q_abi_version(void) { return 1; }

uint64_t b2q_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }
uint64_t b2q_graph_launch_count(void) { return g_graph_launches.load(std::memory_order_relaxed); }

b2q_status b2q_init(int device, int ops_mode) {
    if (device < 0 || device >= 64) return set_error(B2Q_ERR_INVALID, "device index out of range");
    if (ops_mode != -1 && ops_mode != B2Q_OPS_I8 && ops_mode != B2Q_OPS_F16)
        return set_error(B2Q_ERR_INVALID, "unknown operand mode");
    std::lock_guard<std::mutex> lk(g_init_mutex);
    b2q_status st = cuda_check(cudaSetDevice(device), "cudaSetDevice");
    if (st) return st;
    DeviceState* s = &g_states[device];
    if (s->device != device) {
        cudaDeviceProp prop;
        if ((st = cuda_check(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties"))) return st;
        if (prop.major != 10) {
            return set_error(B2Q_ERR_CUDA, "this library is built for sm_100a (B200); device " +
                                               std::string(prop.name) + " has compute capability " +
                                               std::to_string(prop.major) + "." + std::to_string(prop.minor));
        }
        if (!g_encode) {
            void* fn = nullptr;
            cudaDriverEntryPointQueryResult q;
            if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
                q != cudaDriverEntryPointSuccess || !fn)
                return set_error(B2Q_ERR_CUDA, "driver entry point cuTensorMapEncodeTiled not found");
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
        }
        uint32_t* err = nullptr;
        if ((st = cuda_check(cudaMalloc(&err, 256), "cudaMalloc(error word)"))) return B2Q_ERR_NOMEM;
        if ((st = cuda_check(cudaMemset(err, 0, 256), "cudaMemset(error word)"))) return st;
        s->err = err;
        s->num_sms = prop.multiProcessorCount;
        s->device = device;
    }
    if (ops_mode != -1) s->mode = ops_mode;
    return B2Q_OK;
}

b2q_status b2q_tune(int key, int64_t value) {
    B2Q_REQUIRE_STATE();
    ++ds->tune_gen;   // graphs captured under the old settings are not replayed
    switch (key) {
        case B2Q_TUNE_GEMM_BN:
            if (value != 0 && value != 64 && value != 128 && value != 192 && value != 256)
                return set_error(B2Q_ERR_INVALID, "GEMM tile width must be 0, 64, 128, 192 or 256");
            ds->gemm_bn = static_cast<int>(value);
            return B2Q_OK;
        case B2Q_TUNE_TIMEOUT_NS:
            if (value < 1000000 || value > 60000000000ll) return set_error(B2Q_ERR_INVALID, "timeout must be in [1 ms, 60 s]");
            ds->timeout_ns = static_cast<uint64_t>(value);
            return B2Q_OK;
        case B2Q_TUNE_ATTN_EXACT:
            ds->attn_exact = value ? 1 : 0;
            return B2Q_OK;
        case B2Q_TUNE_TEST_STALL:
            ds->test_stall = value ? 1 : 0;
            return B2Q_OK;
        case B2Q_TUNE_ATTN_KERNEL:
            if (value != 0 && value != 1) return set_error(B2Q_ERR_INVALID, "attention kernel must be 0 or 1");
            ds->attn_kernel = static_cast<int>(value);
            return B2Q_OK;
        case B2Q_TUNE_GEMM_CTAS:
            if (value != 0 && value != 1 && value != 2) return set_error(B2Q_ERR_INVALID, "GEMM CTAs per SM must be 0, 1 or 2");
            ds->gemm_ctas = static_cast<int>(value);
            return B2Q_OK;
        case B2Q_TUNE_GRAPHS:
            ds->graphs = value ? 1 : 0;
            return B2Q_OK;
        default:
            return set_error(B2Q_ERR_INVALID, "unknown tuning key");
    }
}

b2q_status b2q_check_device(void* stream, uint32_t* code_out) {
    B2Q_REQUIRE_STATE();
    b2q_status st = cuda_check(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "cudaStreamSynchronize");
    if (st) return st;
    uint32_t code = 0;
    if ((st = cuda_check(cudaMemcpy(&code, ds->err, 4, cudaMemcpyDeviceToHost), "read device error word"))) return st;
    if (code) cudaMemset(ds->err, 0, 4);
    if (code_out) *code_out = code;
    if (code == 5u)   // kDevBadTokenId
        return set_error(B2Q_ERR_DEVICE, "a token id outside the vocabulary (code 5)");
    if (code) return set_error(B2Q_ERR_DEVICE, "a kernel's bounded wait expired (code " + std::to_string(code) + ")");
    return B2Q_OK;
}

// ---------------------------------------------------------------- weights
b2q_status b2q_weight_register(const void* q8_0, int64_t N, int64_t K, int64_t row_bytes, int src_is_host,
                               void* stream, b2q_weight** out) {
    B2Q_REQUIRE_STATE();
    if (!q8_0 || !out) return set_error(B2Q_ERR_INVALID, "null pointer");
    if (N <= 0 || K <= 0 || K % 32 != 0) return set_error(B2Q_ERR_SHAPE, "Q8_0 weight needs N > 0 and K % 32 == 0");
    if (N % 4 != 0) return set_error(B2Q_ERR_SHAPE, "N must be a multiple of 4 (16-byte scale rows)");
    if (K > 8192) return set_error(B2Q_ERR_SHAPE, "K above 8192 is not supported");
    const int64_t Kb = K / 32;
    if (row_bytes < Kb * 34) return set_error(B2Q_ERR_SHAPE, "row_bytes smaller than K/32*34");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    b2q_weight* w = new b2q_weight();
    w->N = N;
    w->K = K;
    w->Kb = Kb;
    w->Nd = (N + 63) / 64 * 64;
    w->mode = ds->mode;
    w->device = ds->device;
    const int es = ops_elem_bytes(w->mode);
    void* src = const_cast<void*>(q8_0);
    void* staged = nullptr;
    b2q_status st = B2Q_OK;
    if (cudaMalloc(&w->q, static_cast<size_t>(N * K * es)) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&w->d), static_cast<size_t>(Kb * w->Nd * 4)) != cudaSuccess) {
        st = set_error(B2Q_ERR_NOMEM, "cudaMalloc of weight planes failed");
        goto fail;
    }
    // scale slots of columns N..Nd-1 stay zero: those columns are computed (as 0) but never stored
    if ((st = cuda_check(cudaMemsetAsync(w->d, 0, static_cast<size_t>(Kb * w->Nd * 4), s), "weight scale clear")))
        goto fail;
    if (src_is_host) {
        if (cudaMalloc(&staged, static_cast<size_t>(N * row_bytes)) != cudaSuccess) {
            st = set_error(B2Q_ERR_NOMEM, "cudaMalloc of weight staging failed");
            goto fail;
        }
        if ((st = cuda_check(cudaMemcpyAsync(staged, q8_0, static_cast<size_t>(N * row_bytes), cudaMemcpyHostToDevice, s),
                             "weight upload")))
            goto fail;
        src = staged;
    }
    if ((st = cuda_check(launch_repack_q8_0(src, N, Kb, row_bytes, w->Nd, w->mode, w->q, w->d, s), "repack launch")))
        goto fail;
    if (staged) {
        if ((st = cuda_check(cudaStreamSynchronize(s), "weight repack"))) goto fail;
        cudaFree(staged);
        staged = nullptr;
    }
    if (!make_weight_maps(w)) {
        st = set_error(B2Q_ERR_CUDA, "cuTensorMapEncodeTiled failed for the weight planes");
        goto fail;
    }
    *out = w;
    return B2Q_OK;
fail:
    if (staged) cudaFree(staged);
    if (w->q) cudaFree(w->q);
    if (w->d) cudaFree(w->d);
    delete w;
    return st;
}

b2q_status b2q_weight_release(b2q_weight* w) {
    if (!w) return B2Q_OK;
    cudaFree(w->q);
    cudaFree(w->d);
    delete w;
    return B2Q_OK;
}

b2q_status b2q_weight_shape(const b2q_weight* w, int64_t* N, int64_t* K) {
    if (!w) return set_error(B2Q_ERR_INVALID, "null weight");
    if (N) *N = w->N;
    if (K) *K = w->K;
    return B2Q_OK;
}

// ---------------------------------------------------------------- activations
size_t b2q_act_bytes(int64_t M, int64_t K) {
    DeviceState* ds = state();
    const int mode = ds ? ds->mode : kOpsF16;
    if (M <= 0 || K <= 0) return 0;
    return act_layout(M, K, mode).bytes;
}

b2q_status b2q_act_layout(int64_t M, int64_t K, int64_t* Kp, int64_t* value_bytes, int64_t* scale_offset,
                          int64_t* scale_ld) {
    B2Q_REQUIRE_STATE();
    if (M <= 0 || K <= 0) return set_error(B2Q_ERR_SHAPE, "M and K must be positive");
    const ActLayout L = act_layout(M, K, ds->mode);
    if (Kp) *Kp = L.Kp;
    if (value_bytes) *value_bytes = L.es;
    if (scale_offset) *scale_offset = static_cast<int64_t>(L.d_offset);
    if (scale_ld) *scale_ld = L.ld;
    return B2Q_OK;
}

b2q_status b2q_quantize_q8_1(const float* x, int64_t M, int64_t K, int64_t ldx, void* act, void* stream) {
    B2Q_REQUIRE_STATE();
    if (!x || !act) return set_error(B2Q_ERR_INVALID, "null pointer");
    if (M <= 0 || K <= 0 || ldx < K) return set_error(B2Q_ERR_SHAPE, "bad M/K/ldx");
    if (round_up(K, 32) > 5120) return set_error(B2Q_ERR_SHAPE, "K above 5120 is not supported by the quantizer");
    if (!aligned(act, 256)) return set_error(B2Q_ERR_ALIGN, "activation buffer must be 256-byte aligned");
    return cuda_check(launch_quantize_q8_1(x, M, K, ldx, act, ds->mode, static_cast<cudaStream_t>(stream)),
                      "quantize launch");
}

b2q_status b2q_ln_quantize_q8_1(const float* x, const float* w, const float* b, float eps, int64_t M, int64_t H,
                                void* act, float* y_opt, void* stream) {
    B2Q_REQUIRE_STATE();
    if (!x || !w || !b || !act) return set_error(B2Q_ERR_INVALID, "null pointer");
    if (M <= 0 || H <= 0 || H % 128 != 0 || (H / 128 != 1 && H / 128 != 2 && H / 128 != 9))
        return set_error(B2Q_ERR_SHAPE, "LayerNorm width must be 128, 256 or 1152");
    if (!aligned(x, 16) || !aligned(w, 16) || !aligned(b, 16) || (y_opt && !aligned(y_opt, 16)))
        return set_error(B2Q_ERR_ALIGN, "LayerNorm rows need 16-byte alignment");
    if (!aligned(act, 256)) return set_error(B2Q_ERR_ALIGN, "activation buffer must be 256-byte aligned");
    return cuda_check(launch_ln_quant(x, w, b, eps, M, H, act, y_opt, ds->mode, static_cast<cudaStream_t>(stream)),
                      "layernorm launch");
}

// ---------------------------------------------------------------- GEMM
static b2q_status check_gemm(DeviceState* ds, const b2q_weight* w, const void* act, int64_t M) {
    if (!w || !act) return set_error(B2Q_ERR_INVALID, "null pointer");
    if (w->device != ds->device) return set_error(B2Q_ERR_INVALID, "weight registered on another device");
    if (w->mode != ds->mode) return set_error(B2Q_ERR_INVALID, "weight registered under another operand mode");
    if (M <= 0 || M > (1 << 30)) return set_error(B2Q_ERR_SHAPE, "bad M");
    if (!aligned(act, 256)) return set_error(B2Q_ERR_ALIGN, "activation buffer must be 256-byte aligned");
    return B2Q_OK;
}

b2q_status b2q_mul_mat_q8_0(const b2q_weight* w, const void* act, int64_t M, void* y, const b2q_epilogue* epi,
                            void* stream) {
    B2Q_REQUIRE_STATE();
    b2q_status st = check_gemm(ds, w, act, M);
    if (st) return st;
    GemmArgs a{};
    a.w = w;
    a.act = act;
    a.M = M;
    a.epi = epi ? epi->kind : B2Q_EPI_NONE;
    a.bias = epi ? epi->bias : nullptr;
    a.residual = epi ? epi->residual : nullptr;
    a.act_out = epi ? epi->act_out : nullptr;
    a.ld_out = epi ? epi->ld_out : 0;
    a.out = y;
    if (a.epi < B2Q_EPI_NONE || a.epi > B2Q_EPI_BIAS_F16) return set_error(B2Q_ERR_INVALID, "unknown epilogue");
    if (a.epi == B2Q_EPI_BIAS_GELU_Q8) {
        if (!a.act_out || !aligned(a.act_out, 256))
            return set_error(B2Q_ERR_ALIGN, "GELU_Q8 needs a 256-byte aligned act_out");
    } else {
        if (!y || !aligned(y, 16)) return set_error(B2Q_ERR_ALIGN, "output must be non-null and 16-byte aligned");
        const int64_t ld = a.ld_out > 0 ? a.ld_out : w->N;
        if (ld < w->N || ld % 4) return set_error(B2Q_ERR_SHAPE, "ld_out must be >= N and a multiple of 4");
    }
    if (a.bias && !aligned(a.bias, 16)) return set_error(B2Q_ERR_ALIGN, "bias must be 16-byte aligned");
    if (a.epi == B2Q_EPI_BIAS_RESIDUAL && (!a.residual || !aligned(a.residual, 16)))
        return set_error(B2Q_ERR_ALIGN, "residual must be non-null and 16-byte aligned");
    return launch_gemm(a, static_cast<cudaStream_t>(stream));
}

b2q_status b2q_mul_mat_q8_0_f32(const b2q_weight* w, const float* x, int64_t M, int64_t x_cols, float* y,
                                void* act_scratch, void* stream) {
    B2Q_REQUIRE_STATE();
    b2q_status st = check_gemm(ds, w, act_scratch, M);
    if (st) return st;
    if (!x || !y) return set_error(B2Q_ERR_INVALID, "null pointer");
    if (x_cols <= 0 || x_cols > w->K) return set_error(B2Q_ERR_SHAPE, "x_cols must be in (0, K]");
    if (!aligned(y, 16)) return set_error(B2Q_ERR_ALIGN, "y must be 16-byte aligned");
    if (round_up(x_cols, 32) != w->K)
        return set_error(B2Q_ERR_SHAPE, "x_cols must round up to the weight's K (K-padding is at most 31 columns)");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // the quantizer zero-fills columns x_cols..K-1 (pad_x_to_w)
    if ((st = cuda_check(launch_quantize_q8_1(x, M, x_cols, x_cols, act_scratch, ds->mode, s), "quantize launch")))
        return st;
    GemmArgs a{};
    a.w = w;
    a.act = act_scratch;
    a.M = M;
    a.epi = B2Q_EPI_NONE;
    a.out = y;
    return launch_gemm(a, s);
}

b2q_status b2q_block_sums(const b2q_weight* w, const void* act, int64_t M, int32_t* sums, void* stream) {
    B2Q_REQUIRE_STATE();
    b2q_status st = check_gemm(ds, w, act, M);
    if (st) return st;
    if (!sums) return set_error(B2Q_ERR_INVALID, "null pointer");
    GemmArgs a{};
    a.w = w;
    a.act = act;
    a.M = M;
    a.epi = B2Q_EPI_NONE;
    a.dump = sums;
    return launch_gemm(a, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------- attention
size_t b2q_attention_scratch_bytes(const int32_t* q_len, int32_t n_seq) {
    if (!q_len || n_seq <= 0) return 0;
    int64_t tiles = 0;
    for (int32_t s = 0; s < n_seq; ++s) tiles += (q_len[s] + 127) / 128;
    return attn_tiles_bytes(static_cast<int>(tiles));
}

b2q_status b2q_attention(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                         const int32_t* q_off, const int32_t* q_len, const int32_t* k_off, const int32_t* k_len,
                         const int32_t* o_off, int32_t n_seq, int32_t n_head, int32_t d_head, float* out, int64_t ldo,
                         void* tiles_scratch, void* stream) {
    B2Q_REQUIRE_STATE();
    (void) ds;
    if (!q || !k || !v || !out || !q_off || !q_len || !k_off || !k_len || !o_off || !tiles_scratch)
        return set_error(B2Q_ERR_INVALID, "null pointer");
    if (d_head != 72) return set_error(B2Q_ERR_SHAPE, "only head_dim 72 is implemented");
    if (n_seq <= 0 || n_head <= 0 || n_head > 65535) return set_error(B2Q_ERR_SHAPE, "bad n_seq / n_head");
    if (ldq % 8 || ldk % 8 || ldv % 8 || ldo % 2 || !aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) ||
        !aligned(out, 8))
        return set_error(B2Q_ERR_ALIGN, "attention rows need 16-byte aligned fp16 rows and 8-byte aligned output");
    for (int32_t s = 0; s < n_seq; ++s)
        if (q_len[s] < 0 || k_len[s] <= 0 || q_off[s] < 0 || k_off[s] < 0 || o_off[s] < 0)
            return set_error(B2Q_ERR_SHAPE, "every sequence needs at least one key");
    const size_t bytes = b2q_attention_scratch_bytes(q_len, n_seq);
    std::string host(bytes, '\0');
    const int n = attn_build_tiles(q_off, q_len, k_off, k_len, o_off, n_seq, host.data(),
                                   static_cast<int>(bytes / attn_tiles_bytes(1)));
    if (n < 0) return set_error(B2Q_ERR_SHAPE, "tile table overflow");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    b2q_status st = cuda_check(cudaMemcpyAsync(tiles_scratch, host.data(), bytes, cudaMemcpyHostToDevice, s),
                               "attention tile upload");
    if (st) return st;
    return cuda_check(launch_attention(static_cast<const __half*>(q), ldq, static_cast<const __half*>(k), ldk,
                                       static_cast<const __half*>(v), ldv, tiles_scratch, n, n_head, out, ldo, s),
                      "attention launch");
}

}  // extern "C"
