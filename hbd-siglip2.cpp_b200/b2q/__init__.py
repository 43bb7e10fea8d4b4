"""Python binding of libb2q.so (include/b2q.h) — the host side used by tests
and benchmarks.  Device buffers are torch CUDA tensors (torch is plumbing
here: memory, streams, process groups); every computation goes through the
C ABI.  There is no fallback: if the library is missing this module raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parents[1]
LIB_PATH = PKG / "lib" / "libb2q.so"

OK = 0
ERR_INVALID, ERR_SHAPE, ERR_ALIGN, ERR_CUDA, ERR_DEVICE, ERR_NOT_INIT, ERR_NOMEM = -1, -2, -3, -4, -5, -6, -7
OPS_I8, OPS_F16 = 0, 1
EPI_NONE, EPI_BIAS, EPI_BIAS_RESIDUAL, EPI_BIAS_GELU_Q8, EPI_BIAS_F16 = 0, 1, 2, 3, 4

#: every symbol include/b2q.h declares (checked by the CPU test suite)
EXPORTS = [
    "b2q_last_error", "b2q_abi_version", "b2q_launch_count", "b2q_graph_launch_count", "b2q_init", "b2q_tune", "b2q_check_device",
    "b2q_weight_register", "b2q_weight_release", "b2q_weight_shape",
    "b2q_act_bytes", "b2q_act_layout", "b2q_quantize_q8_1", "b2q_ln_quantize_q8_1",
    "b2q_mul_mat_q8_0", "b2q_mul_mat_q8_0_f32", "b2q_mul_mat_q8_0_f32_noalloc", "b2q_block_sums",
    "b2q_attention_scratch_bytes", "b2q_attention",
    "b2q_vision_create", "b2q_vision_destroy", "b2q_vision_set_tensor", "b2q_vision_reserve",
    "b2q_vision_encode", "b2q_vision_encode_host", "b2q_vision_submit_host", "b2q_vision_wait",
    "b2q_vision_wait_submitted",
    "b2q_text_create", "b2q_text_destroy", "b2q_text_set_tensor", "b2q_text_reserve", "b2q_text_encode",
    "b2q_text_encode_host", "b2q_score_scratch_bytes", "b2q_score",
    "b2q_gguf_open", "b2q_gguf_close", "b2q_gguf_n_tensors", "b2q_gguf_tensor", "b2q_gguf_scalar_f32",
    "b2q_vision_load_gguf", "b2q_text_load_gguf",
]


class B2QError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"b2q status {status}: {msg}")
        self.status = status


class VisionConfig(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("ffn", C.c_int32), ("n_head", C.c_int32), ("n_layer", C.c_int32),
                ("patch_dim", C.c_int32), ("pos_side", C.c_int32), ("eps", C.c_float)]


class TextConfig(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("ffn", C.c_int32), ("n_head", C.c_int32), ("n_layer", C.c_int32),
                ("vocab", C.c_int32), ("n_pos", C.c_int32), ("eps", C.c_float)]


POOL_MEAN, POOL_PROBE = 0, 1
GGML_F32, GGML_Q8_0 = 0, 8


class Epilogue(C.Structure):
    _fields_ = [("kind", C.c_int), ("bias", C.c_void_p), ("residual", C.c_void_p),
                ("act_out", C.c_void_p), ("ld_out", C.c_int64)]


_lib = None
P, I64 = C.c_void_p, C.c_int64
I32P = C.POINTER(C.c_int32)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run __graft_entry__.build() (no CPU fallback exists)")
        L = C.CDLL(str(LIB_PATH))
        L.b2q_last_error.restype = C.c_char_p
        L.b2q_abi_version.restype = C.c_int
        L.b2q_launch_count.restype = C.c_uint64
        L.b2q_graph_launch_count.restype = C.c_uint64
        L.b2q_init.argtypes = [C.c_int, C.c_int]
        L.b2q_check_device.argtypes = [P, C.POINTER(C.c_uint32)]
        L.b2q_tune.argtypes = [C.c_int, I64]
        L.b2q_weight_register.argtypes = [P, I64, I64, I64, C.c_int, P, C.POINTER(P)]
        L.b2q_weight_release.argtypes = [P]
        L.b2q_weight_shape.argtypes = [P, C.POINTER(I64), C.POINTER(I64)]
        L.b2q_act_bytes.argtypes = [I64, I64]
        L.b2q_act_bytes.restype = C.c_size_t
        L.b2q_act_layout.argtypes = [I64, I64] + [C.POINTER(I64)] * 4
        L.b2q_quantize_q8_1.argtypes = [P, I64, I64, I64, P, P]
        L.b2q_ln_quantize_q8_1.argtypes = [P, P, P, C.c_float, I64, I64, P, P, P]
        L.b2q_mul_mat_q8_0.argtypes = [P, P, I64, P, C.POINTER(Epilogue), P]
        L.b2q_mul_mat_q8_0_f32.argtypes = [P, P, I64, I64, P, P, P]
        L.b2q_mul_mat_q8_0_f32_noalloc.argtypes = [P, P, I64, I64, P, P]
        L.b2q_block_sums.argtypes = [P, P, I64, P, P]
        L.b2q_attention_scratch_bytes.argtypes = [I32P, C.c_int32]
        L.b2q_attention_scratch_bytes.restype = C.c_size_t
        L.b2q_attention.argtypes = [P, I64, P, I64, P, I64, I32P, I32P, I32P, I32P, I32P, C.c_int32, C.c_int32,
                                    C.c_int32, P, I64, P, P]
        L.b2q_vision_create.argtypes = [C.POINTER(VisionConfig), C.POINTER(P)]
        L.b2q_vision_destroy.argtypes = [P]
        L.b2q_vision_set_tensor.argtypes = [P, C.c_char_p, C.c_int32, P, I64, I64, P]
        L.b2q_vision_reserve.argtypes = [P, I64, C.c_int32]
        L.b2q_vision_encode.argtypes = [P, P, I32P, C.c_int32, C.c_int32, P, P]
        L.b2q_vision_encode_host.argtypes = [P, P, I32P, C.c_int32, C.c_int32, P, P]
        L.b2q_vision_submit_host.argtypes = [P, P, I32P, C.c_int32, C.c_int32, P, P]
        L.b2q_vision_wait.argtypes = [P, P]
        L.b2q_vision_wait_submitted.argtypes = [P, C.c_int32]
        L.b2q_text_create.argtypes = [C.POINTER(TextConfig), C.POINTER(P)]
        L.b2q_text_destroy.argtypes = [P]
        L.b2q_text_set_tensor.argtypes = [P, C.c_char_p, C.c_int32, P, I64, I64, P]
        L.b2q_text_reserve.argtypes = [P, C.c_int32]
        L.b2q_text_encode.argtypes = [P, P, C.c_int32, P, P]
        L.b2q_text_encode_host.argtypes = [P, P, C.c_int32, P, P]
        L.b2q_score_scratch_bytes.argtypes = [C.c_int32, C.c_int32, C.c_int32]
        L.b2q_score_scratch_bytes.restype = C.c_size_t
        L.b2q_score.argtypes = [P, C.c_int32, P, C.c_int32, C.c_int32, C.c_float, C.c_float, P, P, P, P]
        L.b2q_gguf_open.argtypes = [C.c_char_p, C.POINTER(P)]
        L.b2q_gguf_close.argtypes = [P]
        L.b2q_gguf_n_tensors.argtypes = [P]
        L.b2q_gguf_n_tensors.restype = I64
        L.b2q_gguf_tensor.argtypes = [P, I64, C.POINTER(C.c_char_p), C.POINTER(C.c_int32), C.POINTER(C.c_int32),
                                      C.POINTER(I64), C.POINTER(P)]
        L.b2q_gguf_scalar_f32.argtypes = [P, C.c_char_p, C.POINTER(C.c_float)]
        L.b2q_vision_load_gguf.argtypes = [P, P, P]
        L.b2q_text_load_gguf.argtypes = [P, P, P]
        for name in EXPORTS:
            fn = getattr(L, name)
            if name not in ("b2q_last_error", "b2q_abi_version", "b2q_act_bytes", "b2q_attention_scratch_bytes",
                            "b2q_launch_count", "b2q_graph_launch_count"):
                fn.restype = C.c_int
        _lib = L
    return _lib


def launch_count() -> int:
    return int(lib().b2q_launch_count())


def graph_launch_count() -> int:
    """Tower encodes the library launched as one captured CUDA graph."""
    return int(lib().b2q_graph_launch_count())


def check(status: int):
    if status != OK:
        raise B2QError(status, lib().b2q_last_error().decode())


def _ptr(t) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


def _host_ptr(a):
    """Address of a host buffer: a torch CPU tensor or a numpy array."""
    return a.data_ptr() if hasattr(a, "data_ptr") else a.ctypes.data


def _stream(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def init(device: int = 0, ops_mode: int = -1):
    check(lib().b2q_init(device, ops_mode))


TUNE_GEMM_BN, TUNE_TIMEOUT_NS, TUNE_ATTN_EXACT, TUNE_TEST_STALL, TUNE_ATTN_KERNEL, TUNE_GEMM_CTAS = 1, 2, 3, 4, 5, 6
TUNE_GRAPHS = 7


def tune(key: int, value: int):
    check(lib().b2q_tune(key, value))


def check_device(stream=None) -> int:
    code = C.c_uint32(0)
    check(lib().b2q_check_device(_stream(stream), C.byref(code)))
    return code.value


class Weight:
    """A registered Q8_0 weight (N rows of K; K-padded tensors pass padded K)."""

    def __init__(self, q8_0, n: int, k: int, row_bytes: int | None = None, stream=None):
        import torch
        row_bytes = row_bytes or (k // 32 * 34)
        handle = C.c_void_p()
        if isinstance(q8_0, np.ndarray):
            buf = np.ascontiguousarray(q8_0)
            check(lib().b2q_weight_register(buf.ctypes.data, n, k, row_bytes, 1, _stream(stream), C.byref(handle)))
        else:
            assert isinstance(q8_0, torch.Tensor) and q8_0.is_cuda
            check(lib().b2q_weight_register(q8_0.data_ptr(), n, k, row_bytes, 0, _stream(stream), C.byref(handle)))
        self.handle = handle
        self.n, self.k = n, k

    def release(self):
        if self.handle:
            lib().b2q_weight_release(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


def act_layout(m: int, k: int):
    kp, es, off, ld = I64(), I64(), I64(), I64()
    check(lib().b2q_act_layout(m, k, C.byref(kp), C.byref(es), C.byref(off), C.byref(ld)))
    return kp.value, es.value, off.value, ld.value


def act_empty(m: int, k: int):
    """Allocate an activation buffer (uint8 torch tensor, 256-byte aligned)."""
    import torch
    nbytes = int(lib().b2q_act_bytes(m, k))
    if nbytes == 0:
        raise B2QError(ERR_SHAPE, "bad activation shape")
    t = torch.empty(nbytes + 256, dtype=torch.uint8, device="cuda")
    off = (-t.data_ptr()) % 256
    return t[off:off + nbytes]


def act_planes(act, m: int, k: int):
    """Decode an activation buffer -> (int8 values [M][Kp], fp32 scales [M][Kb]) as torch tensors."""
    import torch
    kp, es, off, ld = act_layout(m, k)
    if es == 1:
        q = act[: m * kp].view(torch.int8).view(m, kp)
    else:
        q = act[: m * kp * 2].view(torch.float16).view(m, kp).to(torch.int8)
    d = act[off: off + (kp // 32) * ld * 4].view(torch.float32).view(kp // 32, ld)[:, :m].t()
    return q, d


def quantize_q8_1(x, act, m: int, k: int, ldx: int | None = None, stream=None):
    check(lib().b2q_quantize_q8_1(_ptr(x), m, k, ldx or k, _ptr(act), _stream(stream)))


def ln_quantize(x, w, b, eps: float, m: int, h: int, act, y=None, stream=None):
    check(lib().b2q_ln_quantize_q8_1(_ptr(x), _ptr(w), _ptr(b), eps, m, h, _ptr(act), _ptr(y), _stream(stream)))


def mul_mat(w: Weight, act, m: int, y=None, kind: int = EPI_NONE, bias=None, residual=None, act_out=None,
            ld_out: int = 0, stream=None):
    e = Epilogue(kind, _ptr(bias), _ptr(residual), _ptr(act_out), ld_out)
    check(lib().b2q_mul_mat_q8_0(w.handle, _ptr(act), m, _ptr(y), C.byref(e), _stream(stream)))


def mul_mat_f32(w: Weight, x, m: int, x_cols: int, y, scratch, stream=None):
    check(lib().b2q_mul_mat_q8_0_f32(w.handle, _ptr(x), m, x_cols, _ptr(y), _ptr(scratch), _stream(stream)))


def mul_mat_f32_noalloc(w: Weight, x, m: int, x_cols: int, y, stream=None):
    """ggml_mul_mat without caller scratch: uses the library's fixed device
    array (B2Q_NOALLOC_MAX_SCRATCH_BYTES), for callers that cannot allocate."""
    check(lib().b2q_mul_mat_q8_0_f32_noalloc(w.handle, _ptr(x), m, x_cols, _ptr(y), _stream(stream)))


NOALLOC_MAX_SCRATCH_BYTES = 32 << 20


def block_sums(w: Weight, act, m: int, out, stream=None):
    check(lib().b2q_block_sums(w.handle, _ptr(act), m, _ptr(out), _stream(stream)))


def _i32(a):
    arr = np.ascontiguousarray(np.asarray(a, dtype=np.int32))
    return arr, arr.ctypes.data_as(C.POINTER(C.c_int32))


def attention(q, ldq, k, ldk, v, ldv, q_off, q_len, k_off, k_len, o_off, n_head, out, ldo, stream=None):
    """Packed-sequence attention (head_dim 72); q/k/v fp16 torch tensors, out fp32."""
    import torch
    keep = [_i32(x) for x in (q_off, q_len, k_off, k_len, o_off)]
    n_seq = len(keep[0][0])
    nbytes = int(lib().b2q_attention_scratch_bytes(keep[1][1], n_seq))
    scratch = torch.empty(max(nbytes, 16), dtype=torch.uint8, device="cuda")
    check(lib().b2q_attention(_ptr(q), ldq, _ptr(k), ldk, _ptr(v), ldv, keep[0][1], keep[1][1], keep[2][1],
                              keep[3][1], keep[4][1], n_seq, n_head, 72, _ptr(out), ldo, _ptr(scratch),
                              _stream(stream)))
    return scratch


class VisionTower:
    """Batched SigLIP2 vision tower (the C++ driver behind b2q_vision_*)."""

    def __init__(self, cfg):
        self.cfg = cfg
        c = VisionConfig(cfg.hidden, cfg.ffn, cfg.n_head, cfg.n_layer, cfg.patch_dim, cfg.pos_side, cfg.eps)
        h = C.c_void_p()
        check(lib().b2q_vision_create(C.byref(c), C.byref(h)))
        self.handle = h

    def set_tensor(self, name: str, arr: np.ndarray, q8_shape=None, stream=None):
        arr = np.ascontiguousarray(arr)
        if q8_shape is not None:
            n, _, kp = q8_shape
            check(lib().b2q_vision_set_tensor(self.handle, name.encode(), GGML_Q8_0, arr.ctypes.data, kp, n,
                                              _stream(stream)))
        else:
            a = np.ascontiguousarray(arr, np.float32)
            ne0 = a.shape[-1]
            ne1 = a.size // ne0
            check(lib().b2q_vision_set_tensor(self.handle, name.encode(), GGML_F32, a.ctypes.data, ne0, ne1,
                                              _stream(stream)))

    def load(self, ck, stream=None):
        for name, arr in ck.tensors.items():
            if not name.startswith("v."):
                continue
            self.set_tensor(name, arr, ck.q8_shapes.get(name), stream)

    def reserve(self, max_tokens: int, max_images: int):
        check(lib().b2q_vision_reserve(self.handle, max_tokens, max_images))

    def load_gguf(self, g: "Gguf", stream=None):
        """Every "v." tensor of an open GGUF file (b2q_vision_load_gguf)."""
        check(lib().b2q_vision_load_gguf(self.handle, g.handle, _stream(stream)))

    def encode(self, patches, grids, pooling=POOL_PROBE, out=None, stream=None):
        """patches: torch CUDA fp32 [T][patch_dim] (images back to back); grids: [(h, w), ...]."""
        import torch
        g, gp = _i32(np.asarray(grids, np.int32).reshape(-1))
        n = len(grids)
        if out is None:
            out = torch.empty((n, self.cfg.hidden), dtype=torch.float32, device="cuda")
        check(lib().b2q_vision_encode(self.handle, _ptr(patches), gp, n, pooling, _ptr(out), _stream(stream)))
        return out

    def encode_host(self, patches: np.ndarray, grids, pooling=POOL_PROBE, out: np.ndarray | None = None,
                    stream=None):
        """Host in, host out (patch upload and embedding download included)."""
        g, gp = _i32(np.asarray(grids, np.int32).reshape(-1))
        n = len(grids)
        if out is None:
            out = np.empty((n, self.cfg.hidden), np.float32)
        check(lib().b2q_vision_encode_host(self.handle, patches.ctypes.data, gp, n, pooling, out.ctypes.data,
                                           _stream(stream)))
        return out

    def submit_host(self, patches, grids, out, pooling=POOL_PROBE, stream=None):
        """Pipelined host entry point (b2q_vision_submit_host): patches and out
        are pinned host tensors (or any host buffers exposing data_ptr / the
        array interface); returns without waiting, see wait()."""
        g, gp = _i32(np.asarray(grids, np.int32).reshape(-1))
        # the last two submissions' buffers stay referenced until their copies have run
        self._keep = (getattr(self, "_keep", ((), ()))[-1], (g, patches, out))
        check(lib().b2q_vision_submit_host(self.handle, _host_ptr(patches), gp, len(grids), pooling, _host_ptr(out),
                                           _stream(stream)))

    def wait(self, stream=None):
        check(lib().b2q_vision_wait(self.handle, _stream(stream)))

    def wait_submitted(self, back=0):
        """Wait for one submission's embeddings: back 0 = the latest, 1 = the one before."""
        check(lib().b2q_vision_wait_submitted(self.handle, back))

    def close(self):
        if self.handle:
            lib().b2q_vision_destroy(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class TextTower:
    """Batched SigLIP2 text tower (the C++ driver behind b2q_text_*)."""

    def __init__(self, cfg):
        self.cfg = cfg
        c = TextConfig(cfg.hidden, cfg.ffn, cfg.n_head, cfg.n_layer, cfg.vocab, cfg.n_pos, cfg.eps)
        h = C.c_void_p()
        check(lib().b2q_text_create(C.byref(c), C.byref(h)))
        self.handle = h

    def set_tensor(self, name: str, arr: np.ndarray, q8_shape=None, stream=None):
        arr = np.ascontiguousarray(arr)
        if q8_shape is not None:
            n, _, kp = q8_shape
            check(lib().b2q_text_set_tensor(self.handle, name.encode(), GGML_Q8_0, arr.ctypes.data, kp, n,
                                            _stream(stream)))
        else:
            a = np.ascontiguousarray(arr, np.float32)
            ne0 = a.shape[-1]
            check(lib().b2q_text_set_tensor(self.handle, name.encode(), GGML_F32, a.ctypes.data, ne0, a.size // ne0,
                                            _stream(stream)))

    def load(self, ck, stream=None):
        for name, arr in ck.tensors.items():
            if name.startswith("t."):
                self.set_tensor(name, arr, ck.q8_shapes.get(name), stream)

    def reserve(self, max_prompts: int):
        check(lib().b2q_text_reserve(self.handle, max_prompts))

    def load_gguf(self, g: "Gguf", stream=None):
        """Every "t." tensor of an open GGUF file (b2q_text_load_gguf)."""
        check(lib().b2q_text_load_gguf(self.handle, g.handle, _stream(stream)))

    def encode(self, ids, out=None, stream=None):
        """ids: torch CUDA int32 [n_prompts][n_pos]."""
        import torch
        n = ids.shape[0]
        if out is None:
            out = torch.empty((n, self.cfg.hidden), dtype=torch.float32, device="cuda")
        check(lib().b2q_text_encode(self.handle, _ptr(ids), n, _ptr(out), _stream(stream)))
        return out

    def encode_host(self, ids: np.ndarray, stream=None) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty((ids.shape[0], self.cfg.hidden), np.float32)
        check(lib().b2q_text_encode_host(self.handle, ids.ctypes.data, ids.shape[0], out.ctypes.data,
                                         _stream(stream)))
        return out

    def close(self):
        if self.handle:
            lib().b2q_text_destroy(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def score(img, txt, logit_scale: float, logit_bias: float, logits=True, probs=True, stream=None):
    """Image-text sigmoid scores on the device (b2q_score); img [I][H], txt [J][H]
    torch CUDA fp32.  Returns (logits, probs), either None if not requested."""
    import torch
    I, H = img.shape
    J = txt.shape[0]
    scratch = torch.empty(int(lib().b2q_score_scratch_bytes(I, J, H)), dtype=torch.uint8, device="cuda")
    lg = torch.empty((I, J), dtype=torch.float32, device="cuda") if logits else None
    pr = torch.empty((I, J), dtype=torch.float32, device="cuda") if probs else None
    check(lib().b2q_score(_ptr(img), I, _ptr(txt), J, H, float(logit_scale), float(logit_bias), _ptr(lg), _ptr(pr),
                          _ptr(scratch), _stream(stream)))
    return lg, pr


class Gguf:
    """A GGUF checkpoint mapped by the library (b2q_gguf_*)."""

    def __init__(self, path):
        h = C.c_void_p()
        check(lib().b2q_gguf_open(str(path).encode(), C.byref(h)))
        self.handle = h

    def tensors(self):
        """[(name, ggml_type, ne tuple, data address)] in file order."""
        out = []
        for i in range(int(lib().b2q_gguf_n_tensors(self.handle))):
            name, typ, nd = C.c_char_p(), C.c_int32(), C.c_int32()
            ne = (I64 * 4)()
            data = C.c_void_p()
            check(lib().b2q_gguf_tensor(self.handle, i, C.byref(name), C.byref(typ), C.byref(nd), ne, C.byref(data)))
            out.append((name.value.decode(), typ.value, tuple(ne[: nd.value]), data.value))
        return out

    def scalar(self, name: str) -> float:
        v = C.c_float()
        check(lib().b2q_gguf_scalar_f32(self.handle, name.encode(), C.byref(v)))
        return v.value

    def close(self):
        if self.handle:
            lib().b2q_gguf_close(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
