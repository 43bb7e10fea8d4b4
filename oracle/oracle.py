"""ctypes binding of the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and
the CPU-baseline legs of ``bench.py``; never by the product package.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

_lib = None


def build(force: bool = False) -> Path:
    if force or not LIB_PATH.exists() or \
            LIB_PATH.stat().st_mtime < (HERE / "b2q_oracle.c").stat().st_mtime:
        subprocess.run(["make", "-C", str(HERE), "-s"], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = C.CDLL(str(LIB_PATH))
        _declare(_lib)
    return _lib


P = C.c_void_p
I64 = C.c_int64


def _declare(L):
    L.orc_fp16_to_fp32.argtypes = [C.c_uint16]; L.orc_fp16_to_fp32.restype = C.c_float
    L.orc_fp32_to_fp16.argtypes = [C.c_float]; L.orc_fp32_to_fp16.restype = C.c_uint16
    L.orc_expf.argtypes = [C.c_float]; L.orc_expf.restype = C.c_float
    L.orc_div.argtypes = [C.c_float, C.c_float]; L.orc_div.restype = C.c_float
    L.orc_gelu.argtypes = [C.c_float]; L.orc_gelu.restype = C.c_float
    L.orc_gelu_n.argtypes = [C.c_void_p, C.c_int64, C.c_void_p]; L.orc_gelu_n.restype = None
    L.orc_quantize_q8_1_rule.argtypes = [P, I64, I64, I64, I64, P, P, C.c_int]
    L.orc_num_threads.restype = C.c_int
    L.orc_set_num_threads.argtypes = [C.c_int]
    L.orc_quantize_q8_0.argtypes = [P, I64, I64, I64, P]
    L.orc_dequantize_q8_0.argtypes = [P, I64, I64, P]
    L.orc_quantize_q8_1.argtypes = [P, I64, I64, I64, I64, P, P]
    L.orc_gemm_q8.argtypes = [P, I64, I64, P, P, I64, P, P]
    L.orc_layernorm.argtypes = [P, P, P, C.c_float, I64, I64, P]
    L.orc_attention.argtypes = [P, I64, I64, I64, P, P, I64, P]
    L.orc_pos_resize.argtypes = [P, I64, I64, I64, I64, P]
    L.orc_vision_encode.argtypes = [P, P, I64, I64, C.c_int, C.c_int, P]
    L.orc_text_encode.argtypes = [P, P, I64, C.c_int, P]
    L.orc_score.argtypes = [P, I64, P, I64, I64, C.c_float, C.c_float, P, P]
    L.orc_set_rules.argtypes = [C.c_int]
    L.orc_get_rules.restype = C.c_int


def _p(a: np.ndarray):
    assert a.flags.c_contiguous
    return a.ctypes.data_as(C.c_void_p)


RULE_LN, RULE_GELU, RULE_Q8, RULE_GEMM = 1, 2, 4, 8
RULES_REFERENCE = RULE_LN | RULE_GELU | RULE_Q8 | RULE_GEMM


def set_rules(rules: int):
    """Switch the towers' element rules (0 = the canonical order the CUDA
    kernels reproduce; RULES_REFERENCE = the reference kernels' own LayerNorm
    order, tanhf GELU, half-away q8_1 and scale-product accumulation)."""
    lib().orc_set_rules(int(rules))


def get_rules() -> int:
    return int(lib().orc_get_rules())


def set_threads(n: int):
    lib().orc_set_num_threads(int(n))


def num_threads() -> int:
    return int(lib().orc_num_threads())


# ---- scalar -----------------------------------------------------------------
def div(a: float, b: float) -> float:
    return lib().orc_div(float(a), float(b))


def gelu(x: float) -> float:
    return lib().orc_gelu(float(x))


def gelu_vec(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().orc_gelu_n(_p(x), x.size, _p(y))
    return y


def expf(x: float) -> float:
    return lib().orc_expf(float(x))


# ---- formats ----------------------------------------------------------------
def quantize_q8_0(w: np.ndarray, kp: int | None = None) -> np.ndarray:
    w = np.ascontiguousarray(w, np.float32)
    n, k = w.shape
    kp = k if kp is None else kp
    out = np.empty((n, kp // 32 * 34), np.uint8)
    lib().orc_quantize_q8_0(_p(w), n, k, kp, _p(out))
    return out


def dequantize_q8_0(q: np.ndarray, kp: int) -> np.ndarray:
    q = np.ascontiguousarray(q)
    out = np.empty((q.shape[0], kp), np.float32)
    lib().orc_dequantize_q8_0(_p(q), q.shape[0], kp, _p(out))
    return out


def quantize_q8_1(x: np.ndarray, kp: int | None = None, rule: int | None = None):
    """-> (qs int8 [M][Kp], d fp32 [M][Kp/32]); rule selects an alternative
    rounding convention (orc_quantize_q8_1_rule), None = the default."""
    x = np.ascontiguousarray(x, np.float32)
    m, k = x.shape
    kp = k if kp is None else kp
    qs = np.empty((m, kp), np.int8)
    d = np.empty((m, kp // 32), np.float32)
    if rule is None:
        lib().orc_quantize_q8_1(_p(x), m, k, k, kp, _p(qs), _p(d))
    else:
        lib().orc_quantize_q8_1_rule(_p(x), m, k, k, kp, _p(qs), _p(d), int(rule))
    return qs, d


def gemm_q8(w_q8_0: np.ndarray, n: int, kp: int, qs: np.ndarray, dx: np.ndarray,
            block_sums: bool = False):
    m = qs.shape[0]
    y = np.empty((m, n), np.float32)
    bs = np.empty((m, n, kp // 32), np.int32) if block_sums else None
    lib().orc_gemm_q8(_p(np.ascontiguousarray(w_q8_0)), n, kp, _p(np.ascontiguousarray(qs)),
                      _p(np.ascontiguousarray(dx)), m, _p(y), _p(bs) if bs is not None else None)
    return (y, bs) if block_sums else y


def layernorm(x: np.ndarray, w: np.ndarray, b: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().orc_layernorm(_p(x), _p(np.ascontiguousarray(w, np.float32)),
                        _p(np.ascontiguousarray(b, np.float32)), float(eps), x.shape[0], x.shape[1], _p(y))
    return y


def attention(qkv: np.ndarray, n_head: int, seq_lens) -> np.ndarray:
    qkv = np.ascontiguousarray(qkv, np.float32)
    t, h3 = qkv.shape
    h = h3 // 3
    lens = np.asarray(seq_lens, np.int64)
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    out = np.empty((t, h), np.float32)
    lib().orc_attention(_p(qkv), t, h, n_head, _p(offs), _p(lens), len(lens), _p(out))
    return out


def pos_resize(table: np.ndarray, side: int, h: int, w: int) -> np.ndarray:
    table = np.ascontiguousarray(table, np.float32)
    H = table.shape[1]
    out = np.empty((h * w, H), np.float32)
    lib().orc_pos_resize(_p(table), side, H, h, w, _p(out))
    return out


# ---- towers -----------------------------------------------------------------
class _Block(C.Structure):
    _fields_ = [(n, P) for n in ("ln1_w", "ln1_b", "ln2_w", "ln2_b", "qkv_w", "qkv_b", "o_w", "o_b",
                                 "up_w", "up_b", "down_w", "down_b")]


class _Vision(C.Structure):
    _fields_ = ([(n, I64) for n in ("H", "F", "Fp", "n_head", "n_layer", "patch_dim", "pos_side")]
                + [("eps", C.c_float)]
                + [(n, P) for n in ("patch_w", "patch_b", "pos_embd", "blocks", "post_ln_w", "post_ln_b",
                                    "probe", "hq_w", "hk_w", "hv_w", "ho_w", "hq_b", "hk_b", "hv_b", "ho_b",
                                    "hln_w", "hln_b", "hup_w", "hup_b", "hdown_w", "hdown_b")])


class _Text(C.Structure):
    _fields_ = ([(n, I64) for n in ("H", "F", "Fp", "n_head", "n_layer", "vocab", "n_pos")]
                + [("eps", C.c_float)]
                + [(n, P) for n in ("tok_embd", "pos_embd", "blocks", "final_ln_w", "final_ln_b",
                                    "head_w", "head_b")])


def _blocks(ck, pfx, n_layer, keep):
    arr = (_Block * n_layer)()
    for i in range(n_layer):
        b = arr[i]
        t = ck.tensors
        for field, nm in (("ln1_w", "ln1.weight"), ("ln1_b", "ln1.bias"), ("ln2_w", "ln2.weight"),
                          ("ln2_b", "ln2.bias"), ("qkv_w", "attn_qkv.weight"), ("qkv_b", "attn_qkv.bias"),
                          ("o_w", "attn_o.weight"), ("o_b", "attn_o.bias"), ("up_w", "ffn_up.weight"),
                          ("up_b", "ffn_up.bias"), ("down_w", "ffn_down.weight"), ("down_b", "ffn_down.bias")):
            a = np.ascontiguousarray(t[f"{pfx}{i}.{nm}"])
            keep.append(a)
            setattr(b, field, a.ctypes.data)
    keep.append(arr)
    return arr


def vision_encode(ck, patches: np.ndarray, h: int, w: int, pooling: int = 1,
                  quant_act: bool = True) -> np.ndarray:
    cfg = ck.cfg
    keep = []
    W = _Vision()
    W.H, W.F, W.Fp, W.n_head, W.n_layer = cfg.hidden, cfg.ffn, cfg.ffn_pad, cfg.n_head, cfg.n_layer
    W.patch_dim, W.pos_side, W.eps = cfg.patch_dim, cfg.pos_side, cfg.eps
    t = ck.tensors

    def ptr(name):
        a = np.ascontiguousarray(t[name])
        keep.append(a)
        return a.ctypes.data

    W.patch_w, W.patch_b = ptr("v.patch_embd.weight"), ptr("v.patch_embd.bias")
    W.pos_embd = ptr("v.position_embd.weight")
    blocks = _blocks(ck, "v.blk.", cfg.n_layer, keep)
    W.blocks = C.cast(blocks, C.c_void_p)
    W.post_ln_w, W.post_ln_b = ptr("v.post_ln.weight"), ptr("v.post_ln.bias")
    W.probe = ptr("v.head.probe")
    W.hq_w, W.hk_w, W.hv_w, W.ho_w = (ptr(f"v.head.attn_{x}.weight") for x in "qkvo")
    W.hq_b, W.hk_b, W.hv_b, W.ho_b = (ptr(f"v.head.attn_{x}.bias") for x in "qkvo")
    W.hln_w, W.hln_b = ptr("v.head.ln.weight"), ptr("v.head.ln.bias")
    W.hup_w, W.hup_b = ptr("v.head.ffn_up.weight"), ptr("v.head.ffn_up.bias")
    W.hdown_w, W.hdown_b = ptr("v.head.ffn_down.weight"), ptr("v.head.ffn_down.bias")
    x = np.ascontiguousarray(patches, np.float32)
    out = np.empty(cfg.hidden, np.float32)
    lib().orc_vision_encode(C.byref(W), _p(x), h, w, pooling, 1 if quant_act else 0, _p(out))
    return out


def text_encode(ck, ids: np.ndarray, quant_act: bool = True) -> np.ndarray:
    cfg = ck.cfg
    keep = []
    W = _Text()
    W.H, W.F, W.Fp, W.n_head, W.n_layer = cfg.hidden, cfg.ffn, cfg.ffn_pad, cfg.n_head, cfg.n_layer
    W.vocab, W.n_pos, W.eps = cfg.vocab, cfg.n_pos, cfg.eps
    t = ck.tensors

    def ptr(name):
        a = np.ascontiguousarray(t[name])
        keep.append(a)
        return a.ctypes.data

    W.tok_embd, W.pos_embd = ptr("t.token_embd.weight"), ptr("t.position_embd.weight")
    blocks = _blocks(ck, "t.blk.", cfg.n_layer, keep)
    W.blocks = C.cast(blocks, C.c_void_p)
    W.final_ln_w, W.final_ln_b = ptr("t.final_ln.weight"), ptr("t.final_ln.bias")
    W.head_w, W.head_b = ptr("t.head.weight"), ptr("t.head.bias")
    ids = np.ascontiguousarray(ids, np.int32)
    n = ids.shape[0]
    out = np.empty((n, cfg.hidden), np.float32)
    lib().orc_text_encode(C.byref(W), _p(ids), n, 1 if quant_act else 0, _p(out))
    return out


def score(img: np.ndarray, txt: np.ndarray, logit_scale: float, logit_bias: float, with_logits: bool = False):
    img = np.ascontiguousarray(img, np.float32)
    txt = np.ascontiguousarray(txt, np.float32)
    out = np.empty((img.shape[0], txt.shape[0]), np.float32)
    logits = np.empty_like(out) if with_logits else None
    lib().orc_score(_p(img), img.shape[0], _p(txt), txt.shape[0], img.shape[1],
                    float(logit_scale), float(logit_bias), _p(logits) if with_logits else None, _p(out))
    return (out, logits) if with_logits else out
