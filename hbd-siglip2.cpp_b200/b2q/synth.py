"""Seeded synthetic SigLIP2 checkpoints and inputs.

No real checkpoint ships with this build, so every benchmark and test runs on
synthetic weights that follow the reference's GGUF conventions:

* tensor names as loaded by ``src/siglip2_vision.cpp:496-556`` and
  ``src/siglip2_text.cpp:485-520`` (``v.blk.{i}.attn_qkv.weight`` ...);
* dtype policy of ``scripts/convert_siglip2_to_gguf.py:210-290``: projections
  Q8_0, biases / LayerNorm / position tables / probe fp32;
* ``ffn_down`` (K = 4304) zero-padded to K = 4320 before Q8_0 quantization,
  the rule of ``tools/siglip2-quantize/main.cpp:174-186`` (135 blocks).

Weights are N(0, std) with a per-tensor seed derived from the tensor name, so
any subset of tensors can be regenerated independently.  ``quantize_q8_0``
restates gguf-py's Q8_0 codec (``gguf/quants.py:381-401``, documented there as
bit-exact with ggml-quants.c); tests pin it against gguf-py itself.
"""
from __future__ import annotations

import zlib
from dataclasses import dataclass, field

import numpy as np

QK = 32
Q8_0_BLOCK_BYTES = 34


def roundf_half_away(x: np.ndarray) -> np.ndarray:
    """C ``roundf``: round half away from zero (gguf-py ``np_roundf``)."""
    a = np.abs(x)
    r = np.floor(a)
    r += (a - r) >= 0.5
    return np.sign(x) * r


def quantize_q8_0(w: np.ndarray, k_pad: int | None = None) -> np.ndarray:
    """Quantize rows of ``w`` ([N][K] fp32) to ggml Q8_0 bytes ([N][Kp/32*34]).

    ``k_pad`` zero-extends K first (K-padding rule for ffn_down).
    """
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    kp = k if k_pad is None else k_pad
    if kp % QK:
        raise ValueError(f"K={kp} is not a multiple of {QK}")
    if kp != k:
        w = np.concatenate([w, np.zeros((n, kp - k), np.float32)], axis=1)
    blocks = w.reshape(-1, QK)
    d = np.abs(blocks).max(axis=1, keepdims=True) / np.float32(127)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    qs = roundf_half_away(blocks * inv).astype(np.int8)
    out = np.empty((blocks.shape[0], Q8_0_BLOCK_BYTES), np.uint8)
    out[:, :2] = d.astype(np.float16).view(np.uint8)
    out[:, 2:] = qs.view(np.uint8)
    return out.reshape(n, (kp // QK) * Q8_0_BLOCK_BYTES)


def dequantize_q8_0(q: np.ndarray, kp: int) -> np.ndarray:
    n = q.shape[0]
    b = q.reshape(-1, Q8_0_BLOCK_BYTES)
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    x = b[:, 2:].copy().view(np.int8).astype(np.float32)
    return (x * d).reshape(n, kp)


def tensor_seed(name: str, base_seed: int) -> int:
    return (zlib.crc32(name.encode()) ^ (base_seed * 0x9E3779B1)) & 0xFFFFFFFF


def normal(name: str, shape, std: float, base_seed: int) -> np.ndarray:
    rng = np.random.default_rng(tensor_seed(name, base_seed))
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


@dataclass
class TowerConfig:
    """SigLIP2-so400m geometry: width 1152, 27 layers, 16 heads, MLP 4304, 16x16 position table, vocab 256000."""
    hidden: int = 1152
    ffn: int = 4304
    n_head: int = 16
    n_layer: int = 27
    eps: float = 1e-6
    # vision
    patch_dim: int = 768          # 16 x 16 x 3
    pos_side: int = 16            # learned 16x16 position table
    # text
    vocab: int = 256000
    n_pos: int = 64

    @property
    def ffn_pad(self) -> int:
        return (self.ffn + QK - 1) // QK * QK

    @property
    def d_head(self) -> int:
        return self.hidden // self.n_head


@dataclass
class Checkpoint:
    """name -> ndarray.  Q8_0 tensors are uint8 [N][Kp/32*34]; others fp32."""
    cfg: TowerConfig
    tensors: dict = field(default_factory=dict)
    q8_shapes: dict = field(default_factory=dict)   # name -> (N, K, Kp)

    def q8(self, name: str) -> np.ndarray:
        return self.tensors[name]

    def f32(self, name: str) -> np.ndarray:
        return self.tensors[name]


def _proj(ck: Checkpoint, name: str, n: int, k: int, std: float, seed: int,
          bias_std: float, k_pad: int | None = None):
    w = normal(name + ".weight", (n, k), std, seed)
    kp = k if k_pad is None else k_pad
    ck.tensors[name + ".weight"] = quantize_q8_0(w, kp)
    ck.q8_shapes[name + ".weight"] = (n, k, kp)
    ck.tensors[name + ".bias"] = (normal(name + ".bias", (n,), bias_std, seed)
                                  if bias_std > 0 else np.zeros(n, np.float32))


def _ln(ck: Checkpoint, name: str, h: int, seed: int, ln_std: float):
    if ln_std > 0:
        ck.tensors[name + ".weight"] = 1.0 + normal(name + ".weight", (h,), ln_std, seed)
        ck.tensors[name + ".bias"] = normal(name + ".bias", (h,), ln_std, seed)
    else:
        ck.tensors[name + ".weight"] = np.ones(h, np.float32)
        ck.tensors[name + ".bias"] = np.zeros(h, np.float32)


def _block(ck: Checkpoint, pfx: str, cfg: TowerConfig, std, seed, bias_std, ln_std):
    H, F = cfg.hidden, cfg.ffn
    _ln(ck, pfx + "ln1", H, seed, ln_std)
    _proj(ck, pfx + "attn_qkv", 3 * H, H, std, seed, bias_std)
    _proj(ck, pfx + "attn_o", H, H, std, seed, bias_std)
    _ln(ck, pfx + "ln2", H, seed, ln_std)
    _proj(ck, pfx + "ffn_up", F, H, std, seed, bias_std)
    _proj(ck, pfx + "ffn_down", H, F, std, seed, bias_std, k_pad=cfg.ffn_pad)


def vision_checkpoint(cfg: TowerConfig | None = None, seed: int = 0, std: float = 0.02,
                      bias_std: float = 0.0, ln_std: float = 0.0) -> Checkpoint:
    """Synthetic vision tower: weights N(0, std) -> Q8_0; LN gains 1 and biases
    0 unless ``ln_std`` / ``bias_std`` ask for random ones (tests do)."""
    cfg = cfg or TowerConfig()
    ck = Checkpoint(cfg)
    H = cfg.hidden
    _proj(ck, "v.patch_embd", H, cfg.patch_dim, std, seed, bias_std)
    ck.tensors["v.position_embd.weight"] = normal("v.position_embd.weight",
                                                  (cfg.pos_side * cfg.pos_side, H), std, seed)
    for i in range(cfg.n_layer):
        _block(ck, f"v.blk.{i}.", cfg, std, seed, bias_std, ln_std)
    _ln(ck, "v.post_ln", H, seed, ln_std)
    ck.tensors["v.head.probe"] = normal("v.head.probe", (H,), std, seed)
    for p in ("attn_q", "attn_k", "attn_v", "attn_o"):
        _proj(ck, "v.head." + p, H, H, std, seed, bias_std)
    _ln(ck, "v.head.ln", H, seed, ln_std)
    _proj(ck, "v.head.ffn_up", cfg.ffn, H, std, seed, bias_std)
    _proj(ck, "v.head.ffn_down", H, cfg.ffn, std, seed, bias_std, k_pad=cfg.ffn_pad)
    return ck


def text_checkpoint(cfg: TowerConfig | None = None, seed: int = 0, std: float = 0.02,
                    bias_std: float = 0.0, ln_std: float = 0.0) -> Checkpoint:
    cfg = cfg or TowerConfig()
    ck = Checkpoint(cfg)
    H = cfg.hidden
    emb = normal("t.token_embd.weight", (cfg.vocab, H), std, seed)
    ck.tensors["t.token_embd.weight"] = quantize_q8_0(emb)
    ck.q8_shapes["t.token_embd.weight"] = (cfg.vocab, H, H)
    ck.tensors["t.position_embd.weight"] = normal("t.position_embd.weight", (cfg.n_pos, H), std, seed)
    for i in range(cfg.n_layer):
        _block(ck, f"t.blk.{i}.", cfg, std, seed, bias_std, ln_std)
    _ln(ck, "t.final_ln", H, seed, ln_std)
    _proj(ck, "t.head", H, H, std, seed, bias_std)
    return ck


def patches(n_tokens: int, patch_dim: int = 768, seed: int = 0) -> np.ndarray:
    """Pixel patch vectors (16x16x3 = 768 values each) uniform in [-1, 1]."""
    rng = np.random.default_rng(0xB01D ^ seed)
    return rng.uniform(-1.0, 1.0, size=(n_tokens, patch_dim)).astype(np.float32)


def naflex_grids(n_images: int, lo: int = 256, hi: int = 1024, seed: int = 0):
    """Per-image (h, w) patch grids for the NaFlex batch workload: a patch budget drawn
    uniformly from [lo, hi] and an aspect ratio log-uniform in [1/4, 4] (the
    range NaFlex resizing produces for ordinary photos), h = round(sqrt(n r)),
    w = floor(n / h), so h * w stays inside [lo - h, hi]."""
    rng = np.random.default_rng(0xC4 ^ seed)
    grids = []
    for _ in range(n_images):
        n = int(rng.integers(lo, hi + 1))
        r = float(np.exp(rng.uniform(np.log(0.25), np.log(4.0))))
        h = max(1, min(n, int(round(np.sqrt(n * r)))))
        w = max(1, n // h)
        grids.append((h, w))
    return grids


def token_ids(n_prompts: int, n_pos: int = 64, vocab: int = 256000, seed: int = 0) -> np.ndarray:
    """Token ids uniform in [1, vocab) with EOS id 1 at the last position, as
    the text workloads use them (no padding mask)."""
    rng = np.random.default_rng(0x7E47 ^ seed)
    ids = rng.integers(1, vocab, size=(n_prompts, n_pos)).astype(np.int32)
    ids[:, -1] = 1
    return ids
