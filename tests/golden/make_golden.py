"""Generate the golden fixtures under tests/golden/.

The reference ships no stored tensors, so the pins are produced here from the
reference's own dependencies, imported in this container:

* ``q8_0_gguf.npz`` — gguf-py 0.19.0 ``quants.quantize(..., Q8_0)`` outputs
  (the quantizer the reference's converter calls at
  scripts/convert_siglip2_to_gguf.py:263; documented bit-exact with
  ggml-quants.c) for seeded rows plus edge rows: an all-zero block, exact
  .5 ties of the scaled value, blocks whose max element is negative, and a
  K = 4304 row zero-padded to 4320 (tools/siglip2-quantize/main.cpp:174-186).
* ``hf_vision.npz`` / ``hf_text.npz`` — HF transformers Siglip2VisionModel /
  Siglip2TextModel pooled outputs for 2-layer towers whose fp32 weights are
  the dequantized synthetic Q8_0 weights (``b2q.synth``, fixed seeds), the
  architecture check for the oracle's towers (fp32-activation mode).

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "hbd-siglip2.cpp_b200"))
from b2q import synth  # noqa: E402

OUT = Path(__file__).resolve().parent

VISION_SEED, TEXT_SEED = 3, 5
VISION_GRIDS = [(16, 16), (12, 20), (27, 27), (5, 9)]
TEXT_VOCAB = 1000


def q8_0_vectors():
    import gguf
    rng = np.random.default_rng(1234)
    rows = [rng.standard_normal((8, 1152)).astype(np.float32) * 0.02,
            rng.uniform(-3, 3, (4, 256)).astype(np.float32)]
    edge = np.zeros((4, 64), np.float32)
    edge[1, :32] = np.arange(32, dtype=np.float32) - 16.0       # max |x| = 16 at a negative value
    edge[2, :32] = (np.arange(32, dtype=np.float32) + 0.5) * 127.0 / 32.0 / 127.0 * 2.0
    edge[3, 32:] = np.linspace(-1, 1, 32, dtype=np.float32)
    ties = np.zeros((1, 32), np.float32)
    ties[0, 0] = 127.0                                          # d = 1 exactly, id = 1
    ties[0, 1:16] = np.arange(1, 16, dtype=np.float32) + 0.5     # x*id lands on .5 ties
    ties[0, 16:] = -(np.arange(16, dtype=np.float32) + 0.5)
    out = {}
    for i, r in enumerate(rows + [edge, ties]):
        out[f"x{i}"] = r
        out[f"q{i}"] = gguf.quants.quantize(r, gguf.GGMLQuantizationType.Q8_0)
    pad = rng.standard_normal((3, 4304)).astype(np.float32) * 0.02
    padded = np.concatenate([pad, np.zeros((3, 16), np.float32)], axis=1)
    out["xpad"] = pad
    out["qpad"] = gguf.quants.quantize(padded, gguf.GGMLQuantizationType.Q8_0)
    np.savez_compressed(OUT / "q8_0_gguf.npz", **out)


def _deq(ck, name):
    import torch
    n, k, kp = ck.q8_shapes[name]
    return torch.from_numpy(synth.dequantize_q8_0(ck.tensors[name], kp)[:, :k].copy())


def _load_block(L, ck, p):
    import torch
    t = ck.tensors
    f = lambda n: torch.from_numpy(t[n])  # noqa: E731
    H = ck.cfg.hidden
    qkv, qb = _deq(ck, p + "attn_qkv.weight"), f(p + "attn_qkv.bias")
    a = L.self_attn
    for j, lin in enumerate((a.q_proj, a.k_proj, a.v_proj)):
        lin.weight.copy_(qkv[j * H:(j + 1) * H])
        lin.bias.copy_(qb[j * H:(j + 1) * H])
    a.out_proj.weight.copy_(_deq(ck, p + "attn_o.weight"))
    a.out_proj.bias.copy_(f(p + "attn_o.bias"))
    L.layer_norm1.weight.copy_(f(p + "ln1.weight")); L.layer_norm1.bias.copy_(f(p + "ln1.bias"))
    L.layer_norm2.weight.copy_(f(p + "ln2.weight")); L.layer_norm2.bias.copy_(f(p + "ln2.bias"))
    L.mlp.fc1.weight.copy_(_deq(ck, p + "ffn_up.weight")); L.mlp.fc1.bias.copy_(f(p + "ffn_up.bias"))
    L.mlp.fc2.weight.copy_(_deq(ck, p + "ffn_down.weight")); L.mlp.fc2.bias.copy_(f(p + "ffn_down.bias"))


def hf_vision():
    import torch
    from transformers import Siglip2VisionConfig, Siglip2VisionModel
    cfg = synth.TowerConfig(n_layer=2)
    ck = synth.vision_checkpoint(cfg, seed=VISION_SEED, bias_std=0.02, ln_std=0.1)
    hc = Siglip2VisionConfig(hidden_size=cfg.hidden, intermediate_size=cfg.ffn, num_hidden_layers=cfg.n_layer,
                             num_attention_heads=cfg.n_head, num_channels=3, num_patches=256, patch_size=16,
                             hidden_act="gelu_pytorch_tanh", layer_norm_eps=cfg.eps, vision_use_head=True)
    m = Siglip2VisionModel(hc).eval()
    vm, t = m.vision_model, ck.tensors
    f = lambda n: torch.from_numpy(t[n])  # noqa: E731
    with torch.no_grad():
        vm.embeddings.patch_embedding.weight.copy_(_deq(ck, "v.patch_embd.weight"))
        vm.embeddings.patch_embedding.bias.copy_(f("v.patch_embd.bias"))
        vm.embeddings.position_embedding.weight.copy_(f("v.position_embd.weight"))
        for i, L in enumerate(vm.encoder.layers):
            _load_block(L, ck, f"v.blk.{i}.")
        vm.post_layernorm.weight.copy_(f("v.post_ln.weight")); vm.post_layernorm.bias.copy_(f("v.post_ln.bias"))
        hd = vm.head
        hd.probe.copy_(f("v.head.probe").view(1, 1, -1))
        hd.attention.in_proj_weight.copy_(torch.cat([_deq(ck, f"v.head.attn_{x}.weight") for x in "qkv"]))
        hd.attention.in_proj_bias.copy_(torch.cat([f(f"v.head.attn_{x}.bias") for x in "qkv"]))
        hd.attention.out_proj.weight.copy_(_deq(ck, "v.head.attn_o.weight"))
        hd.attention.out_proj.bias.copy_(f("v.head.attn_o.bias"))
        hd.layernorm.weight.copy_(f("v.head.ln.weight")); hd.layernorm.bias.copy_(f("v.head.ln.bias"))
        hd.mlp.fc1.weight.copy_(_deq(ck, "v.head.ffn_up.weight")); hd.mlp.fc1.bias.copy_(f("v.head.ffn_up.bias"))
        hd.mlp.fc2.weight.copy_(_deq(ck, "v.head.ffn_down.weight")); hd.mlp.fc2.bias.copy_(f("v.head.ffn_down.bias"))
        out = {}
        for gi, (h, w) in enumerate(VISION_GRIDS):
            x = synth.patches(h * w, seed=gi)
            r = m(pixel_values=torch.from_numpy(x)[None],
                  pixel_attention_mask=torch.ones(1, h * w, dtype=torch.long),
                  spatial_shapes=torch.tensor([[h, w]]))
            out[f"pooled_{h}x{w}"] = r.pooler_output[0].numpy()
            out[f"mean_{h}x{w}"] = r.last_hidden_state[0].mean(0).numpy()
    np.savez_compressed(OUT / "hf_vision.npz", grids=np.array(VISION_GRIDS), seed=VISION_SEED, **out)


def hf_text():
    import torch
    from transformers import Siglip2TextConfig, Siglip2TextModel
    cfg = synth.TowerConfig(n_layer=2, vocab=TEXT_VOCAB)
    ck = synth.text_checkpoint(cfg, seed=TEXT_SEED, bias_std=0.02, ln_std=0.1)
    hc = Siglip2TextConfig(vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.ffn,
                           num_hidden_layers=cfg.n_layer, num_attention_heads=cfg.n_head,
                           max_position_embeddings=cfg.n_pos, hidden_act="gelu_pytorch_tanh",
                           layer_norm_eps=cfg.eps, projection_size=cfg.hidden)
    m = Siglip2TextModel(hc).eval()
    tm, t = m.text_model, ck.tensors
    f = lambda n: torch.from_numpy(t[n])  # noqa: E731
    with torch.no_grad():
        tm.embeddings.token_embedding.weight.copy_(_deq(ck, "t.token_embd.weight"))
        tm.embeddings.position_embedding.weight.copy_(f("t.position_embd.weight"))
        for i, L in enumerate(tm.encoder.layers):
            _load_block(L, ck, f"t.blk.{i}.")
        tm.final_layer_norm.weight.copy_(f("t.final_ln.weight")); tm.final_layer_norm.bias.copy_(f("t.final_ln.bias"))
        tm.head.weight.copy_(_deq(ck, "t.head.weight")); tm.head.bias.copy_(f("t.head.bias"))
        ids = synth.token_ids(3, cfg.n_pos, cfg.vocab, seed=1)
        r = m(input_ids=torch.from_numpy(ids).long())
    np.savez_compressed(OUT / "hf_text.npz", ids=ids, pooled=r.pooler_output.numpy(), seed=TEXT_SEED,
                        vocab=TEXT_VOCAB)


if __name__ == "__main__":
    q8_0_vectors()
    hf_vision()
    hf_text()
    for p in sorted(OUT.glob("*.npz")):
        print(p.name, p.stat().st_size)
