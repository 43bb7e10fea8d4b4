"""Towers loaded from GGUF files (b2q_*_load_gguf) encode exactly like towers
loaded tensor by tensor, including projections the file stores as F16 or
F32, which the loader quantizes to Q8_0 (K zero-padded to a multiple of 32)."""
import copy

import numpy as np
import pytest

import b2q
from b2q import synth
from gguf_util import write_checkpoint

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
pytest.importorskip("gguf")


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    b2q.init(0)
    b2q.tune(b2q.TUNE_ATTN_EXACT, 1)
    yield
    b2q.tune(b2q.TUNE_ATTN_EXACT, 0)


def test_vision_tower_from_gguf(dev, tmp_path):
    cfg = synth.TowerConfig(n_layer=2)
    ck = synth.vision_checkpoint(cfg, seed=13, bias_std=0.02, ln_std=0.1)
    # layer 0 ffn_down stored F16 with its true K = 4304; layer 1 attn_o stored F32
    down = "v.blk.0.ffn_down.weight"
    w_down = synth.normal(down, (cfg.hidden, cfg.ffn), 0.02, 13).astype(np.float16)
    o1 = "v.blk.1.attn_o.weight"
    w_o1 = synth.normal(o1, (cfg.hidden, cfg.hidden), 0.02, 13)
    p = tmp_path / "vision.gguf"
    write_checkpoint(p, ck, f16_weights={down: w_down}, f32_weights={o1: w_o1})
    # the same values quantized on the host for the tensor-by-tensor path
    ref = copy.copy(ck)
    ref.tensors = dict(ck.tensors)
    ref.tensors[down] = synth.quantize_q8_0(w_down.astype(np.float32), cfg.ffn_pad)
    ref.tensors[o1] = synth.quantize_q8_0(w_o1, cfg.hidden)
    grids = [(16, 16), (9, 12)]
    patches = torch.from_numpy(np.concatenate([synth.patches(h * w, cfg.patch_dim, seed=i)
                                               for i, (h, w) in enumerate(grids)])).cuda()
    a = b2q.VisionTower(cfg)
    g = b2q.Gguf(p)
    a.load_gguf(g)
    g.close()
    b = b2q.VisionTower(cfg)
    b.load(ref)
    ea = a.encode(patches, grids, b2q.POOL_PROBE).cpu().numpy()
    eb = b.encode(patches, grids, b2q.POOL_PROBE).cpu().numpy()
    assert b2q.check_device() == 0
    np.testing.assert_array_equal(ea, eb)


def test_text_tower_and_scalars_from_gguf(dev, tmp_path):
    cfg = synth.TowerConfig(n_layer=2, vocab=300)
    ck = synth.text_checkpoint(cfg, seed=17, bias_std=0.02, ln_std=0.1)
    p = tmp_path / "text.gguf"
    write_checkpoint(p, ck, extra={"mm.logit_scale": np.array([np.log(10.0)], np.float32),
                                   "mm.logit_bias": np.array([-10.0], np.float32)})
    g = b2q.Gguf(p)
    a = b2q.TextTower(cfg)
    a.load_gguf(g)
    assert g.scalar("mm.logit_bias") == -10.0
    assert g.scalar("mm.logit_scale") == np.float32(np.log(10.0))
    g.close()
    b = b2q.TextTower(cfg)
    b.load(ck)
    ids = torch.from_numpy(synth.token_ids(3, cfg.n_pos, cfg.vocab, seed=3)).cuda()
    np.testing.assert_array_equal(a.encode(ids).cpu().numpy(), b.encode(ids).cpu().numpy())
    assert b2q.check_device() == 0
