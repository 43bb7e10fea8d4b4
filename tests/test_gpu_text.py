"""GPU text tower (C++ driver, b2q_text_*) and image-text scoring (b2q_score)
against the CPU oracle on seeded synthetic checkpoints.

The text tower always runs the fixed-order fp32 attention, so its pooled
embeddings are bit-identical to the oracle whatever B2Q_TUNE_ATTN_EXACT says.
Scoring is bit-identical too (double-precision dots in the oracle's column
order, the library's own exp and division in the sigmoid).
"""
import math

import numpy as np
import pytest

import b2q
from b2q import synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    b2q.init(0)


@pytest.fixture
def exact_attention(dev):
    b2q.tune(b2q.TUNE_ATTN_EXACT, 1)
    yield
    b2q.tune(b2q.TUNE_ATTN_EXACT, 0)


@pytest.fixture(scope="module")
def config3(dev):
    """Full text tower: 27 layers, vocab 256000, 5 prompts x 64 ids."""
    cfg = synth.TowerConfig()
    ck = synth.text_checkpoint(cfg, seed=7)
    ids = synth.token_ids(5, cfg.n_pos, cfg.vocab, seed=1)
    tower = b2q.TextTower(cfg)
    tower.load(ck)
    return ck, ids, tower


def encode(tower, ids):
    out = tower.encode(torch.from_numpy(np.ascontiguousarray(ids, np.int32)).cuda())
    torch.cuda.synchronize()
    assert b2q.check_device() == 0
    return out.cpu().numpy()


def test_text_bit_exact_small(oracle, dev):
    cfg = synth.TowerConfig(n_layer=2, vocab=1000)
    ck = synth.text_checkpoint(cfg, seed=5, bias_std=0.02, ln_std=0.1)
    ids = synth.token_ids(3, cfg.n_pos, cfg.vocab, seed=2)
    tower = b2q.TextTower(cfg)
    tower.load(ck)
    got = encode(tower, ids)
    np.testing.assert_array_equal(got, oracle.text_encode(ck, ids))
    # one prompt alone gives the same row (prompts are independent sequences)
    np.testing.assert_array_equal(encode(tower, ids[1:2])[0], got[1])


def test_text_config3_bit_exact_exact_mode(oracle, exact_attention, config3):
    ck, ids, tower = config3
    np.testing.assert_array_equal(encode(tower, ids), oracle.text_encode(ck, ids))


def test_text_config3_bit_exact_default_mode(oracle, dev, config3):
    # the device's attention setting is the tensor-core default here
    ck, ids, tower = config3
    np.testing.assert_array_equal(encode(tower, ids), oracle.text_encode(ck, ids))


def test_text_host_entry_matches_device_entry(config3):
    _, ids, tower = config3
    np.testing.assert_array_equal(tower.encode_host(ids), encode(tower, ids))


def test_text_bad_token_id_is_reported(config3):
    _, ids, tower = config3
    bad = ids.copy()
    bad[0, 3] = 256000
    tower.encode(torch.from_numpy(bad).cuda())
    torch.cuda.synchronize()
    with pytest.raises(b2q.B2QError) as e:
        b2q.check_device()
    assert e.value.status == b2q.ERR_DEVICE and "vocabulary" in str(e.value)
    assert b2q.check_device() == 0          # the word is cleared by the read


@pytest.mark.parametrize("I,J,H", [(1, 1, 1152), (37, 23, 1152), (64, 100, 1152), (5, 3, 40)])
def test_score_bit_exact(oracle, dev, I, J, H):
    rng = np.random.default_rng(I * 100 + J)
    img = rng.standard_normal((I, H)).astype(np.float32)
    txt = rng.standard_normal((J, H)).astype(np.float32)
    img[0] *= 1e-3                          # a short vector: the normalisation still applies
    lg, pr = b2q.score(torch.from_numpy(img).cuda(), torch.from_numpy(txt).cuda(), math.log(10.0), -10.0)
    ref_p, ref_l = oracle.score(img, txt, math.log(10.0), -10.0, with_logits=True)
    np.testing.assert_array_equal(lg.cpu().numpy(), ref_l)
    np.testing.assert_array_equal(pr.cpu().numpy(), ref_p)


def test_zero_shot_chain_bit_exact(oracle, exact_attention):
    """Config-5 chain at small size: vision tower (PROBE) and text tower on the
    GPU, then scoring, against the oracle's chain."""
    cfg = synth.TowerConfig(n_layer=2, vocab=500)
    vck = synth.vision_checkpoint(cfg, seed=21, bias_std=0.02, ln_std=0.1)
    tck = synth.text_checkpoint(cfg, seed=22, bias_std=0.02, ln_std=0.1)
    grids = [(27, 27), (16, 16), (9, 12)]
    patches = [synth.patches(h * w, cfg.patch_dim, seed=30 + i) for i, (h, w) in enumerate(grids)]
    ids = synth.token_ids(4, cfg.n_pos, cfg.vocab, seed=4)
    vt, tt = b2q.VisionTower(cfg), b2q.TextTower(cfg)
    vt.load(vck)
    tt.load(tck)
    img = vt.encode(torch.from_numpy(np.concatenate(patches)).cuda(), grids, b2q.POOL_PROBE)
    txt = tt.encode(torch.from_numpy(ids).cuda())
    _, probs = b2q.score(img, txt, math.log(10.0), -10.0, logits=False)
    torch.cuda.synchronize()
    assert b2q.check_device() == 0
    img_ref = np.stack([oracle.vision_encode(vck, x, h, w, pooling=1) for (h, w), x in zip(grids, patches)])
    txt_ref = oracle.text_encode(tck, ids)
    np.testing.assert_array_equal(probs.cpu().numpy(), oracle.score(img_ref, txt_ref, math.log(10.0), -10.0))
