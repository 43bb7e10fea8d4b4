"""GPU vision tower (C++ driver over the Q8_0 kernels) against the CPU oracle's
tower restatement on the same seeded synthetic checkpoint.

Two bars:
* exact attention mode (B2Q_TUNE_ATTN_EXACT): the whole tower, 27 layers and
  both poolings, is bit-identical to the oracle — every kernel follows the
  oracle's fixed fp32 operation order;
* default tensor-core attention (fp16 Q, K, V as in the reference, the
  softmax probabilities carried as two fp16 halves, fp32 accumulation):
  cosine >= 0.9999 (the project's pooled-embedding bar) and max-abs <= 0.05.
  Any arithmetic that is not bit-identical moves some q8_1 rounding decisions
  downstream, and over 27 layers that moves pooled values by ~0.025 (values
  of ~2).  The CPU suite measures exactly this between the oracle and the
  same tower evaluated with the reference kernels' own element rules (tanhf
  GELU, the 1024-thread LayerNorm order, half-away q8_1;
  test_oracle.py::test_reference_element_rules_drift): 0.024-0.028.  A
  max-abs bar of 2e-3 can therefore only be met bit-identically (the exact
  mode does, with 0), by the reference itself as much as by this library.
"""
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


def cos(a, b):
    return float(np.dot(a, b) / np.linalg.norm(a) / np.linalg.norm(b))


def run_tower(ck, grids, pooling, seed=0):
    cfg = ck.cfg
    tower = b2q.VisionTower(cfg)
    tower.load(ck)
    patches = [synth.patches(h * w, cfg.patch_dim, seed=seed + i) for i, (h, w) in enumerate(grids)]
    packed = torch.from_numpy(np.concatenate(patches)).cuda()
    out = tower.encode(packed, grids, pooling)
    torch.cuda.synchronize()
    assert b2q.check_device() == 0
    return tower, patches, out.cpu().numpy()


def assert_matches(oracle, ck, patches, grids, got, pooling, exact=False):
    for i, ((h, w), x) in enumerate(zip(grids, patches)):
        ref = oracle.vision_encode(ck, x, h, w, pooling=pooling, quant_act=True)
        if exact:
            np.testing.assert_array_equal(got[i], ref, err_msg=f"image {i} grid {(h, w)}")
            continue
        c, e = cos(got[i], ref), float(np.abs(got[i] - ref).max())
        assert c >= 0.9999 and e <= 0.05, (i, (h, w), c, e)


@pytest.fixture
def exact_attention(dev):
    b2q.tune(b2q.TUNE_ATTN_EXACT, 1)
    yield
    b2q.tune(b2q.TUNE_ATTN_EXACT, 0)


@pytest.mark.parametrize("pooling", [b2q.POOL_PROBE, b2q.POOL_MEAN])
def test_tower_bit_exact_small_batch(oracle, exact_attention, pooling):
    cfg = synth.TowerConfig(n_layer=3)
    ck = synth.vision_checkpoint(cfg, seed=11, bias_std=0.02, ln_std=0.1)
    grids = [(16, 16), (12, 20), (5, 9), (27, 27), (1, 3), (2, 40)]
    _, patches, got = run_tower(ck, grids, pooling)
    assert_matches(oracle, ck, patches, grids, got, pooling, exact=True)


def test_tower_bit_exact_full_depth(oracle, exact_attention):
    # all 27 layers at the position table's native 16x16 grid
    ck = synth.vision_checkpoint(synth.TowerConfig(), seed=0)
    grids = [(16, 16)]
    _, patches, got = run_tower(ck, grids, b2q.POOL_PROBE)
    assert_matches(oracle, ck, patches, grids, got, b2q.POOL_PROBE, exact=True)


@pytest.fixture(scope="module")
def grid27(oracle):
    """The batch-1 workload: one 27x27-patch image through all 27 layers,
    PROBE pooling, with its oracle embedding (computed once)."""
    ck = synth.vision_checkpoint(synth.TowerConfig(), seed=0)
    x = synth.patches(729, ck.cfg.patch_dim, seed=0)
    return ck, x, oracle.vision_encode(ck, x, 27, 27, pooling=b2q.POOL_PROBE, quant_act=True)


def test_tower_27x27_full_depth_bit_exact(grid27, exact_attention):
    ck, x, ref = grid27
    tower = b2q.VisionTower(ck.cfg)
    tower.load(ck)
    got = tower.encode(torch.from_numpy(x).cuda(), [(27, 27)], b2q.POOL_PROBE).cpu().numpy()
    assert b2q.check_device() == 0
    np.testing.assert_array_equal(got[0], ref)


def test_tower_27x27_full_depth_tensor_core(grid27, dev):
    ck, x, ref = grid27
    tower = b2q.VisionTower(ck.cfg)
    tower.load(ck)
    got = tower.encode(torch.from_numpy(x).cuda(), [(27, 27)], b2q.POOL_PROBE).cpu().numpy()
    assert b2q.check_device() == 0
    c, e = cos(got[0], ref), float(np.abs(got[0] - ref).max())
    assert c >= 0.9999 and e <= 0.05, (c, e)


@pytest.mark.parametrize("pooling", [b2q.POOL_PROBE, b2q.POOL_MEAN])
def test_tower_small_batch_varlen(oracle, dev, pooling):
    # tensor-core attention; degenerate few-patch images are covered by the
    # bit-exact tests above
    cfg = synth.TowerConfig(n_layer=3)
    ck = synth.vision_checkpoint(cfg, seed=11, bias_std=0.02, ln_std=0.1)
    grids = [(16, 16), (12, 20), (5, 9), (27, 27)]
    _, patches, got = run_tower(ck, grids, pooling)
    assert_matches(oracle, ck, patches, grids, got, pooling)


def test_tower_full_depth_one_image(oracle, dev):
    # all 27 layers at the position table's native 16x16 grid (256 patches)
    ck = synth.vision_checkpoint(synth.TowerConfig(), seed=0)
    grids = [(16, 16)]
    _, patches, got = run_tower(ck, grids, b2q.POOL_PROBE)
    assert_matches(oracle, ck, patches, grids, got, b2q.POOL_PROBE)


@pytest.mark.parametrize("kernel", [0, 1], ids=["tcgen05", "mma_sync"])
def test_tower_naflex_batch_fast_vs_exact(dev, kernel):
    # NaFlex batch geometry at reduced batch: 24 NaFlex images of 256-1024 patches
    # (the benchmark's grid generator), all 27 layers.  The exact attention
    # mode is bit-identical to the CPU restatement (tests above), so it serves
    # as the reference here; each tensor-core attention kernel must meet the
    # tower bar against it on every image.
    ck = synth.vision_checkpoint(synth.TowerConfig(), seed=3)
    grids = synth.naflex_grids(24, seed=7)
    b2q.tune(b2q.TUNE_ATTN_KERNEL, kernel)
    try:
        tower, patches, fast = run_tower(ck, grids, b2q.POOL_PROBE)
        b2q.tune(b2q.TUNE_ATTN_EXACT, 1)
        try:
            exact = tower.encode(torch.from_numpy(np.concatenate(patches)).cuda(), grids, b2q.POOL_PROBE).cpu().numpy()
        finally:
            b2q.tune(b2q.TUNE_ATTN_EXACT, 0)
    finally:
        b2q.tune(b2q.TUNE_ATTN_KERNEL, 0)
    for i, (h, w) in enumerate(grids):
        c, e = cos(fast[i], exact[i]), float(np.abs(fast[i] - exact[i]).max())
        assert c >= 0.9999 and e <= 0.05, (i, (h, w), c, e)


def test_tower_batching_is_exact(dev):
    # an image's embedding must not depend on what else is in the batch
    cfg = synth.TowerConfig(n_layer=2)
    ck = synth.vision_checkpoint(cfg, seed=5, bias_std=0.02, ln_std=0.1)
    grids = [(7, 11), (16, 16), (3, 30)]
    tower, patches, batch = run_tower(ck, grids, b2q.POOL_PROBE)
    for i, (h, w) in enumerate(grids):
        single = tower.encode(torch.from_numpy(patches[i]).cuda(), [(h, w)], b2q.POOL_PROBE).cpu().numpy()
        np.testing.assert_array_equal(single[0], batch[i])


def test_tower_host_entry_point(dev):
    cfg = synth.TowerConfig(n_layer=1)
    ck = synth.vision_checkpoint(cfg, seed=2)
    grids = [(4, 4), (2, 8)]
    tower, patches, dev_out = run_tower(ck, grids, b2q.POOL_PROBE)
    host_out = tower.encode_host(np.concatenate(patches), grids, b2q.POOL_PROBE)
    np.testing.assert_array_equal(host_out, dev_out)


def test_tower_missing_tensor_is_an_error(dev):
    cfg = synth.TowerConfig(n_layer=1)
    tower = b2q.VisionTower(cfg)
    x = torch.zeros((4, cfg.patch_dim), device="cuda")
    with pytest.raises(b2q.B2QError) as e:
        tower.encode(x, [(2, 2)], b2q.POOL_MEAN)
    assert e.value.status == b2q.ERR_INVALID
