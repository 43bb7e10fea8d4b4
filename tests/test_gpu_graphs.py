"""Tower encodes replayed as CUDA graphs (B2Q_TUNE_GRAPHS, on by default).

A call that repeats the previous call's geometry, buffers and settings is
captured once and then replayed.  Every replay must give exactly the bytes
the kernels give when launched one by one, must read the live contents of
its input buffers, and must be dropped when a setting, a tensor or the
geometry changes.  The library's graph-launch counter shows which calls ran
as a graph.
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
    yield
    b2q.tune(b2q.TUNE_GRAPHS, 1)
    b2q.tune(b2q.TUNE_GEMM_CTAS, 0)


@pytest.fixture(scope="module")
def vision(dev):
    cfg = synth.TowerConfig(n_layer=3)
    ck = synth.vision_checkpoint(cfg, seed=3, bias_std=0.02, ln_std=0.1)
    tower = b2q.VisionTower(cfg)
    tower.load(ck)
    return cfg, ck, tower


GRIDS = [(16, 16), (20, 12), (9, 31)]


def _patches(cfg, grids, seed):
    return torch.from_numpy(synth.patches(sum(h * w for h, w in grids), cfg.patch_dim, seed=seed)).cuda()


def _direct(tower, x, grids, pooling, out):
    """The same encode with the kernels launched one by one."""
    b2q.tune(b2q.TUNE_GRAPHS, 0)
    tower.encode(x, grids, pooling, out=out)
    torch.cuda.synchronize()
    assert b2q.check_device() == 0
    b2q.tune(b2q.TUNE_GRAPHS, 1)
    return out.clone()


def test_vision_replay_is_bit_identical_and_counted(vision):
    cfg, _, tower = vision
    x = _patches(cfg, GRIDS, seed=4)
    out = torch.empty((len(GRIDS), cfg.hidden), device="cuda")
    ref = _direct(tower, x, GRIDS, b2q.POOL_PROBE, out)
    g0 = b2q.graph_launch_count()
    kernels = []
    for call in range(4):   # direct, captured (and launched), replayed, replayed
        out.zero_()
        c0 = b2q.launch_count()
        tower.encode(x, GRIDS, b2q.POOL_PROBE, out=out)
        torch.cuda.synchronize()
        kernels.append(b2q.launch_count() - c0)
        assert b2q.check_device() == 0
        assert torch.equal(out, ref), call
    assert b2q.graph_launch_count() - g0 == 3
    # the launch counter reports the graph's kernels on every replay
    assert kernels[0] > 0 and len(set(kernels)) == 1, kernels


def test_vision_replay_reads_live_inputs(vision):
    cfg, _, tower = vision
    x = _patches(cfg, GRIDS, seed=5)
    x1, x2 = x.clone(), _patches(cfg, GRIDS, seed=6)
    out = torch.empty((len(GRIDS), cfg.hidden), device="cuda")
    ref1 = _direct(tower, x, GRIDS, b2q.POOL_MEAN, out)
    x.copy_(x2)
    ref2 = _direct(tower, x, GRIDS, b2q.POOL_MEAN, out)
    assert not torch.equal(ref1, ref2)
    g0 = b2q.graph_launch_count()
    for call, (src, ref) in enumerate([(x1, ref1), (x2, ref2), (x1, ref1), (x2, ref2), (x1, ref1)]):
        x.copy_(src)   # same buffer, new contents
        tower.encode(x, GRIDS, b2q.POOL_MEAN, out=out)
        torch.cuda.synchronize()
        assert b2q.check_device() == 0
        assert torch.equal(out, ref), call
    assert b2q.graph_launch_count() - g0 == 4


def test_vision_graph_dropped_on_changes(vision):
    cfg, ck, tower = vision
    grids2 = [(27, 27)]
    x = _patches(cfg, GRIDS, seed=7)
    y = _patches(cfg, grids2, seed=8)
    out = torch.empty((len(GRIDS), cfg.hidden), device="cuda")
    out2 = torch.empty((1, cfg.hidden), device="cuda")
    ref = _direct(tower, x, GRIDS, b2q.POOL_PROBE, out)
    ref2 = _direct(tower, y, grids2, b2q.POOL_PROBE, out2)

    def run(inp, grids, o):
        tower.encode(inp, grids, b2q.POOL_PROBE, out=o)
        torch.cuda.synchronize()
        assert b2q.check_device() == 0
        return o.clone()

    for _ in range(3):
        assert torch.equal(run(x, GRIDS, out), ref)
    # another geometry, then back: each change runs directly, then recaptures
    for _ in range(3):
        assert torch.equal(run(y, grids2, out2), ref2)
    for _ in range(3):
        assert torch.equal(run(x, GRIDS, out), ref)
    # a setting that changes which kernels run (bit-identical by design)
    b2q.tune(b2q.TUNE_GEMM_CTAS, 1)
    try:
        g0 = b2q.graph_launch_count()
        for _ in range(3):
            assert torch.equal(run(x, GRIDS, out), ref)
        assert b2q.graph_launch_count() - g0 == 2
    finally:
        b2q.tune(b2q.TUNE_GEMM_CTAS, 0)
    # reloading a tensor with other values must not replay the old graph
    w = ck.f32("v.post_ln.bias")
    tower.set_tensor("v.post_ln.bias", w + 0.5)
    try:
        changed = run(x, GRIDS, out)
        assert not torch.equal(changed, ref)
        assert torch.equal(run(x, GRIDS, out), changed)
        assert torch.equal(run(x, GRIDS, out), changed)
    finally:
        tower.set_tensor("v.post_ln.bias", w)
    assert torch.equal(run(x, GRIDS, out), ref)


def test_vision_host_entry_point_replays(vision):
    cfg, _, tower = vision
    x = synth.patches(sum(h * w for h, w in GRIDS), cfg.patch_dim, seed=9)
    out = torch.empty((len(GRIDS), cfg.hidden), device="cuda")
    ref = _direct(tower, torch.from_numpy(x).cuda(), GRIDS, b2q.POOL_PROBE, out).cpu().numpy()
    g0 = b2q.graph_launch_count()
    for call in range(4):
        got = tower.encode_host(x, GRIDS, b2q.POOL_PROBE)
        assert b2q.check_device() == 0
        np.testing.assert_array_equal(got, ref, err_msg=f"call {call}")
    assert b2q.graph_launch_count() - g0 == 3


def test_text_replay_is_bit_identical(dev, oracle):
    cfg = synth.TowerConfig(n_layer=2, vocab=1000)
    ck = synth.text_checkpoint(cfg, seed=11, bias_std=0.02, ln_std=0.1)
    tower = b2q.TextTower(cfg)
    tower.load(ck)
    ids1 = synth.token_ids(3, cfg.n_pos, cfg.vocab, seed=12)
    ids2 = synth.token_ids(3, cfg.n_pos, cfg.vocab, seed=13)
    ref1, ref2 = oracle.text_encode(ck, ids1), oracle.text_encode(ck, ids2)
    ids = torch.from_numpy(np.ascontiguousarray(ids1, np.int32)).cuda()
    out = torch.empty((3, cfg.hidden), device="cuda")
    g0 = b2q.graph_launch_count()
    for call, (src, ref) in enumerate([(ids1, ref1), (ids2, ref2), (ids1, ref1), (ids2, ref2)]):
        ids.copy_(torch.from_numpy(np.ascontiguousarray(src, np.int32)))
        tower.encode(ids, out=out)
        torch.cuda.synchronize()
        assert b2q.check_device() == 0
        np.testing.assert_array_equal(out.cpu().numpy(), ref, err_msg=f"call {call}")
    assert b2q.graph_launch_count() - g0 == 3


def test_caller_capture_records_the_kernels(vision):
    """Inside the caller's own capture the library launches its kernels into
    that capture (its own graph cache stays out of it)."""
    cfg, _, tower = vision
    x = _patches(cfg, GRIDS, seed=14)
    out = torch.empty((len(GRIDS), cfg.hidden), device="cuda")
    ref = _direct(tower, x, GRIDS, b2q.POOL_PROBE, out)
    for _ in range(2):   # the library's own graph exists for this key now
        tower.encode(x, GRIDS, b2q.POOL_PROBE, out=out)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    g0 = b2q.graph_launch_count()
    with torch.cuda.graph(g, stream=side):
        tower.encode(x, GRIDS, b2q.POOL_PROBE, out=out)
    assert b2q.graph_launch_count() == g0   # no graph of its own launched into the capture
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert b2q.check_device() == 0
    assert torch.equal(out, ref)


def test_vision_pipelined_submit_matches_encode_host(vision):
    """b2q_vision_submit_host: two slots in flight, uploads overlapping the
    other slot's encode; every result equals the synchronous entry point's."""
    cfg, _, tower = vision
    T = sum(h * w for h, w in GRIDS)
    inputs = [torch.from_numpy(synth.patches(T, cfg.patch_dim, seed=20 + i)).pin_memory() for i in range(3)]
    refs = [tower.encode_host(x.numpy(), GRIDS, b2q.POOL_PROBE) for x in inputs]
    assert b2q.check_device() == 0
    outs = [torch.empty((len(GRIDS), cfg.hidden), dtype=torch.float32).pin_memory() for _ in range(7)]
    order = [0, 1, 2, 0, 1, 2, 0]
    for i, o in zip(order, outs[:4]):
        tower.submit_host(inputs[i], GRIDS, o)
    tower.wait()
    for i, o in zip(order[4:], outs[4:]):
        tower.submit_host(inputs[i], GRIDS, o)
    tower.wait()
    assert b2q.check_device() == 0
    for n, (i, o) in enumerate(zip(order, outs)):
        np.testing.assert_array_equal(o.numpy(), refs[i], err_msg=f"submission {n}")


def test_vision_wait_submitted_orders_the_results(vision):
    """b2q_vision_wait_submitted(back=1) hands over the batch before the latest
    submission while the latest one still runs; each batch's embeddings equal
    the synchronous entry point's."""
    cfg, _, tower = vision
    T = sum(h * w for h, w in GRIDS)
    inputs = [torch.from_numpy(synth.patches(T, cfg.patch_dim, seed=30 + i)).pin_memory() for i in range(2)]
    refs = [tower.encode_host(x.numpy(), GRIDS, b2q.POOL_PROBE) for x in inputs]
    outs = [torch.empty((len(GRIDS), cfg.hidden), dtype=torch.float32).pin_memory() for _ in range(2)]
    order = [0, 1, 1, 0, 0, 1]
    for i, src in enumerate(order):
        tower.submit_host(inputs[src], GRIDS, outs[i % 2])
        if i > 0:
            tower.wait_submitted(1)
            np.testing.assert_array_equal(outs[(i - 1) % 2].numpy(), refs[order[i - 1]], err_msg=f"batch {i - 1}")
    tower.wait_submitted(0)
    np.testing.assert_array_equal(outs[(len(order) - 1) % 2].numpy(), refs[order[-1]])
    assert b2q.check_device() == 0
