"""The no-allocation ggml_mul_mat entry point (b2q_mul_mat_q8_0_f32_noalloc).

Callers that cannot allocate device memory (an op hook inside another
framework's graph executor sees only the op's tensors and must not call
cudaMalloc mid-graph) use this variant: its q8_1 scratch is a fixed array in
the library.  This file is named to be collected last, so a run that stops at
the first failure has run every other test first; it also passes on its own
in a fresh process (it sets the device up itself).
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


def one_call(w_q, n, kp, x, k):
    """Run the same GEMM through the scratch-taking entry point and the
    no-alloc one; return both outputs."""
    m = x.shape[0]
    W = b2q.Weight(w_q, n, kp)
    xd = torch.from_numpy(x).cuda()
    ref = torch.empty((m, n), dtype=torch.float32, device="cuda")
    b2q.mul_mat_f32(W, xd, m, k, ref, b2q.act_empty(m, kp))
    got = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    b2q.mul_mat_f32_noalloc(W, xd, m, k, got)
    torch.cuda.synchronize()
    assert b2q.check_device() == 0
    return got.cpu().numpy(), ref.cpu().numpy()


def test_noalloc_matches_scratch_entry_point_twice(dev):
    rng = np.random.default_rng(0)
    # first call: fc2 shape with the K padding 4304 -> 4320
    w1 = synth.quantize_q8_0(rng.standard_normal((1152, 4304)).astype(np.float32) * 0.02, 4320)
    x1 = rng.standard_normal((700, 4304)).astype(np.float32)
    got, ref = one_call(w1, 1152, 4320, x1, 4304)
    np.testing.assert_array_equal(got, ref)
    # second call, different shape: the shared scratch keeps the first call's
    # contents and must not leak into this result
    w2 = synth.quantize_q8_0(rng.standard_normal((3456, 1152)).astype(np.float32) * 0.02)
    x2 = rng.standard_normal((129, 1152)).astype(np.float32)
    got, ref = one_call(w2, 3456, 1152, x2, 1152)
    np.testing.assert_array_equal(got, ref)


def test_noalloc_rejects_sizes_beyond_the_scratch(dev):
    rng = np.random.default_rng(1)
    w = synth.quantize_q8_0(rng.standard_normal((64, 4320)).astype(np.float32) * 0.02)
    W = b2q.Weight(w, 64, 4320)
    m = b2q.NOALLOC_MAX_SCRATCH_BYTES // 4320 + 1      # more than the array holds
    x = torch.zeros((m, 4320), dtype=torch.float32, device="cuda")
    y = torch.empty((m, 64), dtype=torch.float32, device="cuda")
    with pytest.raises(b2q.B2QError) as e:
        b2q.mul_mat_f32_noalloc(W, x, m, 4320, y)
    assert e.value.status == b2q.ERR_SHAPE
    assert "no-alloc" in str(e.value)
