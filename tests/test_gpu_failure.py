"""Failure detection on the GPU without a GPU fault: every wait inside the
GEMM and the tcgen05 attention is bounded.  With B2Q_TUNE_TEST_STALL the TMA producer issues nothing,
so the MMA issuer's wait for the first stage and the epilogue's wait for the
first accumulator run out (after the 1 ms limit set here), the CTA aborts its
other roles, releases TMEM and returns; the host
reads the code through b2q_check_device, and the context stays usable: the
next launch is bit-exact."""
import numpy as np
import pytest

import b2q
from b2q import synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_expired_wait_is_reported_and_context_survives(oracle):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    b2q.init(0)
    M, N, K = 512, 1152, 1152
    rng = np.random.default_rng(5)
    wq = synth.quantize_q8_0((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    x = rng.standard_normal((M, K)).astype(np.float32)
    W = b2q.Weight(wq, N, K)
    act = b2q.act_empty(M, K)
    b2q.quantize_q8_1(torch.from_numpy(x).cuda(), act, M, K)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    try:
        b2q.tune(b2q.TUNE_TIMEOUT_NS, 1_000_000)
        b2q.tune(b2q.TUNE_TEST_STALL, 1)
        b2q.mul_mat(W, act, M, y)
        with pytest.raises(b2q.B2QError) as e:
            b2q.check_device()
        # the MMA issuer (code 1) or an epilogue warp (code 3) reports first
        assert e.value.status == b2q.ERR_DEVICE and "wait expired" in str(e.value)
    finally:
        b2q.tune(b2q.TUNE_TEST_STALL, 0)
        b2q.tune(b2q.TUNE_TIMEOUT_NS, 2_000_000_000)
    assert b2q.check_device() == 0
    b2q.mul_mat(W, act, M, y)
    torch.cuda.synchronize()
    assert b2q.check_device() == 0
    qs, d = oracle.quantize_q8_1(x, K)
    np.testing.assert_array_equal(y.cpu().numpy(), oracle.gemm_q8(wq, N, K, qs, d))
    W.release()


def test_attention_expired_wait_is_reported_and_context_survives(oracle):
    # the attention's MMA issuer idles: every thread's wait for the score
    # tile expires, the CTA leaves its key loop together, releases TMEM and
    # returns; the next launch is correct
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    b2q.init(0)
    H, NH, lens = 1152, 16, [200, 64]
    T = sum(lens)
    rng = np.random.default_rng(9)
    qkv = rng.standard_normal((T, 3 * H)).astype(np.float16)
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]])
    t = torch.from_numpy(qkv).cuda()
    out = torch.zeros((T, H), dtype=torch.float32, device="cuda")

    def run():
        b2q.attention(t, 3 * H, t[:, H:], 3 * H, t[:, 2 * H:], 3 * H, offs, lens, offs, lens, offs, NH, out, H)

    b2q.tune(b2q.TUNE_ATTN_KERNEL, 0)
    try:
        b2q.tune(b2q.TUNE_TIMEOUT_NS, 1_000_000)
        b2q.tune(b2q.TUNE_TEST_STALL, 1)
        run()
        with pytest.raises(b2q.B2QError) as e:
            b2q.check_device()
        assert e.value.status == b2q.ERR_DEVICE and "wait expired" in str(e.value)
    finally:
        b2q.tune(b2q.TUNE_TEST_STALL, 0)
        b2q.tune(b2q.TUNE_TIMEOUT_NS, 2_000_000_000)
    assert b2q.check_device() == 0
    run()
    torch.cuda.synchronize()
    assert b2q.check_device() == 0
    ref = oracle.attention(qkv.astype(np.float32), NH, lens)
    got = out.cpu().numpy()
    assert np.abs(got - ref).max() <= 2e-3
