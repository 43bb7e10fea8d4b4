"""GPU attention (head_dim 72, packed variable-length sequences) against the
CPU oracle's flash-attention restatement.

The oracle keeps K and V in fp16 (as the reference casts them,
src/siglip2_vision.cpp:164-165) and computes the softmax in double; the GPU
kernel also rounds Q and the probabilities to fp16 for its tensor-core
products, so the bar is a tolerance: max |err| <= 2e-3 and per-row cosine
>= 0.99999 on unit-scale inputs.
"""
import numpy as np
import pytest

import b2q

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

H, NH = 1152, 16


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    b2q.init(0)


@pytest.fixture(params=[0, 1], ids=["tcgen05", "mma_sync"])
def kernel(request, dev):
    """Both tensor-core kernels (B2Q_TUNE_ATTN_KERNEL) meet the same bar."""
    b2q.tune(b2q.TUNE_ATTN_KERNEL, request.param)
    yield request.param
    b2q.tune(b2q.TUNE_ATTN_KERNEL, 0)


def check_close(out, ref):
    err = np.abs(out - ref).max()
    cos = (out * ref).sum(1) / (np.linalg.norm(out, axis=1) * np.linalg.norm(ref, axis=1) + 1e-30)
    assert err <= 2e-3, err
    assert cos.min() >= 0.99999, cos.min()


@pytest.mark.parametrize("lens", [[1], [7], [64, 65], [127, 128, 129], [729], [1, 5, 100, 256, 1024], [3000]])
def test_self_attention_varlen(oracle, kernel, lens):
    rng = np.random.default_rng(len(lens) * 1000 + sum(lens))
    T = sum(lens)
    qkv = rng.standard_normal((T, 3 * H)).astype(np.float32)
    qkv16 = qkv.astype(np.float16)
    ref = oracle.attention(qkv16.astype(np.float32), NH, lens)
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]])
    t = torch.from_numpy(qkv16).cuda()
    out = torch.full((T, H), float("nan"), dtype=torch.float32, device="cuda")
    b2q.attention(t, 3 * H, t[:, H:], 3 * H, t[:, 2 * H:], 3 * H, offs, lens, offs, lens, offs, NH, out, H)
    torch.cuda.synchronize()
    check_close(out.cpu().numpy(), ref)


def test_large_logits(oracle, kernel):
    # scores spanning hundreds of units: the running max moves between key
    # tiles and most probabilities underflow
    rng = np.random.default_rng(11)
    lens = [300, 77]
    T = sum(lens)
    qkv = (rng.standard_normal((T, 3 * H)) * np.r_[np.full(H, 4.0), np.full(H, 4.0), np.ones(H)]).astype(np.float16)
    ref = oracle.attention(qkv.astype(np.float32), NH, lens)
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]])
    t = torch.from_numpy(qkv).cuda()
    out = torch.full((T, H), float("nan"), dtype=torch.float32, device="cuda")
    b2q.attention(t, 3 * H, t[:, H:], 3 * H, t[:, 2 * H:], 3 * H, offs, lens, offs, lens, offs, NH, out, H)
    torch.cuda.synchronize()
    check_close(out.cpu().numpy(), ref)


def test_probe_query_shared_row(oracle, kernel):
    # attention-pool head: one probe query (shared by every image) against each image's keys
    rng = np.random.default_rng(7)
    lens = [729, 300, 1]
    T = sum(lens)
    qrow = rng.standard_normal((1, H)).astype(np.float16)
    kv = rng.standard_normal((T, 2 * H)).astype(np.float16)
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]])
    q = torch.from_numpy(qrow).cuda()
    kvt = torch.from_numpy(kv).cuda()
    out = torch.zeros((len(lens), H), dtype=torch.float32, device="cuda")
    b2q.attention(q, H, kvt, 2 * H, kvt[:, H:], 2 * H, [0] * len(lens), [1] * len(lens), offs, lens,
                  list(range(len(lens))), NH, out, H)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for i, (o, L) in enumerate(zip(offs, lens)):
        packed = np.zeros((L + 1, 3 * H), np.float32)
        packed[:, :H] = qrow.astype(np.float32)
        packed[1:, H:] = kv[o:o + L].astype(np.float32)
        # oracle: query row 0 attends to keys 1..L -> run over rows 1..L with row-0 query replicated
        packed2 = np.concatenate([np.repeat(qrow.astype(np.float32), L, 0), kv[o:o + L].astype(np.float32)], 1)
        ref = oracle.attention(packed2, NH, [L])[0:1]
        check_close(got[i:i + 1], ref)


def test_attention_rejects_bad_head_dim(dev):
    t = torch.zeros((4, 3 * H), dtype=torch.float16, device="cuda")
    out = torch.zeros((4, H), dtype=torch.float32, device="cuda")
    import ctypes as C
    arr = (C.c_int32 * 1)(0)
    ln = (C.c_int32 * 1)(4)
    scratch = torch.empty(64, dtype=torch.uint8, device="cuda")
    st = b2q.lib().b2q_attention(t.data_ptr(), 3 * H, t.data_ptr(), 3 * H, t.data_ptr(), 3 * H, arr, ln, arr, ln,
                                 arr, 1, NH, 64, out.data_ptr(), H, scratch.data_ptr(), None)
    assert st == b2q.ERR_SHAPE
