"""The ggml op-hook adapter executed on the GPU: built with the stand-ins of
tests/adapter_stub (the fork's hook registrar and the reference megakernel's
two hooks, which count the calls that reach them), installed, and driven the
way ggml-cuda's node loop drives it, with stand-in ggml_tensor nodes whose
data live in device memory.

Checks: a Q8_0 MUL_MAT node is computed by libb2q on ggml's stream and
matches the CPU oracle bit-exactly (also the K-padded fc2 form); every other
node, and a mul_mat the library does not take, reaches the reference's hook;
the graph-begin hook is forwarded; after b2q_ggml_release_weights new weights
at the same address are used (no stale repack); a second host thread without
its own scratch does not touch the shared no-alloc array but gets its node
back (false), and computes it once it registers scratch."""
import ctypes as C
import threading

import numpy as np
import pytest

import adapter_util as A
import b2q
from b2q import synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def hook(tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    b2q.init(0)
    L = A.load(A.build(tmp_path_factory.mktemp("adapter")))
    assert L.b2q_ggml_install(0)
    assert L.stub_installed() == 1
    return L


@pytest.fixture(autouse=True)
def unload_between_tests(hook):
    # each test is a model load: its weight buffers are freed afterwards and
    # the allocator may hand their addresses to the next test, so the cached
    # registrations are dropped the way the reference's unload path drops them
    yield
    torch.cuda.synchronize()
    hook.b2q_ggml_release_weights()


def tensor(ttype, ne, data, op=A.GGML_OP_NONE, src=()):
    t = A.GgmlTensor()
    t.type, t.op = ttype, op
    for i in range(4):
        t.ne[i] = ne[i] if i < len(ne) else 1
    if ttype == A.GGML_TYPE_Q8_0:
        row = ne[0] // 32 * 34
        nb = [34, row, row * ne[1], row * ne[1]]
    else:
        es = 4 if ttype == A.GGML_TYPE_F32 else 2
        nb = [es, es * t.ne[0], es * t.ne[0] * t.ne[1], es * t.ne[0] * t.ne[1] * t.ne[2]]
    for i in range(4):
        t.nb[i] = nb[i]
    for i, s in enumerate(src):
        t.src[i] = C.cast(C.pointer(s), C.c_void_p)
    t.data = data
    return t


def mul_mat_node(w_dev, N, Kp, x_dev, M, K, y_dev, wtype=A.GGML_TYPE_Q8_0):
    W = tensor(wtype, (Kp, N), w_dev.data_ptr())
    X = tensor(A.GGML_TYPE_F32, (K, M), x_dev.data_ptr())
    D = tensor(A.GGML_TYPE_F32, (N, M), y_dev.data_ptr(), op=A.GGML_OP_MUL_MAT, src=(W, X))
    return W, X, D


def stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def case(oracle, M, N, K, Kp, seed):
    rng = np.random.default_rng(seed)
    w_q = synth.quantize_q8_0((rng.standard_normal((N, K)) * 0.02).astype(np.float32), Kp)
    x = rng.standard_normal((M, K)).astype(np.float32)
    qs, dx = oracle.quantize_q8_1(x, Kp)
    return w_q, x, oracle.gemm_q8(w_q, N, Kp, qs, dx)


@pytest.mark.parametrize("M,N,K,Kp", [(37, 1152, 1152, 1152), (20, 1152, 4304, 4320)], ids=["qkv-like", "fc2-padded"])
def test_q8_0_mul_mat_is_claimed_and_exact(oracle, hook, M, N, K, Kp):
    w_q, x, ref = case(oracle, M, N, K, Kp, M + N)
    w_dev = torch.from_numpy(w_q.reshape(-1)).cuda()
    x_dev = torch.from_numpy(x).cuda()
    y_dev = torch.zeros((M, N), device="cuda")
    nodes = mul_mat_node(w_dev, N, Kp, x_dev, M, K, y_dev)
    before = hook.stub_ref_op_calls()
    assert hook.stub_run_op(C.byref(nodes[2]), stream()) == 1
    torch.cuda.synchronize()
    assert b2q.check_device() == 0
    assert hook.stub_ref_op_calls() == before          # the reference's hook never saw it
    np.testing.assert_array_equal(y_dev.cpu().numpy(), ref)


def test_other_nodes_reach_the_reference_hook(oracle, hook):
    M, N, K = 8, 64, 64
    x_dev = torch.zeros((M, K), device="cuda")
    y_dev = torch.zeros((M, N), device="cuda")
    before = hook.stub_ref_op_calls()
    # an element-wise node
    add = tensor(A.GGML_TYPE_F32, (N, M), y_dev.data_ptr(), op=A.GGML_OP_ADD)
    assert hook.stub_run_op(C.byref(add), stream()) == 0
    # a mul_mat with an F16 weight is not this library's
    w16 = torch.zeros((N, K), dtype=torch.float16, device="cuda")
    nodes = mul_mat_node(w16, N, K, x_dev, M, K, y_dev, wtype=A.GGML_TYPE_F16)
    assert hook.stub_run_op(C.byref(nodes[2]), stream()) == 0
    assert hook.stub_ref_op_calls() == before + 2
    b0 = hook.stub_ref_begin_calls()
    hook.stub_run_begin()
    assert hook.stub_ref_begin_calls() == b0 + 1


def test_reload_at_the_same_address_uses_the_new_weights(oracle, hook):
    M, N, K = 16, 256, 1152
    w1, x, ref1 = case(oracle, M, N, K, K, 1)
    w2, _, _ = case(oracle, M, N, K, K, 2)
    qs, dx = oracle.quantize_q8_1(x, K)
    ref2 = oracle.gemm_q8(w2, N, K, qs, dx)
    w_dev = torch.from_numpy(w1.reshape(-1)).cuda()
    x_dev = torch.from_numpy(x).cuda()
    y_dev = torch.zeros((M, N), device="cuda")
    nodes = mul_mat_node(w_dev, N, K, x_dev, M, K, y_dev)
    assert hook.stub_run_op(C.byref(nodes[2]), stream()) == 1
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y_dev.cpu().numpy(), ref1)
    # encoder unload, then a reload whose weights land at the same address
    hook.b2q_ggml_release_weights()
    w_dev.copy_(torch.from_numpy(w2.reshape(-1)))
    assert hook.stub_run_op(C.byref(nodes[2]), stream()) == 1
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y_dev.cpu().numpy(), ref2)


def test_second_thread_needs_its_own_scratch(oracle, hook):
    M, N, K = 24, 128, 1152
    w_q, x, ref = case(oracle, M, N, K, K, 3)
    w_dev = torch.from_numpy(w_q.reshape(-1)).cuda()
    x_dev = torch.from_numpy(x).cuda()
    # this (first) thread already owns the device's shared no-alloc array
    y0 = torch.zeros((M, N), device="cuda")
    nodes0 = mul_mat_node(w_dev, N, K, x_dev, M, K, y0)
    assert hook.stub_run_op(C.byref(nodes0[2]), stream()) == 1
    result = {}

    def other():
        torch.cuda.set_device(0)
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            y = torch.zeros((M, N), device="cuda")
            nodes = mul_mat_node(w_dev, N, K, x_dev, M, K, y)
            result["without"] = hook.stub_run_op(C.byref(nodes[2]), C.c_void_p(s.cuda_stream))
            scratch = b2q.act_empty(M, K)
            hook.b2q_ggml_set_scratch(C.c_void_p(scratch.data_ptr()), scratch.numel())
            result["with"] = hook.stub_run_op(C.byref(nodes[2]), C.c_void_p(s.cuda_stream))
            s.synchronize()
            result["y"] = y.cpu().numpy()
            hook.b2q_ggml_set_scratch(None, 0)

    t = threading.Thread(target=other)
    t.start()
    t.join(timeout=120)
    torch.cuda.synchronize()
    assert result["without"] == 0 and result["with"] == 1
    np.testing.assert_array_equal(result["y"], ref)
    np.testing.assert_array_equal(y0.cpu().numpy(), ref)
