"""The ggml op-hook adapter (hbd-siglip2.cpp_b200/adapter/b2q_ggml_hook.cpp)
is built inside hbd-siglip2.cpp against its ggml fork, which is not present
here.  On the CPU: it compiles and links (with -Wall -Werror) against a
stand-in ggml.h and a stub hook registrar, exports its three entry points,
and the stand-in tensor layout matches the ctypes view the GPU test uses."""
import ctypes as C

import pytest

import adapter_util as A


def test_adapter_builds_and_exports(tmp_path):
    try:
        so = A.build(tmp_path)
    except RuntimeError as e:
        if "no g++" in str(e):
            pytest.skip("no g++")
        raise
    L = A.load(so)
    for name in A.EXPORTS:
        assert hasattr(L, name)
    assert L.stub_tensor_size() == C.sizeof(A.GgmlTensor)
    assert L.stub_installed() == 0          # nothing installed until b2q_ggml_install
