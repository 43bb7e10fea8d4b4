"""CPU tests of the C ABI boundary: the library loads, exports every symbol
include/b2q.h declares, and rejects calls before b2q_init with a status code
(no GPU needed; nothing here launches a kernel)."""
import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def header_symbols():
    text = (ROOT / "include" / "b2q.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b2q_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    import b2q
    assert header_symbols() == sorted(b2q.EXPORTS)


def test_library_exports_every_symbol():
    import b2q
    if not b2q.LIB_PATH.exists():
        pytest.skip("libb2q.so not built")
    L = C.CDLL(str(b2q.LIB_PATH))
    for name in header_symbols():
        assert hasattr(L, name), name


def test_calls_before_init_fail_cleanly():
    import b2q
    if not b2q.LIB_PATH.exists():
        pytest.skip("libb2q.so not built")
    L = b2q.lib()
    assert L.b2q_abi_version() == 1
    st = L.b2q_quantize_q8_1(None, 4, 32, 32, None, None)
    assert st in (b2q.ERR_NOT_INIT, b2q.ERR_INVALID)
    st = L.b2q_mul_mat_q8_0(None, None, 4, None, None, None)
    assert st in (b2q.ERR_NOT_INIT, b2q.ERR_INVALID)
    assert L.b2q_last_error()
    assert L.b2q_weight_release(None) == b2q.OK
