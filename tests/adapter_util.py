"""Builds the ggml op-hook adapter (hbd-siglip2.cpp_b200/adapter) together
with the stand-ins of tests/adapter_stub into a shared library, and the
ctypes view of the stand-in ggml_tensor."""
import ctypes as C
import shutil
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
STUB = ROOT / "tests" / "adapter_stub"
LIBDIR = ROOT / "hbd-siglip2.cpp_b200" / "lib"
EXPORTS = ["b2q_ggml_install", "b2q_ggml_set_scratch", "b2q_ggml_release_weights"]

GGML_TYPE_F32, GGML_TYPE_F16, GGML_TYPE_Q8_0 = 0, 1, 8
GGML_OP_NONE, GGML_OP_ADD, GGML_OP_MUL_MAT = 0, 2, 29


class GgmlTensor(C.Structure):
    _fields_ = [("type", C.c_int), ("ne", C.c_int64 * 4), ("nb", C.c_size_t * 4), ("op", C.c_int),
                ("src", C.c_void_p * 10), ("data", C.c_void_p)]


def build(out_dir: Path) -> Path:
    gxx = shutil.which("g++")
    if not gxx:
        raise RuntimeError("no g++")
    out = out_dir / "libb2q_ggml_hook_test.so"
    cmd = [gxx, "-std=c++17", "-O2", "-fPIC", "-shared", "-Wall", "-Werror", f"-I{STUB}", f"-I{ROOT / 'include'}",
           "-I/usr/local/cuda/include", str(ROOT / "hbd-siglip2.cpp_b200" / "adapter" / "b2q_ggml_hook.cpp"),
           str(STUB / "stub.cpp"), f"-L{LIBDIR}", "-lb2q", f"-Wl,-rpath,{LIBDIR}", "-L/usr/local/cuda/lib64",
           "-lcudart", "-o", str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(r.stderr)
    return out


def load(path: Path):
    L = C.CDLL(str(path))
    L.b2q_ggml_install.argtypes = [C.c_int]
    L.b2q_ggml_install.restype = C.c_bool
    L.b2q_ggml_set_scratch.argtypes = [C.c_void_p, C.c_size_t]
    L.b2q_ggml_release_weights.argtypes = []
    L.stub_run_op.argtypes = [C.POINTER(GgmlTensor), C.c_void_p]
    L.stub_tensor_size.restype = C.c_size_t
    return L
