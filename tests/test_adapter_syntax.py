"""The ggml op-hook adapter (hbd-siglip2.cpp_b200/adapter/b2q_ggml_hook.cpp)
is built inside hbd-siglip2.cpp against its ggml fork, which is not present
here.  This checks that the file is well-formed C++ against a stand-in
ggml.h that declares only the public names the adapter uses (ggml_tensor's
type/op/ne/nb/src/data, the two type ids, GGML_OP_MUL_MAT,
ggml_is_contiguous)."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]

STAND_IN = """
#pragma once
#include <cstddef>
#include <cstdint>
enum ggml_type { GGML_TYPE_F32 = 0, GGML_TYPE_Q8_0 = 8 };
enum ggml_op { GGML_OP_NONE = 0, GGML_OP_MUL_MAT = 1 };
#define GGML_MAX_SRC 10
struct ggml_tensor {
    enum ggml_type type;
    int64_t ne[4];
    size_t nb[4];
    enum ggml_op op;
    struct ggml_tensor * src[GGML_MAX_SRC];
    void * data;
};
bool ggml_is_contiguous(const struct ggml_tensor * t);
"""


def test_adapter_is_well_formed(tmp_path):
    gxx = shutil.which("g++")
    if not gxx:
        pytest.skip("no g++")
    (tmp_path / "ggml.h").write_text(STAND_IN)
    cuda_inc = Path("/usr/local/cuda/include")
    cmd = [gxx, "-std=c++17", "-fsyntax-only", "-Wall", "-Werror", f"-I{tmp_path}", f"-I{ROOT / 'include'}",
           f"-I{cuda_inc}", str(ROOT / "hbd-siglip2.cpp_b200" / "adapter" / "b2q_ggml_hook.cpp")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
