"""Generate tests/golden/gemm_small.npz: known-answer vectors for the Q8_0 x
q8_1 GEMM at small shapes, produced by the CPU oracle (oracle/), whose Q8_0
codec is itself pinned to gguf-py by q8_0_gguf.npz.

Per case (M, N, K, Kp): the Q8_0 bytes of seeded N(0, 0.02) weight rows,
the seeded fp32 activations, the q8_1 planes (int8 values, fp32 scales), the
int32 block sums S[m][n][kb] and the fp32 output in the canonical order.  The
CPU suite checks that the oracle still reproduces every vector; the GPU suite
checks the CUDA path against the stored vectors directly.

Run from the repository root:  python tests/golden/make_gemm_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "hbd-siglip2.cpp_b200"))
sys.path.insert(0, str(ROOT / "oracle"))
from b2q import synth  # noqa: E402

OUT = Path(__file__).resolve().parent / "gemm_small.npz"

# (M, N, K, Kp): M covers 1, ragged and >128 rows; N the 16/80 tails; K one
# block, the width, and the fc2 width padded 4304 -> 4320.
CASES = [(1, 16, 32, 32), (7, 80, 1152, 1152), (8, 16, 4304, 4320), (129, 16, 96, 96),
         (3, 16, 768, 768)]


def main():
    import oracle as O
    O.build()
    out = {"cases": np.array(CASES, np.int64)}
    for i, (M, N, K, Kp) in enumerate(CASES):
        rng = np.random.default_rng(100 + i)
        w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        x = rng.standard_normal((M, K)).astype(np.float32)
        if i == 0:
            x[0, :] = 0.0                      # an all-zero activation block: d = 0, q = 0
        wq = synth.quantize_q8_0(w, Kp)
        qs, d = O.quantize_q8_1(x, Kp)
        y, s = O.gemm_q8(wq, N, Kp, qs, d, block_sums=True)
        out.update({f"wq{i}": wq, f"x{i}": x, f"qs{i}": qs, f"d{i}": d, f"s{i}": s, f"y{i}": y})
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
