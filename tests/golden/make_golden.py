"""Regenerates tests/golden/gemv_golden.npz (run from the repo root).

Inputs are seeded (numpy PCG64): weights N(0, 0.02) quantised by the
library's host quantiser (gi_quantize), activations N(0, 1).  Outputs come
from the CPU oracle (oracle/goinfer_ref.c, the restatement of go-infer's
GEMVEngine.MatMul*).  Shapes include rows that are not a multiple of 16 and
Q8_0/Q6_K rows whose byte length is only 2-byte aligned.
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path[:0] = [os.path.join(ROOT, "go-infer_b200"), os.path.join(ROOT, "oracle")]

import goinfer_cuda as G  # noqa: E402
import oracle as O  # noqa: E402

CASES = [
    # name, type, rows, cols, weight seed, x seed
    ("q4k_48x512", G.TYPE_Q4_K, 48, 512, 101, 102),
    ("q4k_37x768", G.TYPE_Q4_K, 37, 768, 103, 104),
    ("q6k_40x512", G.TYPE_Q6_K, 40, 512, 105, 106),
    ("q6k_20x768", G.TYPE_Q6_K, 20, 768, 107, 108),
    ("q8_0_36x288", G.TYPE_Q8_0, 36, 288, 109, 110),
    ("q8_0_33x512", G.TYPE_Q8_0, 33, 512, 111, 112),
]


def main():
    out = {}
    for name, qt, rows, cols, ws, xs in CASES:
        w = np.random.default_rng(ws).normal(0.0, 0.02, size=(rows, cols)).astype(np.float32)
        x = np.random.default_rng(xs).normal(0.0, 1.0, size=cols).astype(np.float32)
        raw = G.quantize(qt, w)
        y = O.matmul(qt, x, raw, rows, cols)
        out[name + "__shape"] = np.array([qt, rows, cols], dtype=np.int64)
        out[name + "__w"] = raw
        out[name + "__x"] = x
        out[name + "__y"] = y
    np.savez_compressed(os.path.join(ROOT, "tests", "golden", "gemv_golden.npz"), **out)
    print("wrote", len(CASES), "cases")


if __name__ == "__main__":
    main()
