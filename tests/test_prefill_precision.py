"""Why the prefill GEMM feeds its activations as an fp16 hi + lo pair.

The tensor-core prefill (go-infer_b200/csrc/gemm_tc.cu, stage_tokens_kernel)
scales each token row by a power of two (its largest magnitude just below
2^10) and splits it into fp16 hi + lo, so every B operand is MMA'd twice.
A single fp16 (or bf16) operand would halve the tensor-core work.  This
emulates the three representations on the CPU -- the products and sums in
float64, so only the representation of x differs -- against the reference's
float32 MatMulQ4_K per token (pkg/engine/forward.go:482-495 over
pkg/math/gemv.go:134-167), with the parity bar of the GPU tests.  The pair
passes with room to spare; a single operand fails, fp16 by ~60x at the worst
element and bf16 by ~600x.  So the split stays.
"""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))

from _util import REL_TOL, plain_rel_err, rel_err, seeded_weights  # noqa: E402

GGML_Q4_K = 12


def staged(x, mode):
    """x [tokens, cols] float32 as the tensor core sees it, in float64:
    stage_tokens_kernel's per-token power of two (largest |x| < 2^10), then
    the fp16 hi + lo pair, fp16 alone, or bf16 (round to nearest even)."""
    m = np.abs(x).max(axis=1, keepdims=True)
    e = 10 - np.frexp(m)[1]  # 2^(E-1) <= m < 2^E: the row's largest |x| lands in [2^9, 2^10)
    xs = np.ldexp(x.astype(np.float64), e).astype(np.float32)
    if mode == "hi+lo":
        hi = xs.astype(np.float16).astype(np.float32)
        v = hi.astype(np.float64) + (xs - hi).astype(np.float16).astype(np.float64)
    elif mode == "fp16":
        v = xs.astype(np.float16).astype(np.float64)
    else:  # bf16
        u = xs.view(np.uint32).astype(np.uint64)
        u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
        v = u.astype(np.uint32).view(np.float32).astype(np.float64)
    return np.ldexp(v, -e)


@pytest.fixture(scope="module")
def q4k_case():
    import oracle as O
    import quantize_np as Q
    rows, cols, tokens = 2048, 4096, 16
    raw = Q.quantize_q4_k(seeded_weights(7, rows, cols))
    rb = (cols // 256) * 144
    w = np.stack([O.dequantize(GGML_Q4_K, raw[r * rb:(r + 1) * rb], cols) for r in range(rows)])
    x = np.random.default_rng(3).normal(0.0, 1.0, size=(tokens, cols)).astype(np.float32)
    ref = O.matmul_batch(GGML_Q4_K, x, raw, tokens, rows, cols)
    return w.astype(np.float64), x, ref


@pytest.mark.parametrize("mode,passes", [("hi+lo", True), ("fp16", False), ("bf16", False)])
def test_activation_operand_against_the_bar(q4k_case, mode, passes):
    w, x, ref = q4k_case
    y = staged(x, mode) @ w.T
    e = rel_err(y, ref)
    print(f"{mode}: max rel err {e.max():.2e} (floored), p99 {np.quantile(e, 0.99):.2e}, "
          f"median plain {np.median(plain_rel_err(y, ref)):.2e}")
    if passes:
        assert e.max() <= REL_TOL / 4
    else:
        assert e.max() > 10 * REL_TOL  # not a near miss
