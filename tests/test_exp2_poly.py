"""CPU check of the attention kernel's FMA-pipe exp2 (exp2_fma2 in attn_fwd.cu).

The kernel computes a quarter of the softmax exponentials without MUFU: x is split
into n + f by the 1.5*2^23 shifter, 2^f comes from a degree-3 polynomial and n is
added into the exponent field.  This restates those float32 steps in numpy, with
the coefficients read from the kernel source, and bounds the error against exp2
over the range the softmax feeds it (x <= 2^8 above the running max, clamped at
-125 below)."""
import pathlib
import re

import numpy as np

SRC = pathlib.Path(__file__).resolve().parents[1] / "turing-sm75_b200" / "csrc" / "attn_fwd.cu"


def _coeffs():
    text = SRC.read_text()
    vals = {k: np.float32(float(v)) for k, v in re.findall(r"(kP[0-3]) = ([0-9.eE+-]+)f", text)}
    assert sorted(vals) == ["kP0", "kP1", "kP2", "kP3"], vals
    return vals["kP0"], vals["kP1"], vals["kP2"], vals["kP3"]


def exp2_fma2_np(x):
    """float32 restatement of exp2_fma2 (every product and sum rounded to float32)."""
    p0, p1, p2, p3 = _coeffs()
    f32 = np.float32
    x = np.maximum(x.astype(f32), f32(-125.0))
    shift = f32(12582912.0)
    t = (x + shift).astype(f32)
    n = (t - shift).astype(f32)
    f = (x - n).astype(f32)  # fma(n, -1, x) is exact here
    q = (p3 * f + p2).astype(f32)
    q = (q * f + p1).astype(f32)
    q = (q * f + p0).astype(f32)
    bits = (q.view(np.uint32).astype(np.uint64) + (t.view(np.uint32).astype(np.uint64) << np.uint64(23)))
    return (bits & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32)


def test_relative_error_below_bf16_rounding():
    x = np.linspace(-125.0, 8.0, 1_000_001, dtype=np.float64).astype(np.float32)
    got = exp2_fma2_np(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(got - ref) / ref
    assert rel.max() < 1e-4, rel.max()  # 16-bit P rounds at 2^-9 = 2e-3


def test_integer_and_half_integer_points():
    x = np.array([-125, -64, -10.5, -1, -0.5, 0, 0.5, 1, 3.5, 8], dtype=np.float32)
    got = exp2_fma2_np(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    assert np.all(np.abs(got - ref) / ref < 1e-4)


def test_masked_scores_give_tiny_positive_not_garbage():
    # -inf (a masked key) and anything below -125 clamp to 2^-125: finite, positive,
    # negligible against a row sum >= 1
    x = np.array([-np.inf, -1e30, -200.0, -125.5], dtype=np.float32)
    got = exp2_fma2_np(x)
    assert np.all(np.isfinite(got)) and np.all(got > 0) and np.all(got < 1e-37)
