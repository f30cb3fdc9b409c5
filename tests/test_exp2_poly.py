"""CPU check of the FMA-pipe exp2 in csrc/fa_fwd_kernel.cuh (`exp2_poly2`).

The kernel can route a share of its exp2s through a polynomial instead of `ex2.approx`
(`FA_POLY_PAIRS_OF_8`).  This test replays the routine's exact fp32 / bit steps in numpy --
clamp, round-to-integer by adding 1.5 * 2^23, f = x - n, degree-4 Horner with fused
multiply-adds, and n added to the exponent field -- using the constants read from the kernel
source, and checks the result against exp2 over the whole range a softmax step can produce
(masked logits are -inf).  A clamp one lower (-127) would let 2^f < 1 borrow through the
exponent field into the sign bit, giving a NaN pattern; the test shows that too.
"""
from __future__ import annotations

import re
from pathlib import Path

import numpy as np

KERNEL = Path(__file__).resolve().parents[1] / "flash_attn_npu_b200" / "csrc" / "fa_fwd_kernel.cuh"


def _constants():
    src = KERNEL.read_text()
    body = src[src.index("float2 exp2_poly2(float2 x)"):]
    body = body[:body.index("return q;")]
    coeffs = [float(m) for m in re.findall(r"c\d = ([-+0-9.eE]+)f", body)]
    clamp = float(re.search(r"fmaxf\(x\.x, (-[0-9.]+)f\)", body).group(1))
    assert len(coeffs) == 5
    return np.array(coeffs, dtype=np.float32), np.float32(clamp)


def _fma(a, b, c):
    # fp32 fused multiply-add: exact product in fp64, one rounding of the sum to fp32
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def exp2_poly_emulated(x, coeffs, clamp):
    x = np.maximum(np.asarray(x, dtype=np.float32), clamp)
    r = np.float32(12582912.0)  # 1.5 * 2^23
    t = (x + r).astype(np.float32)
    n = (t - r).astype(np.float32)
    f = _fma(n, np.full_like(n, -1.0), x)
    c0, c1, c2, c3, c4 = (np.full_like(f, c) for c in coeffs)
    q = _fma(c4, f, c3)
    q = _fma(q, f, c2)
    q = _fma(q, f, c1)
    q = _fma(q, f, c0)
    bits = q.view(np.uint32) + (t.view(np.uint32) << np.uint32(23))
    return bits.astype(np.uint32).view(np.float32)


def test_exp2_poly_matches_exp2_over_the_softmax_range():
    coeffs, clamp = _constants()
    x = np.concatenate([np.linspace(-300.0, 8.0, 400001, dtype=np.float32),
                        np.array([-np.inf, -127.0, -126.5, -126.0, -125.5, 0.0, 8.0],
                                 dtype=np.float32)])
    with np.errstate(invalid="ignore", over="ignore"):
        y = exp2_poly_emulated(x, coeffs, clamp)
    assert np.all(np.isfinite(y)) and np.all(y >= 0.0)
    ref = np.exp2(x.astype(np.float64))
    normal = x >= -125.0
    rel = np.abs(y[normal].astype(np.float64) / ref[normal] - 1.0)
    assert rel.max() < 3e-6, rel.max()
    # below 2^-125 the result is only required to be tiny and non-negative
    assert np.all(y[~normal] <= 2.0 ** -124)


def test_clamp_one_lower_would_produce_nan():
    coeffs, _ = _constants()
    with np.errstate(invalid="ignore"):
        y = exp2_poly_emulated(np.array([-127.0, -126.6], dtype=np.float32), coeffs,
                               np.float32(-127.0))
    assert np.isnan(y[0]) or y[0] < 0.0
