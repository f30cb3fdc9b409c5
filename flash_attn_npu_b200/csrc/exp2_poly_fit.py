"""Derivation of the exp2 polynomial used on the FMA pipe in fa_fwd_kernel.cuh.

2^x is split as 2^n * 2^f with n = round(x), f = x - n in [-0.5, 0.5] (Cody-Waite style range
reduction); 2^f is approximated by a degree-4 polynomial whose coefficients minimise the
maximum relative error on [-0.5, 0.5] (Lawson's iteratively reweighted least squares, a
standard route to the minimax fit).  Printed: coefficients (fp32) and the max relative error
of fp32 Horner evaluation -- about 2.7e-6, far below the 1e-4 logsumexp tolerance.

Run:  python flash_attn_npu_b200/csrc/exp2_poly_fit.py
"""
import numpy as np


def fit(deg: int, iters: int = 200):
    f = np.cos(np.linspace(0.0, np.pi, 20001)) * 0.5
    y = np.exp2(f)
    V = np.vander(f, deg + 1, increasing=True)
    w = np.ones_like(f)
    for _ in range(iters):
        A = V / y[:, None] * np.sqrt(w)[:, None]
        c, *_ = np.linalg.lstsq(A, np.sqrt(w), rcond=None)
        err = np.abs(V @ c / y - 1.0)
        w = w * err
        w /= w.sum()
    return c.astype(np.float32)


def horner_rel_err(c32):
    ff = np.linspace(-0.5, 0.5, 200001).astype(np.float32)
    p = np.float32(c32[-1])
    for cj in c32[-2::-1]:
        p = (p * ff + cj).astype(np.float32)
    return float(np.abs(p.astype(np.float64) / np.exp2(ff.astype(np.float64)) - 1.0).max())


if __name__ == "__main__":
    c = fit(4)
    print("coefficients c0..c4:", ", ".join(f"{x:.9e}f" for x in c))
    print(f"max relative error (fp32 Horner): {horner_rel_err(c):.3e}")
