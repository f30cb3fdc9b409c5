"""The CPU oracle is pinned against fixtures produced by the reference's own attention path.

tests/golden/*.npz were written by tests/golden/make_golden.py, which imports the reference
evaluator (evaluate_attention.py) and runs its `_torch_attention_reference` (:134-143).
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle.attention_ref import attention_ref_numpy, attention_ref_torch, attention_ref_sliced

FIXTURES = sorted(GOLDEN.glob("*.npz"))


def _load(path):
    d = np.load(path)
    dtype = getattr(torch, str(d["dtype"]))
    q = torch.from_numpy(d["q"]).to(dtype)
    k = torch.from_numpy(d["k"]).to(dtype)
    v = torch.from_numpy(d["v"]).to(dtype)
    return d, q, k, v, bool(d["causal"]), float(d["sm_scale"])


def test_fixtures_present():
    names = {p.stem for p in FIXTURES}
    assert {"cfg1_fp32", "cfg1_fp16"} <= names
    assert len(FIXTURES) >= 6


@pytest.mark.parametrize("path", FIXTURES, ids=lambda p: p.stem)
def test_torch_oracle_matches_reference_fixture(path):
    d, q, k, v, causal, scale = _load(path)
    out, lse = attention_ref_torch(q, k, v, causal, scale)
    np.testing.assert_allclose(out.numpy(), d["out_fp32"], rtol=0, atol=2e-6)
    np.testing.assert_allclose(lse.numpy(), d["lse_fp32"], rtol=0, atol=2e-6)


@pytest.mark.parametrize("path", FIXTURES, ids=lambda p: p.stem)
def test_numpy_oracle_matches_reference_fixture(path):
    d, q, k, v, causal, scale = _load(path)
    out, lse = attention_ref_numpy(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                   causal, scale)
    # float64 restatement vs the reference's fp32 evaluation: fp32 rounding only
    np.testing.assert_allclose(out, d["out_fp32"], rtol=0, atol=2e-5)
    np.testing.assert_allclose(lse, d["lse_fp32"], rtol=0, atol=2e-5)


def test_cfg1_fp32_cast_output_equals_fp32_output():
    d = np.load(GOLDEN / "cfg1_fp32.npz")
    # for fp32 inputs the reference's final `.to(q.dtype)` is the identity
    np.testing.assert_array_equal(d["out_cast"], d["out_fp32"])


def test_cfg1_inputs_are_the_seeded_recipe():
    d = np.load(GOLDEN / "cfg1_fp32.npz")
    g = torch.Generator().manual_seed(0)
    q = torch.randn((1, 2, 128, 64), generator=g)
    np.testing.assert_array_equal(d["q"], q.numpy())


# ---- known answers written from the mathematics ---------------------------------------
def test_zero_query_gives_uniform_attention():
    torch.manual_seed(1)
    n, dim = 37, 16
    q = torch.zeros(1, 1, n, dim)
    k = torch.randn(1, 1, n, dim)
    v = torch.randn(1, 1, n, dim)
    out, lse = attention_ref_torch(q, k, v, False, 0.3)
    torch.testing.assert_close(out[0, 0], v[0, 0].mean(0, keepdim=True).expand(n, dim),
                               atol=1e-6, rtol=0)
    torch.testing.assert_close(lse, torch.full_like(lse, math.log(n)), atol=1e-6, rtol=0)
    # causal: row i averages v[:i+1] and lse = log(i+1)
    out_c, lse_c = attention_ref_torch(q, k, v, True, 0.3)
    for i in (0, 5, n - 1):
        torch.testing.assert_close(out_c[0, 0, i], v[0, 0, : i + 1].mean(0), atol=1e-6, rtol=0)
        assert abs(lse_c[0, 0, i].item() - math.log(i + 1)) < 1e-6


def test_causal_first_row_selects_first_value():
    torch.manual_seed(2)
    q, k, v = (torch.randn(2, 3, 20, 32) for _ in range(3))
    out, lse = attention_ref_torch(q, k, v, True, 0.125)
    torch.testing.assert_close(out[:, :, 0], v[:, :, 0], atol=1e-6, rtol=0)
    torch.testing.assert_close(lse[:, :, 0], 0.125 * (q[:, :, 0] * k[:, :, 0]).sum(-1),
                               atol=1e-5, rtol=0)


def test_dominant_logit_selects_one_row():
    torch.manual_seed(3)
    n, dim = 64, 32
    k = torch.randn(1, 1, n, dim)
    v = torch.randn(1, 1, n, dim)
    q = 40.0 * k[:, :, 17:18].expand(1, 1, n, dim) / k[0, 0, 17].norm()
    out, _ = attention_ref_torch(q, k, v, False, 1.0)
    torch.testing.assert_close(out[0, 0], v[0, 0, 17].expand(n, dim), atol=1e-3, rtol=0)


def test_sliced_matches_full():
    torch.manual_seed(4)
    q, k, v = (torch.randn(2, 3, 50, 16) for _ in range(3))
    out, lse = attention_ref_torch(q, k, v, True, 0.25)
    so, sl = attention_ref_sliced(q, k, v, True, 0.25, slices=[(1, 2), (0, 0)])
    torch.testing.assert_close(so[(1, 2)], out[1, 2])
    torch.testing.assert_close(sl[(0, 0)], lse[0, 0])


# ----------------------------------------------------------------------------- fp8 V oracle
from oracle.attention_ref import attention_kernel_order_fp8v, attention_ref_fp8v_online  # noqa: E402


def _fp8_inputs(S, D, seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, 2, S, D, generator=g).to(dtype)
    k = torch.randn(1, 2, S, D, generator=g).to(dtype)
    v = torch.randn(1, 2, S, D, generator=g).to(torch.float8_e5m2)
    return q, k, v


@pytest.mark.parametrize("causal", [False, True])
def test_fp8v_orders_agree_within_e5m2_rounding(causal):
    """Both fp8-V restatements round P to e5m2 (2 mantissa bits); they differ from the exact
    fp32 attention, and from each other, only by that rounding; the LSE is unaffected."""
    q, k, v = _fp8_inputs(384, 64, 1)
    ex_o, ex_l = attention_ref_torch(q, k, v.float(), causal, 0.125)
    on_o, on_l = attention_ref_fp8v_online(q, k, v, causal, 0.125)
    ko_o, ko_l = attention_kernel_order_fp8v(q, k, v, causal, 0.125)
    for o in (on_o, ko_o):
        err = (o - ex_o).abs()
        assert err.mean().item() < 1e-2 and err.max().item() < 0.15
        assert err.mean().item() > 1e-4  # the rounding is really applied
    assert torch.allclose(on_l, ex_l, atol=1e-5) and torch.allclose(ko_l, ex_l, atol=1e-5)


def test_fp8v_single_block_orders_coincide():
    """With one key block both orders round P at the row maximum: identical up to exp vs exp2
    (a rounding flip needs p within ~1e-7 of an e5m2 midpoint)."""
    q, k, v = _fp8_inputs(96, 32, 2)
    on_o, _ = attention_ref_fp8v_online(q, k, v, False, 0.2, block_n=128)
    ko_o, _ = attention_kernel_order_fp8v(q, k, v, False, 0.2, block_n=128)
    assert (on_o - ko_o).abs().max().item() < 1e-3


def test_fp8v_kernel_order_moves_base_only_past_threshold():
    """A later block whose max exceeds the base by at most 8 (log2 units) keeps the base, so its
    p reach 2^8; past the threshold the base moves and O is rescaled -- either way the result
    equals the exact attention when every p is exactly representable in e5m2."""
    S, D = 256, 32
    k = torch.zeros(1, 1, S, D)
    q = torch.zeros(1, 1, 1, D)
    q[..., 0] = 1.0
    v = torch.randn(1, 1, S, D, generator=torch.Generator().manual_seed(3)).to(torch.float8_e5m2)
    for jump in (4.0, 20.0):  # log2-unit jump of the second block's logits
        kk = k.clone()
        kk[..., 128:, 0] = jump / 1.4426950408889634
        out, _ = attention_kernel_order_fp8v(q, kk, v, False, 1.0)
        ref, _ = attention_ref_torch(q, kk, v.float(), False, 1.0)
        assert torch.allclose(out, ref, atol=1e-5, rtol=1e-5), jump
