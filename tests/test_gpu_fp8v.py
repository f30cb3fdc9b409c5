"""GPU parity of the fp8-V kernel (V in float8 e5m2, Q/K/O 16-bit), through the C ABI.

The reference's fp8_v mode (flash_attention_forward.py:704, :996) rounds P to float8e5 before
the P.V dot and keeps the unrounded sum l.  Bars:
  - against `attention_kernel_order_fp8v` (the same fp8 product with the kernel's exponent
    bases, so P is rounded at the kernel's values): max-abs 2e-2, mean-abs 1e-3 -- residual
    differences are the 16-bit output rounding, accumulation order and rare e5m2 rounding flips
    where ex2.approx and exp2 straddle a rounding midpoint;
  - against the unquantised fp32 attention: the e5m2 rounding of P itself (2 mantissa bits, up
    to 12.5 % per element), max-abs 0.15 and mean-abs 1e-2 on these N(0,1) inputs -- the
    reference-order restatement (`attention_ref_fp8v_online`) sits at the same distance;
  - logsumexp: unaffected by the rounding of P, the usual 1e-4 (+2e-6 |lse|) bar.
"""
from __future__ import annotations

import pytest
import torch

import flash_attention_forward as faf
from flash_attn_npu_b200 import ops
from oracle.attention_ref import (attention_kernel_order_fp8v, attention_ref_fp8v_online,
                                  attention_ref_torch)

pytestmark = pytest.mark.gpu

KO_MAX, KO_MEAN = 2e-2, 1e-3
EXACT_MAX, EXACT_MEAN = 0.15, 1e-2
LSE_ABS, LSE_REL = 1e-4, 2e-6


def _inputs(B, H, S, D, dtype, seed, device):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, S, D, generator=g).to(dtype)
    k = torch.randn(B, H, S, D, generator=g).to(dtype)
    v = torch.randn(B, H, S, D, generator=g).to(torch.float8_e5m2)
    return q.to(device), k.to(device), v.to(device)


def _default_block_n(head_dim):
    return 64 if head_dim == 256 else 128


def _run(B, H, S, D, dtype, causal, seed, device, bm=0, bn=0):
    q, k, v = _inputs(B, H, S, D, dtype, seed, device)
    scale = D ** -0.5
    status = torch.zeros(1, dtype=torch.int32, device=device)
    out, lse = ops.forward(q, k, v, causal, scale, block_m=bm, block_n=bn, status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    assert out.dtype == dtype and out.shape == q.shape and lse.shape == (B, H, S)
    qc, kc, vc = q.cpu(), k.cpu(), v.cpu()
    ko_out, _ = attention_kernel_order_fp8v(qc, kc, vc, causal, scale,
                                            block_n=bn or _default_block_n(D))
    ex_out, ex_lse = attention_ref_torch(qc, kc, vc.float(), causal, scale)
    out_c, lse_c = out.float().cpu(), lse.cpu()
    assert torch.isfinite(out_c).all()
    e_ko = (out_c - ko_out).abs()
    assert e_ko.max().item() <= KO_MAX, f"vs kernel order: max {e_ko.max().item():.3e}"
    assert e_ko.mean().item() <= KO_MEAN, f"vs kernel order: mean {e_ko.mean().item():.3e}"
    e_ex = (out_c - ex_out).abs()
    assert e_ex.max().item() <= EXACT_MAX, f"vs exact: max {e_ex.max().item():.3e}"
    assert e_ex.mean().item() <= EXACT_MEAN, f"vs exact: mean {e_ex.mean().item():.3e}"
    lerr = (lse_c - ex_lse).abs()
    assert bool((lerr <= LSE_ABS + LSE_REL * ex_lse.abs()).all()), f"lse {lerr.max().item():.3e}"
    return out_c, ex_out, q, k, v


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [32, 64, 128, 256])
def test_fp8v_head_dims(head_dim, dtype, causal, cuda_device):
    _run(1, 2, 300, head_dim, dtype, causal, seed=11, device=cuda_device)


@pytest.mark.parametrize("seqlen", [1, 65, 129, 1000])
@pytest.mark.parametrize("causal", [False, True])
def test_fp8v_ragged_lengths(seqlen, causal, cuda_device):
    _run(2, 3, seqlen, 128, torch.bfloat16, causal, seed=seqlen, device=cuda_device)


@pytest.mark.parametrize("tile,head_dim", [((256, 128), 128), ((128, 128), 128), ((128, 128), 64),
                                           ((128, 128), 256), ((128, 64), 256)],
                         ids=lambda x: str(x))
def test_fp8v_tiles(tile, head_dim, cuda_device):
    _run(1, 2, 513, head_dim, torch.float16, False, seed=5, device=cuda_device,
         bm=tile[0], bn=tile[1])


def test_fp8v_same_distance_as_reference_order(cuda_device):
    """The kernel is no further from exact attention than the reference's own fp8 order."""
    out, ex_out, q, k, v = _run(2, 4, 1024, 128, torch.bfloat16, False, seed=3, device=cuda_device)
    ref8, _ = attention_ref_fp8v_online(q.cpu(), k.cpu(), v.cpu(), False, 128 ** -0.5)
    kern = (out - ex_out).abs().mean().item()
    refo = (ref8 - ex_out).abs().mean().item()
    assert kern <= 1.5 * refo + 1e-4, (kern, refo)


def test_fp8v_exact_when_p_is_representable(cuda_device):
    """q = 0: every probability is 1 (exact in e5m2), so O is the plain mean of V."""
    B, H, S, D = 1, 2, 256, 128
    _, k, v = _inputs(B, H, S, D, torch.bfloat16, 7, cuda_device)
    q = torch.zeros_like(k)
    out, lse = ops.forward(q, k, v, False, D ** -0.5)
    torch.cuda.synchronize()
    mean_v = v.float().mean(dim=2, keepdim=True).expand(B, H, S, D)
    assert (out.float() - mean_v).abs().max().item() <= 1e-2
    assert torch.allclose(lse, torch.full_like(lse, float(torch.log(torch.tensor(float(S))))),
                          atol=1e-5)


def test_fp8v_module_api(cuda_device):
    q, k, v = _inputs(1, 2, 200, 64, torch.float16, 9, cuda_device)
    out, lse = faf.attention(q, k, v, True, 0.125, return_lse=True)
    torch.cuda.synchronize()
    assert out.dtype == torch.float16
    ko, _ = attention_kernel_order_fp8v(q.cpu(), k.cpu(), v.cpu(), True, 0.125)
    assert (out.float().cpu() - ko).abs().max().item() <= KO_MAX


def test_fp8v_rejects_unsupported(cuda_device):
    q, k, v = _inputs(1, 1, 64, 16, torch.bfloat16, 1, cuda_device)
    with pytest.raises(ValueError):
        ops.forward(q, k, v, False, 0.25)  # head_dim 16
    q32 = torch.randn(1, 1, 64, 64, device=cuda_device)
    v8 = torch.randn(1, 1, 64, 64, device=cuda_device).to(torch.float8_e5m2)
    with pytest.raises(ValueError):
        ops.forward(q32, q32, v8, False, 0.125)  # fp32 q/k
