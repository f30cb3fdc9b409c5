"""Stand-in for `torch_npu` so the reference's scripts run unchanged on CUDA.

The reference evaluator and tuner (ZyEng-Art/flash_attn_npu evaluate_attention.py,
tune_flash_attention_forward.py) `import torch_npu` and call `torch.npu.synchronize()`,
`torch.npu.empty_cache()` and the vendor operator `torch_npu.npu_fusion_attention`
(evaluate_attention.py:12, 99, 104-131, 162).  Put this directory on PYTHONPATH and those
calls land on CUDA:

    PYTHONPATH=flash_attn_npu_b200/npu_shim python evaluate_attention.py \\
        --candidate flash_attention_forward.py

`npu_fusion_attention` is answered according to FA_SHIM_BASELINE:
  sdpa   (default) torch.nn.functional.scaled_dot_product_attention -- the CUDA library
         attention stands in for the Ascend vendor op in the evaluator's speed comparison
  raise  raise RuntimeError, so the evaluator's correctness check falls back to its fp32
         torch reference (evaluate_attention.py:151-156)
Only the BNSD layout the evaluator uses is supported.
"""
from __future__ import annotations

import os
import types

import torch

__version__ = "0.0-cuda-shim"


def _npu_namespace():
    ns = types.SimpleNamespace()
    ns.synchronize = torch.cuda.synchronize
    ns.empty_cache = torch.cuda.empty_cache
    ns.is_available = torch.cuda.is_available
    ns.device_count = torch.cuda.device_count
    ns.current_device = torch.cuda.current_device
    ns.set_device = torch.cuda.set_device
    return ns


if not hasattr(torch, "npu"):
    torch.npu = _npu_namespace()


def _is_causal_mask(mask: torch.Tensor, sq: int, sk: int) -> bool:
    if mask is None or mask.dtype != torch.bool or tuple(mask.shape[-2:]) != (sq, sk):
        return False
    ref = torch.triu(torch.ones((sq, sk), dtype=torch.bool, device=mask.device), diagonal=1)
    return bool(torch.equal(mask.reshape(-1, sq, sk)[0], ref))


def npu_fusion_attention(query, key, value, head_num, input_layout="BNSD", pse=None,
                         padding_mask=None, atten_mask=None, scale=1.0, keep_prob=1.0,
                         pre_tockens=2147483647, next_tockens=2147483647, inner_precise=0,
                         prefix=None, sparse_mode=0, **_unused):
    """Attention with the vendor operator's calling convention; returns a tuple whose [0] is
    the output (the evaluator reads only [0]).  `atten_mask` True means "masked out"."""
    mode = os.environ.get("FA_SHIM_BASELINE", "sdpa").strip().lower()
    if mode == "raise":
        raise RuntimeError("npu_fusion_attention is not available on CUDA (FA_SHIM_BASELINE=raise)")
    if input_layout != "BNSD":
        raise RuntimeError(f"torch_npu shim supports input_layout='BNSD' only, got {input_layout!r}")
    if keep_prob != 1.0:
        raise RuntimeError("torch_npu shim does not implement dropout (keep_prob != 1)")
    if pse is not None or padding_mask is not None:
        raise RuntimeError("torch_npu shim does not implement pse / padding_mask")
    sq, sk = query.shape[-2], key.shape[-2]
    causal = _is_causal_mask(atten_mask, sq, sk) or (atten_mask is None and next_tockens == 0)
    attn_mask = None
    if atten_mask is not None and not causal:
        attn_mask = ~atten_mask.to(torch.bool)
    out = torch.nn.functional.scaled_dot_product_attention(
        query, key, value, attn_mask=attn_mask, is_causal=causal, scale=float(scale))
    return (out, None, None, None, 0, 0, 0)
