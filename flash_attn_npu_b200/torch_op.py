"""`torch.ops.flash_attn_b200.fwd`: the forward registered as a PyTorch custom operator.

The operator wraps `ops.forward` (the C-ABI launch on the current stream) so the kernel can sit
inside code that PyTorch traces or captures: a fake implementation gives output shapes,
dtypes and strides without running anything (meta tensors, FakeTensorMode, torch.compile
graphs with the operator left opaque), and the launch itself is capture-safe (no allocation in
the C ABI, no host synchronisation), so it can be recorded into a CUDA graph.

    out, lse = torch.ops.flash_attn_b200.fwd(q, k, v, causal, sm_scale, 0, 0, 0, 0)

Arguments follow `ops.forward`: the last four are BLOCK_M, BLOCK_N, NUM_STAGES,
PERSISTENT_CTAS, each 0 for the library default.
"""
from __future__ import annotations

import torch

from . import ops


def _out_like(q: torch.Tensor) -> torch.Tensor:
    """Output allocation rule of `ops.forward` from shapes and strides alone: q's layout when a
    TMA tensor map can describe it (unit inner stride, 16-byte strides), else contiguous."""
    eb = q.element_size()
    ok = q.stride(-1) == 1 and all(
        q.shape[d] <= 1 or (q.stride(d) * eb) % 16 == 0 for d in range(3))
    return torch.empty_like(q) if ok else q.new_empty(q.shape)


@torch.library.custom_op("flash_attn_b200::fwd", mutates_args=())
def fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool, sm_scale: float,
        block_m: int = 0, block_n: int = 0, num_stages: int = 0,
        persistent_ctas: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    return ops.forward(q, k, v, causal, sm_scale, block_m=block_m, block_n=block_n,
                       num_stages=num_stages, persistent_ctas=persistent_ctas)


@fwd.register_fake
def _fwd_fake(q, k, v, causal, sm_scale, block_m=0, block_n=0, num_stages=0,
              persistent_ctas=0):
    ops.validate_layout(q, k, v)
    z, h, n_ctx, _ = q.shape
    return _out_like(q), q.new_empty((z, h, n_ctx), dtype=torch.float32)
