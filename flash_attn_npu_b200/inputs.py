"""Seeded synthetic inputs for the five benchmark configurations.

No dataset is involved: each configuration is a shape, a dtype, a mask and a value
distribution.  Draws use a CPU `torch.Generator` in fp32, in a fixed order, then cast to
the compute dtype, so the CPU oracle and the GPU see identical bits.  Layout is
[B, H, S, D] contiguous (the reference's BNSD layout, flash_attention_forward.py:1308-1312).

The reference evaluator's own cases keep its own recipe (`normal(0, 0.5)` drawn on the
device after `torch.manual_seed(seed)`, evaluate_attention.py:90-95); `evaluator_inputs`
reproduces it.
"""
from __future__ import annotations

import dataclasses
import math

import torch


@dataclasses.dataclass(frozen=True)
class AttnConfig:
    name: str
    batch: int
    heads: int
    seqlen: int
    head_dim: int
    dtype: torch.dtype
    causal: bool
    seed: int
    sm_scale: float
    recipe: str  # "randn", "half_randn", "outliers"

    @property
    def shape(self):
        return (self.batch, self.heads, self.seqlen, self.head_dim)

    def flops(self) -> float:
        return attention_flops(self.batch, self.heads, self.seqlen, self.head_dim, self.causal)

    def bytes(self) -> float:
        return attention_bytes(self.batch, self.heads, self.seqlen, self.head_dim,
                               torch.tensor([], dtype=self.dtype).element_size())

    def describe(self) -> dict:
        return {"workload": self.name, "B": self.batch, "H": self.heads, "S": self.seqlen,
                "D": self.head_dim, "dtype": str(self.dtype).replace("torch.", ""),
                "causal": self.causal, "sm_scale": self.sm_scale, "seed": self.seed,
                "inputs": self.recipe}


CONFIGS = {
    "cfg1_fp32": AttnConfig("cfg1_fp32", 1, 2, 128, 64, torch.float32, False, 0, 1 / 8, "randn"),
    "cfg1_fp16": AttnConfig("cfg1_fp16", 1, 2, 128, 64, torch.float16, False, 0, 1 / 8, "randn"),
    "cfg2": AttnConfig("cfg2", 4, 16, 1024, 64, torch.float16, False, 1, 1 / 8, "randn"),
    "cfg3": AttnConfig("cfg3", 8, 32, 4096, 128, torch.bfloat16, True, 2, 1 / math.sqrt(128),
                       "half_randn"),
    "cfg4": AttnConfig("cfg4", 16, 16, 8192, 128, torch.bfloat16, False, 3, 1 / math.sqrt(128),
                       "randn"),
    "cfg5": AttnConfig("cfg5", 2, 64, 16384, 128, torch.float16, True, 4, 1 / math.sqrt(128),
                       "outliers"),
}

# Sequence lengths that are not a multiple of the 128-key block, beside their tile-multiple
# neighbours (the reference drops the keys past the last full block, flash_attention_forward.py
# :846-869, and asserts N_CTX % BLOCK_M == 0, :976; these measure what the masked tails cost).
RAGGED_CONFIGS = {
    "cfg4_s8191": AttnConfig("cfg4_s8191", 16, 16, 8191, 128, torch.bfloat16, False, 3,
                             1 / math.sqrt(128), "randn"),
    "causal_s1024": AttnConfig("causal_s1024", 64, 16, 1024, 128, torch.bfloat16, True, 5,
                               1 / math.sqrt(128), "randn"),
    "causal_s1000": AttnConfig("causal_s1000", 64, 16, 1000, 128, torch.bfloat16, True, 5,
                               1 / math.sqrt(128), "randn"),
    "causal_s2048": AttnConfig("causal_s2048", 32, 16, 2048, 128, torch.bfloat16, True, 6,
                               1 / math.sqrt(128), "randn"),
    "causal_s2049": AttnConfig("causal_s2049", 32, 16, 2049, 128, torch.bfloat16, True, 6,
                               1 / math.sqrt(128), "randn"),
}
CONFIGS.update(RAGGED_CONFIGS)

HEADLINE = "cfg4"


def attention_flops(b, h, s, d, causal) -> float:
    """4*B*H*S^2*D (two GEMMs), halved when causal."""
    f = 4.0 * b * h * s * s * d
    return f * 0.5 if causal else f


def attention_bytes(b, h, s, d, elt_bytes) -> float:
    """Algorithmic HBM traffic: read Q, K, V once, write O, write fp32 LSE."""
    return 4.0 * b * h * s * d * elt_bytes + 4.0 * b * h * s


def make_inputs(cfg: AttnConfig, device="cpu", heads_slice: slice | None = None):
    """Draw q, k, v for `cfg` on the CPU generator, cast, move to `device`.

    `heads_slice` restricts the returned tensors to a range of flattened (b*H + h) slices
    after drawing the full tensors (so a shard sees exactly the bits the full run sees).
    """
    g = torch.Generator().manual_seed(cfg.seed)
    shape = cfg.shape
    if cfg.recipe == "randn":
        q = torch.randn(shape, generator=g)
        k = torch.randn(shape, generator=g)
        v = torch.randn(shape, generator=g)
    elif cfg.recipe == "half_randn":
        q = torch.randn(shape, generator=g) * 0.5
        k = torch.randn(shape, generator=g) * 0.5
        v = torch.randn(shape, generator=g) * 0.5
    elif cfg.recipe == "outliers":
        q = torch.randn(shape, generator=g)
        k = torch.randn(shape, generator=g)
        mq = torch.rand(shape, generator=g) < 0.01
        mk = torch.rand(shape, generator=g) < 0.01
        v = torch.rand(shape, generator=g) * 2.0 - 1.0
        q[mq] *= 20.0
        k[mk] *= 20.0
    else:
        raise ValueError(cfg.recipe)
    out = []
    for t in (q, k, v):
        t = t.to(cfg.dtype)
        if heads_slice is not None:
            t = t.reshape(cfg.batch * cfg.heads, cfg.seqlen, cfg.head_dim)[heads_slice]
            t = t.reshape(-1, 1, cfg.seqlen, cfg.head_dim)
        out.append(t.to(device))
    return tuple(out)


def evaluator_inputs(device, dtype, z, h, n_ctx, head_dim, seed):
    """The reference evaluator's recipe (evaluate_attention.py:90-95)."""
    torch.manual_seed(seed)
    q = torch.empty((z, h, n_ctx, head_dim), dtype=dtype, device=device).normal_(mean=0.0, std=0.5)
    k = torch.empty((z, h, n_ctx, head_dim), dtype=dtype, device=device).normal_(mean=0.0, std=0.5)
    v = torch.empty((z, h, n_ctx, head_dim), dtype=dtype, device=device).normal_(mean=0.0, std=0.5)
    return q, k, v


# The reference evaluator's shape lists (evaluate_attention.py:15-43), as data.
EVALUATOR_CORRECTNESS_CASES = [
    (1, 1, 64, 64, False), (1, 1, 64, 64, True), (1, 1, 128, 128, False), (1, 1, 128, 128, True),
    (1, 2, 1024, 64, False), (1, 2, 1024, 64, True), (4, 32, 64, 64, False),
    (4, 32, 64, 64, True), (4, 32, 128, 128, False), (4, 32, 256, 128, True),
    (4, 32, 512, 64, True), (4, 32, 1024, 64, False), (4, 32, 1024, 64, True),
    (4, 32, 1024, 128, False), (4, 32, 2048, 64, True), (4, 32, 2048, 128, False),
    (4, 32, 4096, 64, False), (128, 8, 1024, 64, False),
]
EVALUATOR_PERFORMANCE_CASES = [
    (128, 8, 1024, 128, True), (128, 8, 1024, 256, True), (128, 8, 2048, 128, True),
    (128, 8, 2048, 256, False), (128, 8, 4096, 128, False), (128, 8, 8192, 64, False),
]
