"""Tile-config schema and heuristics for the sm_100a kernel family.

The reference keys tile choices by shape `(Z, H, N_CTX, HEAD_DIM, causal) -> (BLOCK_M, BLOCK_N)`
(presets block, flash_attention_forward.py:156-173; JSON `tuned_configs`,
tune_flash_attention_forward.py:428-440).  The B200 kernel keeps that schema and adds two
pipeline knobs, so a preset is either the reference's 2-tuple or a 4-tuple
`(BLOCK_M, BLOCK_N, NUM_STAGES, PERSISTENT_CTAS)`; in JSON the extra knobs are the keys
`NUM_STAGES` and `PERSISTENT_CTAS` (0 = library default: deepest ring / one CTA per SM).

Meaning of the knobs on sm_100a:
  BLOCK_M          query rows per CTA: 128 (one TMEM accumulator tile) or 256 (two tiles
                   sharing each K/V tile, ping-ponged between two softmax warpgroups)
  BLOCK_N          keys per pipeline step: 64 or 128 (N of the Q.K^T MMA)
  NUM_STAGES       depth of the K/V shared-memory ring (each stage holds one K or one V tile)
  PERSISTENT_CTAS  grid of the persistent kernel, which runs every fp16/bf16 call at head_dim
                   64/128 with the 256 x 128 tile: each CTA loops over tiles; 0 = one CTA per
                   SM.  Other configurations run one CTA per tile and refuse a non-zero
                   value.
"""
from __future__ import annotations

import dataclasses

import torch

SMEM_LIMIT = 232448  # 227 KiB opt-in dynamic shared memory per CTA on sm_100
TMEM_COLUMNS = 512
MAX_STAGES = 8

BLOCK_M_CHOICES = (128, 256)
BLOCK_N_CHOICES = (64, 128)


@dataclasses.dataclass(frozen=True)
class TileConfig:
    block_m: int
    block_n: int
    num_stages: int = 0
    persistent_ctas: int = 0

    @classmethod
    def from_preset(cls, preset) -> "TileConfig":
        if isinstance(preset, dict):
            return cls(int(preset["BLOCK_M"]), int(preset["BLOCK_N"]),
                       int(preset.get("NUM_STAGES", 0)), int(preset.get("PERSISTENT_CTAS", 0)))
        vals = tuple(int(x) for x in preset)
        if len(vals) == 2:
            return cls(vals[0], vals[1])
        if len(vals) == 4:
            return cls(*vals)
        raise ValueError(f"preset must have 2 or 4 entries, got {preset!r}")

    def as_dict(self) -> dict:
        return {"BLOCK_M": self.block_m, "BLOCK_N": self.block_n,
                "NUM_STAGES": self.num_stages, "PERSISTENT_CTAS": self.persistent_ctas}

    def as_preset(self) -> tuple:
        if self.num_stages == 0 and self.persistent_ctas == 0:
            return (self.block_m, self.block_n)
        return (self.block_m, self.block_n, self.num_stages, self.persistent_ctas)

    def replace(self, **kw) -> "TileConfig":
        return dataclasses.replace(self, **kw)


def _elt_bytes(dtype) -> int:
    return 4 if dtype == torch.float32 else 2


# Shared memory of the persistent kernel (csrc/fa_fwd_ws.cuh) besides its K/V ring: base
# alignment, two query tiles, two 8 KiB output staging buffers and its barrier/statistics block.
_WS_SHARED_BLOCK = 2384


def persistent_kernel_shape(head_dim: int, dtype, cfg: TileConfig) -> bool:
    """True when the persistent warp-specialised kernel can serve (dtype, head_dim, tile):
    fp16 or bf16, head_dim 64 or 128, BLOCK_M 256 and BLOCK_N 128."""
    return (dtype in (torch.float16, torch.bfloat16) and head_dim in (64, 128)
            and cfg.block_m == 256 and cfg.block_n == 128)


def persistent_kernel_serves(head_dim: int, dtype, cfg: TileConfig, sm_scale: float = 1.0) -> bool:
    """True when a call runs on the persistent kernel (mirrors `use_ws` in csrc/fa_fwd_api.cu):
    a shape it serves and a positive scale."""
    return persistent_kernel_shape(head_dim, dtype, cfg) and sm_scale > 0


def geometry(head_dim: int, dtype, cfg: TileConfig) -> dict | None:
    """Shared-memory / TMEM footprint of one CTA, mirroring `Geo` in csrc/fa_fwd_kernel.cuh and
    `WsGeo` in csrc/fa_fwd_ws.cuh."""
    eb = _elt_bytes(dtype)
    qt = cfg.block_m // 128
    if cfg.block_m not in BLOCK_M_CHOICES or cfg.block_n not in BLOCK_N_CHOICES:
        return None
    if persistent_kernel_shape(head_dim, dtype, cfg):
        q_tile = 128 * head_dim * eb
        kv_tile = 128 * head_dim * eb
        fixed = 1024 + 2 * q_tile + 2 * 8192 + _WS_SHARED_BLOCK
        stages = min((SMEM_LIMIT - fixed) // kv_tile, MAX_STAGES)
        return {"q_tile_bytes": q_tile, "kv_tile_bytes": kv_tile, "smem_fixed": fixed,
                "max_stages": stages, "tmem_columns": 2 * (128 + head_dim), "threads": 512,
                "persistent": True}
    tmem = qt * (cfg.block_n + head_dim)
    if tmem > TMEM_COLUMNS:
        return None
    if dtype == torch.float32:
        if head_dim > 128 or head_dim < 32:
            return None
        if qt == 2 and (head_dim > 64 or cfg.block_n != 64):
            return None
    q_tile = 128 * head_dim * eb
    kv_tile = cfg.block_n * head_dim * eb
    fixed = 1024 + qt * q_tile + 256
    stages = min((SMEM_LIMIT - fixed) // kv_tile, MAX_STAGES)
    if stages < 2:
        return None
    return {"q_tile_bytes": q_tile, "kv_tile_bytes": kv_tile, "smem_fixed": fixed,
            "max_stages": stages, "tmem_columns": tmem, "threads": 128 + 128 * qt,
            "persistent": False}


def is_supported(head_dim: int, dtype, cfg: TileConfig) -> bool:
    g = geometry(head_dim, dtype, cfg)
    if g is None:
        return False
    return cfg.num_stages == 0 or 2 <= cfg.num_stages <= g["max_stages"]


def max_stages(head_dim: int, dtype, cfg: TileConfig) -> int:
    g = geometry(head_dim, dtype, cfg)
    return 0 if g is None else g["max_stages"]


def heuristic(n_ctx: int, head_dim: int, causal: bool, dtype=None) -> TileConfig:
    """Default tile when no preset matches (same rule as fa_fwd_sm100_default_tile)."""
    del causal
    if dtype == torch.float32:
        return TileConfig(128, 64)
    if head_dim == 256:
        return TileConfig(128, 64)
    return TileConfig(256 if n_ctx > 128 else 128, 128)


def candidates(head_dim: int, dtype) -> list[TileConfig]:
    """Every (BLOCK_M, BLOCK_N, NUM_STAGES) the kernel family supports for a head_dim/dtype."""
    out = []
    for bm in BLOCK_M_CHOICES:
        for bn in BLOCK_N_CHOICES:
            base = TileConfig(bm, bn)
            g = geometry(head_dim, dtype, base)
            if g is None:
                continue
            for st in range(2, g["max_stages"] + 1):
                out.append(base.replace(num_stages=st))
    return out
