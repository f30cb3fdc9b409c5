"""(b, h) sharding across ranks and the verification gather, on gloo CPU ranks (world size 2/3)."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flash_attn_npu_b200 import inputs as fa_inputs
from flash_attn_npu_b200 import sharding
from oracle.attention_ref import attention_ref_torch


@pytest.mark.parametrize("n,w", [(256, 1), (256, 2), (256, 8), (128, 8), (7, 3), (2, 8), (0, 4)])
def test_shard_ranges_partition(n, w):
    ranges = [sharding.shard_range(n, w, r) for r in range(w)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (a0, b0), (a1, _b1) in zip(ranges, ranges[1:]):
        assert b0 == a1
    sizes = sharding.shard_counts(n, w)
    assert max(sizes) - min(sizes) <= 1 and sum(sizes) == n


def test_headline_split_matches_the_plan():
    # cfg4: 256 (b,h) slices -> 256/128/64/32 per GPU at 1/2/4/8 GPUs
    for w, per in ((1, 256), (2, 128), (4, 64), (8, 32)):
        assert set(sharding.shard_counts(256, w)) == {per}


def test_take_shard_is_a_view_of_contiguous_slices():
    t = torch.arange(2 * 3 * 4 * 2, dtype=torch.float32).reshape(2, 3, 4, 2)
    s = sharding.take_shard(t, 2, 1)
    assert s.shape == (3, 1, 4, 2)
    assert torch.equal(s[0, 0], t[1, 0])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = fa_inputs.AttnConfig("tiny", 2, 3, 40, 16, torch.float32, True, 11, 0.25, "randn")
        q, k, v = fa_inputs.make_inputs(cfg, "cpu")
        n = cfg.batch * cfg.heads
        a, b = sharding.shard_range(n, world, rank)
        flat = lambda t: t.reshape(n, cfg.seqlen, cfg.head_dim)  # noqa: E731
        # each rank computes its slices (the CPU oracle stands in for the GPU kernel here)
        out, lse = attention_ref_torch(flat(q)[a:b], flat(k)[a:b], flat(v)[a:b], True, 0.25)
        out_all = sharding.gather_shards(out.reshape(b - a, 1, cfg.seqlen, cfg.head_dim), n,
                                         world, rank)
        lse_all = sharding.gather_shards(lse.reshape(b - a, 1, cfg.seqlen), n, world, rank)
        if rank == 0:
            ro, rl = attention_ref_torch(q, k, v, True, 0.25)
            ok = (torch.allclose(out_all.reshape(ro.shape), ro, atol=1e-6) and
                  torch.allclose(lse_all.reshape(rl.shape), rl, atol=1e-6))
            result_q.put(ok)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_shard_and_gather(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) is True
