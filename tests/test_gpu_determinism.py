"""Run-to-run determinism of the kernel and of the CPU oracle, in one process and across fresh
processes.

The kernel's reduction order is fixed by construction (one CTA owns a query tile, the key
blocks are visited in a fixed order, every thread owns one row), so repeated launches on the
same inputs must give bit-identical `out` and `lse`, whatever process they run in.  The CPU
oracle (oracle/attention_ref.py) is checked the same way, so that a parity error that moves
between runs can be pinned on the side that moved.
"""
from __future__ import annotations

import hashlib
import json
import subprocess
import sys

import pytest
import torch

from conftest import REPO

pytestmark = pytest.mark.gpu

REPEATS = 20
CFG3_SLICE = 37  # flattened (b * H + h) index of the cfg3 slice checked


def _digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes()
                          ).hexdigest()


def _cases():
    """(name, q, k, v, causal, scale) on the CPU: the smoke case in both masks and one slice of
    cfg3 (B8 H32 S4096 D128 bf16 causal, its own seeded draw)."""
    from flash_attn_npu_b200 import inputs as fa_inputs
    g = torch.Generator().manual_seed(0)
    shape = (2, 4, 384, 128)
    q, k, v = (torch.randn(shape, generator=g).to(torch.bfloat16) for _ in range(3))
    cfg = fa_inputs.CONFIGS["cfg3"]
    q3, k3, v3 = fa_inputs.make_inputs(cfg, "cpu", heads_slice=slice(CFG3_SLICE, CFG3_SLICE + 1))
    return [("smoke_full", q, k, v, False, 128 ** -0.5),
            ("smoke_causal", q, k, v, True, 128 ** -0.5),
            ("cfg3_slice", q3, k3, v3, True, cfg.sm_scale)]


def _kernel_digests(repeats: int) -> dict[str, list[str]]:
    from flash_attn_npu_b200 import ops
    out = {}
    for name, q, k, v, causal, scale in _cases():
        qd, kd, vd = (t.cuda() for t in (q, k, v))
        runs = []
        for _ in range(repeats):
            o, l = ops.forward(qd, kd, vd, causal, scale)
            torch.cuda.synchronize()
            runs.append(_digest(o) + _digest(l))
        out[name] = runs
    return out


def _oracle_digests() -> dict[str, str]:
    from oracle.attention_ref import attention_ref_torch
    out = {}
    for name, q, k, v, causal, scale in _cases()[:2]:
        o, l = attention_ref_torch(q, k, v, causal, scale)
        out[name] = _digest(o) + _digest(l)
    return out


def _child_main() -> None:
    print("DIGESTS " + json.dumps({"kernel": _kernel_digests(2), "oracle": _oracle_digests()}),
          flush=True)


def _run_child(extra_env=None) -> dict:
    import os
    env = dict(os.environ)
    env.update(extra_env or {})
    res = subprocess.run([sys.executable, __file__, "child"], cwd=str(REPO), env=env,
                         capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    line = [ln for ln in res.stdout.splitlines() if ln.startswith("DIGESTS ")][-1]
    return json.loads(line[len("DIGESTS "):])


def test_kernel_bitwise_deterministic_in_process_and_across_processes(cuda_device):
    here = _kernel_digests(REPEATS)
    for name, runs in here.items():
        assert len(set(runs)) == 1, f"{name}: {len(set(runs))} distinct results in {REPEATS} runs"
    oracle_here = _oracle_digests()
    # two fresh processes; the second with a single host thread, which changes how the CPU
    # oracle's matmuls are split across cores
    for extra in ({}, {"OMP_NUM_THREADS": "1"}):
        child = _run_child(extra)
        for name, runs in child["kernel"].items():
            assert set(runs) == {here[name][0]}, f"{name} differs in a fresh process ({extra})"
        assert child["oracle"] == oracle_here, f"the CPU oracle moved across processes ({extra})"


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "child":
        sys.path.insert(0, str(REPO))
        _child_main()
