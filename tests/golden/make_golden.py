"""Generate the golden fixtures under tests/golden/ from the reference's own attention path.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden.py --reference /path/to/flash_attn_npu

It imports the reference evaluator `evaluate_attention.py` by path with a stub `torch_npu`
module (the evaluator imports torch_npu at the top, evaluate_attention.py:12, but its fp32
oracle `_torch_attention_reference`, :134-143, is plain torch), runs that function on CPU on
seeded inputs, and stores inputs + outputs as compressed .npz files.  The logsumexp target is
`torch.logsumexp` of the same fp32 scores the reference function builds (:135-141); the
reference kernel's `M` output is that quantity (flash_attention_forward.py:1022, 1031).

Cases:
  cfg1_fp32 / cfg1_fp16  B=1 H=2 S=128 D=64 non-causal, q,k,v = torch.randn (seed 0, CPU
                         generator, drawn in order q, k, v), sm_scale = 1/sqrt(64)
  eval_<i>_<dtype>       the evaluator's own small CORRECTNESS_CASES (:15-34) whose inputs fit
                         in a few hundred KB, drawn by the evaluator's `_make_inputs` on CPU
                         (normal(0, 0.5), seed = idx) with its default sm_scale 0.5
"""
from __future__ import annotations

import argparse
import importlib.util
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def load_reference_evaluator(ref_dir: Path):
    if "torch_npu" not in sys.modules:
        stub = types.ModuleType("torch_npu")
        stub.__doc__ = "stub: only the evaluator's import line needs it"
        sys.modules["torch_npu"] = stub
    spec = importlib.util.spec_from_file_location("ref_evaluate_attention",
                                                  ref_dir / "evaluate_attention.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _lse_from_reference_scores(q, k, causal, sm_scale):
    # The same score construction as evaluate_attention.py:135-141, then logsumexp.
    scores = torch.matmul(q.float(), k.float().transpose(-2, -1)) * sm_scale
    if causal:
        mask = torch.triu(torch.ones((q.shape[-2], k.shape[-2]), dtype=torch.bool), diagonal=1)
        scores = scores.masked_fill(mask, float("-inf"))
    return torch.logsumexp(scores, dim=-1)


def _save(name, q, k, v, causal, sm_scale, out_ref, lse_ref, out_cast=None):
    path = HERE / f"{name}.npz"
    payload = dict(
        q=q.float().numpy(), k=k.float().numpy(), v=v.float().numpy(),
        dtype=np.array(str(q.dtype).replace("torch.", "")),
        causal=np.array(bool(causal)), sm_scale=np.array(float(sm_scale), dtype=np.float64),
        out_fp32=out_ref.float().numpy(), lse_fp32=lse_ref.float().numpy(),
    )
    if out_cast is not None:
        payload["out_cast"] = out_cast.float().numpy()
    np.savez_compressed(path, **payload)
    return path


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--reference", required=True, type=Path,
                    help="directory holding the reference's evaluate_attention.py")
    args = ap.parse_args(argv)
    ev = load_reference_evaluator(args.reference)
    ref_fn = ev._torch_attention_reference
    written = []

    # cfg1: B=1 H=2 S=128 D=64, non-causal, scale 1/8, randn seed 0 (q, k, v in order)
    g = torch.Generator().manual_seed(0)
    shape = (1, 2, 128, 64)
    q32 = torch.randn(shape, generator=g)
    k32 = torch.randn(shape, generator=g)
    v32 = torch.randn(shape, generator=g)
    scale = 1.0 / 8.0
    for dt, name in ((torch.float32, "cfg1_fp32"), (torch.float16, "cfg1_fp16")):
        q, k, v = q32.to(dt), k32.to(dt), v32.to(dt)
        # fp32-upcast inputs keep the reference's final `.to(q.dtype)` a no-op
        out = ref_fn(q.float(), k.float(), v.float(), False, scale)
        out_cast = ref_fn(q, k, v, False, scale) if dt == torch.float32 else None
        lse = _lse_from_reference_scores(q, k, False, scale)
        written.append(_save(name, q, k, v, False, scale, out, lse, out_cast))

    # Small evaluator correctness cases, inputs drawn exactly as the evaluator draws them.
    for idx, (z, h, n, d, causal) in enumerate(ev.CORRECTNESS_CASES):
        if z * h * n * d > 2 * 128 * 128:   # keep the fixtures small
            continue
        for dt in (torch.float16, torch.bfloat16):
            q, k, v = ev._make_inputs("cpu", dt, z, h, n, d, idx)
            out = ref_fn(q.float(), k.float(), v.float(), causal, ev.DEFAULT_SM_SCALE)
            lse = _lse_from_reference_scores(q, k, causal, ev.DEFAULT_SM_SCALE)
            name = f"eval_{idx:02d}_{str(dt).replace('torch.', '')}"
            written.append(_save(name, q, k, v, causal, ev.DEFAULT_SM_SCALE, out, lse))

    for p in written:
        print(p.relative_to(HERE.parent.parent), p.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
