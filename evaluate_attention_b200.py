#!/usr/bin/env python3
"""The reference evaluator's scoring run, restated for the B200 module.

Restates the flow of ZyEng-Art/flash_attn_npu `evaluate_attention.py` (main, :576-659) for a CUDA
device, driving a candidate module through its public `attention(q, k, v, causal, sm_scale)`:

- correctness suite: the evaluator's 18 shapes, each drawn with its input recipe and seed
  (seed + case index, :90-95, :596-609); a case passes when `allclose(reference, candidate,
  atol, rtol)` (:293-308) and is worth 40 / 18 points (:284-286);
- performance suite: its six shapes (seed + 18 + index, :611-624); the candidate's output must
  first match the vendor operator's, then both are timed in alternating pairs -- wall clock
  around each call plus a device synchronize, the order flipped every iteration (:233-264) --
  and a case scores 10 * min(baseline / candidate, 1) on the chosen statistic (:329-361);
- a JSON and a text report in --report-dir, and the totals out of 100.

The vendor operator (CANN's `npu_fusion_attention`, :104-131) has no CUDA build; its stand-in
here is torch's `scaled_dot_product_attention` on the same tensors with `is_causal` (the cuDNN /
flash backends on a B200), the same stand-in the tuner uses.  The reference builds an S x S mask
inside every baseline call because the NPU operator takes its causal mask as a tensor; the CUDA
library takes a flag, so no mask is built.  `--reference fp32` scores correctness against the
fp32 torch attention instead (the evaluator's fallback, :134-156).

    python evaluate_attention_b200.py --dtype bfloat16 --report-dir reports_bf16
"""
from __future__ import annotations

import argparse
import dataclasses
import importlib.util
import json
import math
import statistics
import sys
import time
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
if str(HERE) not in sys.path:
    sys.path.insert(0, str(HERE))

from flash_attn_npu_b200 import inputs as fa_inputs  # noqa: E402

CORRECTNESS_POINTS = 40.0
PERFORMANCE_POINTS = 60.0
SPEED_METRICS = ("avg_us", "median_us", "trimmed_avg_us", "min_us")


# ----------------------------------------------------------------------------- statistics
def sample_stats(samples_us: list[float], trim_ratio: float) -> dict:
    """Summary of one timing series: mean, median, trimmed mean (trim_ratio cut from each end,
    at most all but the middle element), extremes, spread, p10 / p90 (linear interpolation)."""
    xs = sorted(float(x) for x in samples_us)
    n = len(xs)

    def quantile(q):
        pos = (n - 1) * q
        lo, hi = math.floor(pos), math.ceil(pos)
        return xs[lo] + (xs[hi] - xs[lo]) * (pos - lo)

    cut = min(int(n * trim_ratio), (n - 1) // 2)
    kept = xs[cut:n - cut]
    mean = statistics.fmean(xs)
    sd = statistics.pstdev(xs) if n > 1 else 0.0
    return {"avg_us": mean, "median_us": statistics.median(xs),
            "trimmed_avg_us": statistics.fmean(kept), "min_us": xs[0], "max_us": xs[-1],
            "stddev_us": sd, "cv": sd / mean if mean else None, "p10_us": quantile(0.10),
            "p90_us": quantile(0.90), "iters": n}


def case_score(points: float, baseline_us: float | None, candidate_us: float | None) -> tuple:
    """(speedup, score): points x min(baseline / candidate, 1), nothing without both times."""
    if not baseline_us or not candidate_us or candidate_us <= 0:
        return None, 0.0
    speedup = baseline_us / candidate_us
    return speedup, points * min(max(speedup, 0.0), 1.0)


# ----------------------------------------------------------------------------- attention
def vendor_stand_in(q, k, v, causal, sm_scale):
    return torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=causal,
                                                            scale=sm_scale)


def fp32_attention(q, k, v, causal, sm_scale):
    """fp32 softmax(q k^T * scale) v, -inf above the diagonal when causal (the evaluator's own
    fallback reference, evaluate_attention.py:134-143)."""
    s = torch.matmul(q.float(), k.float().transpose(-2, -1)) * sm_scale
    if causal:
        n, m = q.shape[-2], k.shape[-2]
        s = s.masked_fill(torch.ones(n, m, dtype=torch.bool, device=q.device).triu(1),
                          float("-inf"))
    return torch.matmul(torch.softmax(s, dim=-1), v.float())


def paired_timing(baseline, candidate, warmup: int, iters: int, sync) -> tuple:
    """Wall-clock microseconds of both callables, interleaved; even iterations run the baseline
    first, odd ones the candidate first, each call followed by a device synchronize."""
    for _ in range(warmup):
        baseline()
        candidate()
    sync()
    times = {"baseline": [], "candidate": []}
    fns = {"baseline": baseline, "candidate": candidate}
    for it in range(iters):
        for name in (("baseline", "candidate") if it % 2 == 0 else ("candidate", "baseline")):
            t0 = time.perf_counter()
            fns[name]()
            sync()
            times[name].append((time.perf_counter() - t0) * 1e6)
    return times["baseline"], times["candidate"]


# ----------------------------------------------------------------------------- suites
@dataclasses.dataclass
class CaseResult:
    shape: tuple
    seed: int
    passed: bool = False
    max_abs_diff: float | None = None
    baseline: dict | None = None
    candidate: dict | None = None
    speedup: float | None = None
    score: float = 0.0
    error: str | None = None

    def record(self) -> dict:
        z, h, n, d, causal = self.shape
        out = {"Z": z, "H": h, "N_CTX": n, "HEAD_DIM": d, "causal": causal, "seed": self.seed,
               "passed": self.passed, "max_abs_diff": self.max_abs_diff, "score": self.score,
               "error": self.error}
        if self.baseline is not None or self.speedup is not None:
            out.update(baseline=self.baseline, candidate=self.candidate, speedup=self.speedup)
        return out


def _run(fn, result: CaseResult):
    try:
        fn()
    except Exception as exc:  # noqa: BLE001  (a failing case scores zero, the run goes on)
        result.error = f"{type(exc).__name__}: {exc}"
    torch.cuda.empty_cache()
    return result


@torch.no_grad()
def correctness_case(module, args, shape, seed, dtype) -> CaseResult:
    res = CaseResult(shape, seed)

    def body():
        z, h, n, d, causal = shape
        q, k, v = fa_inputs.evaluator_inputs(module.DEVICE, dtype, z, h, n, d, seed)
        ref_fn = fp32_attention if args.reference == "fp32" else vendor_stand_in
        ref = ref_fn(q, k, v, causal, args.sm_scale).to(dtype)
        out = module.attention(q, k, v, causal, args.sm_scale).to(dtype)
        res.max_abs_diff = (out - ref).abs().max().item()
        res.passed = bool(torch.allclose(ref, out, atol=args.atol, rtol=args.rtol))
        res.score = CORRECTNESS_POINTS / len(fa_inputs.EVALUATOR_CORRECTNESS_CASES) * res.passed
    return _run(body, res)


@torch.no_grad()
def performance_case(module, args, shape, seed, dtype) -> CaseResult:
    res = CaseResult(shape, seed)

    def body():
        z, h, n, d, causal = shape
        q, k, v = fa_inputs.evaluator_inputs(module.DEVICE, dtype, z, h, n, d, seed)
        base = lambda: vendor_stand_in(q, k, v, causal, args.sm_scale)  # noqa: E731
        cand = lambda: module.attention(q, k, v, causal, args.sm_scale).to(dtype)  # noqa: E731
        ref, out = base().to(dtype), cand()
        res.max_abs_diff = (out - ref).abs().max().item()
        res.passed = bool(torch.allclose(ref, out, atol=args.atol, rtol=args.rtol))
        if not res.passed:
            return
        tb, tc = paired_timing(base, cand, args.warmup, args.iters, torch.cuda.synchronize)
        res.baseline, res.candidate = (sample_stats(tb, args.trim_ratio),
                                       sample_stats(tc, args.trim_ratio))
        res.speedup, res.score = case_score(
            PERFORMANCE_POINTS / len(fa_inputs.EVALUATOR_PERFORMANCE_CASES),
            res.baseline[args.speed_metric], res.candidate[args.speed_metric])
    return _run(body, res)


# ----------------------------------------------------------------------------- reports
def summarize(kind: str, results: list[CaseResult], total_points: float) -> dict:
    speedups = [r.speedup for r in results if r.speedup is not None]
    return {"cases": [r.record() for r in results], "passed": sum(r.passed for r in results),
            "total": len(results), "score": sum(r.score for r in results),
            "max_score": total_points if results else 0.0,
            **({"mean_speedup": statistics.fmean(speedups) if speedups else None,
                "median_speedup": statistics.median(speedups) if speedups else None}
               if kind == "performance" else {})}


def _fmt(x, digits=3):
    return "n/a" if x is None else f"{x:.{digits}f}"


def write_reports(report_dir: Path, summary: dict) -> tuple[Path, Path]:
    report_dir.mkdir(parents=True, exist_ok=True)
    jpath, tpath = report_dir / "evaluation_report.json", report_dir / "evaluation_report.txt"
    jpath.write_text(json.dumps(summary, indent=2))
    cor, perf = summary["correctness"], summary["performance"]
    metric = summary["config"]["speed_metric"]
    lines = [f"candidate {summary['config']['candidate_module']} on {summary['config']['device']}"
             f" ({summary['config']['dtype']})",
             f"correctness {_fmt(cor['score'])} / {_fmt(cor['max_score'])} "
             f"({cor['passed']}/{cor['total']} passed); performance {_fmt(perf['score'])} / "
             f"{_fmt(perf['max_score'])} (mean speedup {_fmt(perf.get('mean_speedup'), 4)}); "
             f"total {_fmt(summary['total_score'])} / 100", "", "correctness:"]
    for i, c in enumerate(cor["cases"]):
        lines.append(f"  {i:2d} ({c['Z']},{c['H']},{c['N_CTX']},{c['HEAD_DIM']},"
                     f"{'causal' if c['causal'] else 'full'}) passed={c['passed']} "
                     f"max|diff|={_fmt(c['max_abs_diff'], 6)} {c['error'] or ''}".rstrip())
    lines += ["", f"performance ({metric}, wall clock per call incl. synchronize):"]
    for i, c in enumerate(perf["cases"]):
        b = (c.get("baseline") or {}).get(metric)
        t = (c.get("candidate") or {}).get(metric)
        lines.append(f"  {i:2d} ({c['Z']},{c['H']},{c['N_CTX']},{c['HEAD_DIM']},"
                     f"{'causal' if c['causal'] else 'full'}) match={c['passed']} "
                     f"vendor={_fmt(b, 1)} us candidate={_fmt(t, 1)} us "
                     f"speedup={_fmt(c.get('speedup'), 4)} score={_fmt(c['score'])} "
                     f"{c['error'] or ''}".rstrip())
    tpath.write_text("\n".join(lines) + "\n")
    return jpath, tpath


# ----------------------------------------------------------------------------- CLI
def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--candidate", default=str(HERE / "flash_attention_forward.py"))
    ap.add_argument("--mode", choices=["all", "correctness", "performance"], default="all")
    ap.add_argument("--dtype", default="float16", choices=["float16", "fp16", "bfloat16", "bf16"])
    ap.add_argument("--sm-scale", dest="sm_scale", type=float, default=0.5)
    ap.add_argument("--atol", type=float, default=1e-2)
    ap.add_argument("--rtol", type=float, default=1e-2)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--iters", type=int, default=30)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--speed-metric", dest="speed_metric", choices=SPEED_METRICS,
                    default="median_us")
    ap.add_argument("--trim-ratio", dest="trim_ratio", type=float, default=0.1)
    ap.add_argument("--reference", choices=["vendor", "fp32"], default="vendor",
                    help="correctness reference: the vendor-operator stand-in or fp32 torch")
    ap.add_argument("--report-dir", dest="report_dir", default=str(HERE / "evaluation_reports"))
    return ap


def load_module(path: Path):
    spec = importlib.util.spec_from_file_location("candidate_attention", str(path))
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def main(argv=None) -> dict:
    args = build_parser().parse_args(argv)
    dtype = torch.bfloat16 if args.dtype in ("bfloat16", "bf16") else torch.float16
    path = Path(args.candidate).resolve()
    module = load_module(path)
    n_cor = len(fa_inputs.EVALUATOR_CORRECTNESS_CASES)
    cor, perf = [], []
    if args.mode in ("all", "correctness"):
        for i, shape in enumerate(fa_inputs.EVALUATOR_CORRECTNESS_CASES):
            cor.append(correctness_case(module, args, shape, args.seed + i, dtype))
            print(f"correctness {i + 1}/{n_cor} {shape}: passed={cor[-1].passed}", flush=True)
    if args.mode in ("all", "performance"):
        for i, shape in enumerate(fa_inputs.EVALUATOR_PERFORMANCE_CASES):
            perf.append(performance_case(module, args, shape, args.seed + n_cor + i, dtype))
            r = perf[-1]
            print(f"performance {i + 1}/{len(fa_inputs.EVALUATOR_PERFORMANCE_CASES)} {shape}: "
                  f"match={r.passed} speedup={_fmt(r.speedup, 4)}", flush=True)
    summary = {"config": {"candidate_module": path.name, "device": torch.cuda.get_device_name(),
                          "dtype": str(dtype).replace("torch.", ""),
                          **{k: v for k, v in vars(args).items()
                             if k not in ("candidate", "report_dir")},
                          "vendor_operator": "torch.nn.functional.scaled_dot_product_attention",
                          "scoring": {"correctness_total": CORRECTNESS_POINTS,
                                      "performance_total": PERFORMANCE_POINTS,
                                      "performance_case": "10 * min(vendor / candidate, 1) "
                                                          "when the outputs match"}},
               "correctness": summarize("correctness", cor, CORRECTNESS_POINTS),
               "performance": summarize("performance", perf, PERFORMANCE_POINTS)}
    summary["total_score"] = summary["correctness"]["score"] + summary["performance"]["score"]
    jpath, tpath = write_reports(Path(args.report_dir), summary)
    print(f"total {summary['total_score']:.3f} / 100; reports: {jpath}, {tpath}")
    return summary


if __name__ == "__main__":
    main()
