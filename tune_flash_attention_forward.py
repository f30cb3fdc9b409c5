#!/usr/bin/env python3
"""Offline tile tuner for the B200 FlashAttention forward; rewrites the presets block.

Same command line, JSON schema and presets-block rewrite as the reference tuner
(ZyEng-Art/flash_attn_npu tune_flash_attention_forward.py), re-targeted at the sm_100a kernel:

- the sweep covers the sm_100a knobs: BLOCK_M in {128, 256} (one or two 128-row TMEM tiles),
  BLOCK_N in {64, 128} and every K/V ring depth NUM_STAGES that fits shared memory
  (reference sweep: (BM, BN) in {16..256}^2, tune_flash_attention_forward.py:76-115);
- each shape's candidates are timed in a spawned worker process with a per-candidate wall-clock
  limit; a candidate that fails, faults or hangs is recorded with its error and the worker is
  replaced, so the sweep always finishes (reference: per-candidate try/except, :224-237);
- timing uses CUDA events on the launch stream (reference: perf_counter around
  fn(); synchronize, :135-152);
- the JSON keeps `meta / tuned_configs / results` (:428-444) and adds the keys NUM_STAGES and
  PERSISTENT_CTAS to each config; existing files are merged shape by shape (:182-214), so an
  interrupted tuning run resumes by passing the same --output-json;
- the presets block between the two marker comments is rewritten with 4-tuples
  (BLOCK_M, BLOCK_N, NUM_STAGES, PERSISTENT_CTAS) (reference rewrite: :277-317).

The vendor baseline is the evaluator's `_baseline_attention` when --evaluate-module is given
(with the torch_npu stand-in in flash_attn_npu_b200/npu_shim answering it on CUDA), otherwise
torch's scaled_dot_product_attention.
"""
from __future__ import annotations

import argparse
import dataclasses
import importlib.util
import json
import multiprocessing as mp
import queue
import statistics
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
if str(HERE) not in sys.path:
    sys.path.insert(0, str(HERE))

DEFAULT_SM_SCALE = 0.5
DEFAULT_SEED = 0
DEFAULT_TUNE_ITERS = 3
DEFAULT_FINAL_ITERS = 5
DEFAULT_OUTPUT_JSON = "flash_attention_forward_tuned.json"
DEFAULT_CANDIDATE_MODULE = "flash_attention_forward.py"
DEFAULT_TIMEOUT_S = 60.0

PRESET_BEGIN = "# BEGIN AUTO-TUNED DEFAULT TILING PRESETS"
PRESET_END = "# END AUTO-TUNED DEFAULT TILING PRESETS"

# The reference evaluator's PERFORMANCE_CASES (evaluate_attention.py:36-43), used when no
# --shape and no --evaluate-module is given.
DEFAULT_SHAPES = [
    (128, 8, 1024, 128, True),
    (128, 8, 1024, 256, True),
    (128, 8, 2048, 128, True),
    (128, 8, 2048, 256, False),
    (128, 8, 4096, 128, False),
    (128, 8, 8192, 64, False),
]


# ------------------------------------------------------------------------- shape keys
_TRUE_WORDS = frozenset(("1", "true", "t", "yes", "y"))
_FALSE_WORDS = frozenset(("0", "false", "f", "no", "n"))


@dataclasses.dataclass(frozen=True, order=True)
class ShapeKey:
    """One tuned shape.  Its text forms are the interface the tuner shares with its users:
    `Z:H:N_CTX:HEAD_DIM:causal01` keys in `tuned_configs`, the `Z/H/N_CTX/HEAD_DIM/causal`
    fields of each `results` row, and `Z,H,N_CTX,HEAD_DIM,causal` on the command line."""

    z: int
    h: int
    n_ctx: int
    head_dim: int
    causal: bool

    @classmethod
    def from_cli(cls, text: str) -> "ShapeKey":
        fields = [f.strip() for f in str(text).split(",")]
        if len(fields) != 5:
            raise ValueError(f"--shape wants five comma-separated fields "
                             f"Z,H,N_CTX,HEAD_DIM,causal; got {text!r}")
        flag = fields[4].lower()
        if flag not in _TRUE_WORDS | _FALSE_WORDS:
            raise ValueError(f"causal field of --shape must be a boolean word, got {fields[4]!r}")
        return cls(*(int(f) for f in fields[:4]), flag in _TRUE_WORDS)

    @classmethod
    def from_record(cls, rec: dict) -> "ShapeKey":
        return cls(int(rec["Z"]), int(rec["H"]), int(rec["N_CTX"]), int(rec["HEAD_DIM"]),
                   bool(rec["causal"]))

    @classmethod
    def from_key(cls, key: str) -> "ShapeKey":
        z, h, n_ctx, head_dim, causal = (int(x) for x in key.split(":"))
        return cls(z, h, n_ctx, head_dim, bool(causal))

    def key(self) -> str:
        return ":".join(str(x) for x in (*self.as_tuple()[:4], int(self.causal)))

    def record(self) -> dict:
        return dict(zip(("Z", "H", "N_CTX", "HEAD_DIM", "causal"), self.as_tuple()))

    def as_tuple(self) -> tuple:
        return (self.z, self.h, self.n_ctx, self.head_dim, self.causal)


def load_module_from_path(path: Path, name: str):
    """Import a Python file by path (the candidate module or the evaluator)."""
    spec = importlib.util.spec_from_file_location(name, str(path))
    if spec is None or spec.loader is None:
        raise ImportError(f"cannot import {path}")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def _dtype_from_name(name: str):
    import torch
    normalized = name.strip().lower()
    if normalized in {"float16", "fp16"}:
        return torch.float16
    if normalized in {"bfloat16", "bf16"}:
        return torch.bfloat16
    raise ValueError(f"Unsupported dtype: {name}")


def _generate_tiling_candidates(shape, dtype_name: str = "float16"):
    """Every sm_100a tile the kernel family instantiates for this head_dim / dtype, as dicts
    with BLOCK_M, BLOCK_N, NUM_STAGES, PERSISTENT_CTAS.  Sequences of at most 128 rows skip
    the two-tile BLOCK_M=256 variants (the second tile would be all padding)."""
    from flash_attn_npu_b200 import tiling
    _z, _h, n_ctx, head_dim, _causal = shape
    dtype = _dtype_from_name(dtype_name)
    out = []
    for cfg in tiling.candidates(head_dim, dtype):
        if cfg.block_m == 256 and n_ctx <= 128:
            continue
        out.append(cfg.as_dict())
    return out


def _error_summary(exc) -> str:
    message = str(exc).strip()
    if not message:
        return exc.__class__.__name__
    return message.splitlines()[0][:240]


def _stats(samples_us):
    return {"avg_us": statistics.mean(samples_us), "min_us": min(samples_us),
            "max_us": max(samples_us), "median_us": statistics.median(samples_us)}


# ------------------------------------------------------------------------- worker side
def _worker_main(module_path, shape, dtype_name, sm_scale, seed, iters, tasks, results):
    """Child process: time candidates handed over `tasks` until it receives None."""
    try:
        import torch
        module = load_module_from_path(Path(module_path), "flash_attention_candidate")
        z, h, n_ctx, head_dim, causal = shape
        dtype = _dtype_from_name(dtype_name)
        torch.manual_seed(seed)
        dev = getattr(module, "DEVICE", "cuda")
        q = torch.empty((z, h, n_ctx, head_dim), dtype=dtype, device=dev).normal_(0.0, 0.5)
        k = torch.empty_like(q).normal_(0.0, 0.5)
        v = torch.empty_like(q).normal_(0.0, 0.5)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
    except Exception as exc:  # noqa: BLE001
        results.put(("fatal", _error_summary(exc)))
        return
    results.put(("ready", None))
    while True:
        cfg = tasks.get()
        if cfg is None:
            return
        try:
            if hasattr(module, "_launch_kernel_config"):
                def run():
                    return module._launch_kernel_config(q, k, v, causal, sm_scale, cfg)
            else:
                def run():
                    return module._launch_kernel(q, k, v, causal, sm_scale,
                                                 bm=cfg["BLOCK_M"], bn=cfg["BLOCK_N"])
            run()
            torch.cuda.synchronize()
            samples = []
            for _ in range(iters):
                start.record()
                run()
                end.record()
                end.synchronize()
                samples.append(start.elapsed_time(end) * 1e3)
            results.put(("ok", {"config": cfg, **_stats(samples)}))
        except Exception as exc:  # noqa: BLE001
            results.put(("ok", {"config": cfg, "avg_us": None, "error": _error_summary(exc)}))


class _Pool:
    """One spawned worker per shape; replaced whenever a candidate crashes or times out."""

    def __init__(self, module_path, shape, dtype_name, sm_scale, seed, iters, timeout_s):
        self.args = (str(module_path), shape, dtype_name, sm_scale, seed, iters)
        self.timeout_s = timeout_s
        self.ctx = mp.get_context("spawn")
        self.proc = None

    def _start(self):
        self.tasks = self.ctx.Queue()
        self.results = self.ctx.Queue()
        self.proc = self.ctx.Process(target=_worker_main, args=(*self.args, self.tasks, self.results),
                                     daemon=True)
        self.proc.start()
        kind, payload = self.results.get(timeout=max(self.timeout_s, 120.0))
        if kind == "fatal":
            self.close()
            raise RuntimeError(f"worker could not start: {payload}")

    def measure(self, cfg):
        if self.proc is None or not self.proc.is_alive():
            self._start()
        self.tasks.put(cfg)
        deadline = time.monotonic() + self.timeout_s
        while True:
            try:
                kind, payload = self.results.get(timeout=1.0)
                return payload
            except queue.Empty:
                if not self.proc.is_alive():
                    self.proc = None
                    return {"config": cfg, "avg_us": None,
                            "error": f"worker exited with code {self._exitcode()}"}
                if time.monotonic() > deadline:
                    self.close()
                    return {"config": cfg, "avg_us": None,
                            "error": f"timed out after {self.timeout_s:.0f} s"}

    def _exitcode(self):
        return None if self.proc is None else self.proc.exitcode

    def close(self):
        if self.proc is not None:
            try:
                self.tasks.put(None)
                self.proc.join(timeout=5)
            except Exception:
                pass
            if self.proc.is_alive():
                self.proc.kill()
                self.proc.join(timeout=5)
        self.proc = None


# ------------------------------------------------------------------------- parent side
def _measure_in_process(fn, iters, torch):
    fn()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    samples, out = [], None
    for _ in range(iters):
        start.record()
        out = fn()
        end.record()
        end.synchronize()
        samples.append(start.elapsed_time(end) * 1e3)
    return out, {**_stats(samples), "samples_us": samples, "iters": iters}


def _baseline_fn(eval_module, q, k, v, h, causal, sm_scale):
    import torch
    if eval_module is not None and hasattr(eval_module, "_baseline_attention"):
        return lambda: eval_module._baseline_attention(q, k, v, h, causal, sm_scale)
    return lambda: torch.nn.functional.scaled_dot_product_attention(
        q, k, v, is_causal=causal, scale=sm_scale)


def tune_case(module, module_path, eval_module, shape, dtype_name, sm_scale, seed, tune_iters,
              final_iters, timeout_s, use_subprocess=True):
    import torch
    z, h, n_ctx, head_dim, causal = shape
    candidate_rows = []
    configs = _generate_tiling_candidates(shape, dtype_name)
    if use_subprocess:
        pool = _Pool(module_path, shape, dtype_name, sm_scale, seed, tune_iters, timeout_s)
        try:
            for cfg in configs:
                candidate_rows.append(pool.measure(cfg))
        finally:
            pool.close()
    dtype = _dtype_from_name(dtype_name)
    torch.manual_seed(seed)
    dev = module.DEVICE
    q = torch.empty((z, h, n_ctx, head_dim), dtype=dtype, device=dev).normal_(0.0, 0.5)
    k = torch.empty_like(q).normal_(0.0, 0.5)
    v = torch.empty_like(q).normal_(0.0, 0.5)

    def launch(cfg):
        return module._launch_kernel_config(q, k, v, causal, sm_scale, cfg)[0]

    if not use_subprocess:
        for cfg in configs:
            try:
                _, st = _measure_in_process(lambda: launch(cfg), tune_iters, torch)
                candidate_rows.append({"config": cfg, "avg_us": st["avg_us"],
                                       "min_us": st["min_us"], "max_us": st["max_us"]})
            except Exception as exc:  # noqa: BLE001
                candidate_rows.append({"config": cfg, "avg_us": None,
                                       "error": _error_summary(exc)})

    viable = [row for row in candidate_rows if row.get("avg_us") is not None]
    viable.sort(key=lambda row: row["avg_us"])
    if not viable:
        raise RuntimeError(f"no viable config found for shape {shape}")
    best = viable[0]["config"]
    candidate_out, cand_stats = _measure_in_process(lambda: launch(best), final_iters, torch)
    ref_out, base_stats = _measure_in_process(
        _baseline_fn(eval_module, q, k, v, h, causal, sm_scale), final_iters, torch)
    try:
        max_abs_diff = torch.max(torch.abs(candidate_out.float() - ref_out.float())).item()
        correctness_error = None
    except Exception as exc:  # noqa: BLE001
        max_abs_diff, correctness_error = None, _error_summary(exc)
    result = {
        **ShapeKey(*shape).record(),
        "best_config": best,
        "candidate_avg_us": cand_stats["avg_us"],
        "candidate_min_us": cand_stats["min_us"],
        "candidate_max_us": cand_stats["max_us"],
        "baseline_avg_us": base_stats["avg_us"],
        "baseline_min_us": base_stats["min_us"],
        "baseline_max_us": base_stats["max_us"],
        "speedup_vs_baseline": base_stats["avg_us"] / cand_stats["avg_us"],
        "max_abs_diff": max_abs_diff,
        "correctness_error": correctness_error,
        "candidates": [{k2: v2 for k2, v2 in row.items() if k2 != "median_us"}
                       for row in candidate_rows],
    }
    del q, k, v
    return result


def merge_tuned_payloads(previous: dict, current: dict) -> dict:
    """Resume-by-merge: `current` wins shape by shape; `results` keep first-seen order."""
    rows: dict[ShapeKey, dict] = {}
    for row in list(previous.get("results", [])) + list(current.get("results", [])):
        if isinstance(row, dict):
            rows[ShapeKey.from_record(row)] = row  # dict keeps the first insertion position
    merged = dict(current)
    merged["tuned_configs"] = {**previous.get("tuned_configs", {}),
                               **current.get("tuned_configs", {})}
    merged["results"] = list(rows.values())
    return merged


def merge_into_existing(output_path: Path, payload: dict) -> dict:
    """Merge `payload` with the JSON already at `output_path` (unreadable or absent: as is)."""
    try:
        previous = json.loads(output_path.read_text(encoding="utf-8"))
    except (OSError, ValueError):
        return payload
    return merge_tuned_payloads(previous, payload) if isinstance(previous, dict) else payload


_PRESET_HEADER = (
    "# Default tiling presets captured from offline tuning.",
    "# This block is rewritten by `tune_flash_attention_forward.py`.",
    "# (Z, H, N_CTX, HEAD_DIM, causal): (BLOCK_M, BLOCK_N, NUM_STAGES, PERSISTENT_CTAS)",
)


def render_presets_block(tuned_configs: dict) -> str:
    """The text between (and including) the two markers for a `tuned_configs` table."""
    knobs = ("BLOCK_M", "BLOCK_N", "NUM_STAGES", "PERSISTENT_CTAS")
    entries = sorted((ShapeKey.from_key(k), cfg) for k, cfg in tuned_configs.items())
    body = [f"    {shape.as_tuple()!r}: ({', '.join(str(int(cfg.get(n, 0))) for n in knobs)}),"
            for shape, cfg in entries]
    return "\n".join([PRESET_BEGIN, *_PRESET_HEADER, "DEFAULT_TILING_PRESETS = {", *body, "}",
                      PRESET_END])


def write_presets(module_path: Path, tuned_json_path: Path) -> None:
    """Replace the presets block of `module_path` with the table in `tuned_json_path`."""
    tuned_configs = json.loads(tuned_json_path.read_text(encoding="utf-8")).get(
        "tuned_configs") or {}
    if not tuned_configs:
        raise ValueError(f"{tuned_json_path} holds no tuned_configs")
    text = module_path.read_text(encoding="utf-8")
    head, sep, rest = text.partition(PRESET_BEGIN)
    _, sep_end, tail = rest.partition(PRESET_END)
    if not sep or not sep_end:
        raise RuntimeError(f"{module_path} lacks the preset markers {PRESET_BEGIN!r} / "
                           f"{PRESET_END!r}")
    module_path.write_text(head + render_presets_block(tuned_configs) + tail, encoding="utf-8")


def build_arg_parser():
    parser = argparse.ArgumentParser(
        description="Offline tune flash_attention_forward.py (sm_100a) and optionally apply tuned "
                    "tiling presets.")
    parser.add_argument("--candidate-module",
                        default=str(HERE / DEFAULT_CANDIDATE_MODULE),
                        help="Path to flash_attention_forward.py")
    parser.add_argument("--evaluate-module", default=None,
                        help="Optional path to the reference evaluate_attention.py (its "
                             "_baseline_attention and PERFORMANCE_CASES are used)")
    parser.add_argument("--output-json", default=str(HERE / DEFAULT_OUTPUT_JSON),
                        help="Path to write tuned configs JSON")
    parser.add_argument("--sm-scale", type=float, default=DEFAULT_SM_SCALE)
    parser.add_argument("--seed", type=int, default=DEFAULT_SEED)
    parser.add_argument("--dtype", default="float16",
                        choices=["float16", "fp16", "bfloat16", "bf16"])
    parser.add_argument("--tune-iters", type=int, default=DEFAULT_TUNE_ITERS)
    parser.add_argument("--final-iters", type=int, default=DEFAULT_FINAL_ITERS)
    parser.add_argument("--timeout", type=float, default=DEFAULT_TIMEOUT_S,
                        help="wall-clock limit per candidate (seconds)")
    parser.add_argument("--no-subprocess", action="store_true",
                        help="time candidates in this process (no fault isolation)")
    parser.add_argument("--replace-output", action="store_true",
                        help="Overwrite output JSON instead of merging new shapes into it.")
    parser.add_argument("--shape", action="append",
                        help="Shape 'Z,H,N_CTX,HEAD_DIM,causal'. May be passed multiple times.")
    parser.add_argument("--skip-apply", action="store_true",
                        help="Only write tuned JSON, do not rewrite the presets block.")
    parser.add_argument("--apply-only", action="store_true",
                        help="Skip tuning and only rewrite the presets block from the JSON.")
    return parser


def main(argv=None):
    args = build_arg_parser().parse_args(argv)
    candidate_module_path = Path(args.candidate_module).resolve()
    output_json_path = Path(args.output_json).resolve()
    if args.apply_only:
        write_presets(candidate_module_path, output_json_path)
        print(f"Applied tuned presets from {output_json_path} to {candidate_module_path}")
        return 0

    candidate_module = load_module_from_path(candidate_module_path, "flash_attention_candidate")
    evaluate_module = None
    if args.evaluate_module:
        shim = HERE / "flash_attn_npu_b200" / "npu_shim"
        if str(shim) not in sys.path:
            sys.path.insert(0, str(shim))
        evaluate_module = load_module_from_path(Path(args.evaluate_module).resolve(),
                                       "flash_attention_evaluate")
    if args.shape:
        shapes = [ShapeKey.from_cli(raw).as_tuple() for raw in args.shape]
    elif evaluate_module is not None:
        shapes = [tuple(s) for s in evaluate_module.PERFORMANCE_CASES]
    else:
        shapes = list(DEFAULT_SHAPES)

    results = []
    for idx, shape in enumerate(shapes, start=1):
        print(f"[{idx}/{len(shapes)}] tuning shape={shape}", flush=True)
        result = tune_case(candidate_module, candidate_module_path, evaluate_module, shape,
                           args.dtype, args.sm_scale, args.seed, args.tune_iters,
                           args.final_iters, args.timeout, not args.no_subprocess)
        print("  best: "
              f"config={result['best_config']}, "
              f"candidate_avg_us={result['candidate_avg_us']:.3f}, "
              f"baseline_avg_us={result['baseline_avg_us']:.3f}, "
              f"speedup={result['speedup_vs_baseline']:.3f}", flush=True)
        results.append(result)

    tuned_table = {ShapeKey.from_record(item).key(): item["best_config"] for item in results}
    import torch
    payload = {
        "meta": {
            # file names only: the JSON is committed and must not carry machine paths
            "candidate_module": candidate_module_path.name,
            "evaluate_module": Path(args.evaluate_module).name if args.evaluate_module else None,
            "dtype": args.dtype,
            "sm_scale": args.sm_scale,
            "seed": args.seed,
            "tune_iters": args.tune_iters,
            "final_iters": args.final_iters,
            "timeout_s": args.timeout,
            "device": torch.cuda.get_device_name(0) if torch.cuda.is_available() else None,
            "baseline": "evaluate_module._baseline_attention" if evaluate_module is not None
            else "torch.nn.functional.scaled_dot_product_attention",
        },
        "tuned_configs": tuned_table,
        "results": results,
    }
    if not args.replace_output:
        payload = merge_into_existing(output_json_path, payload)
    output_json_path.write_text(json.dumps(payload, indent=2, ensure_ascii=True) + "\n",
                                encoding="utf-8")
    print(f"Tuned config JSON written to: {output_json_path}")
    if not args.skip_apply:
        write_presets(candidate_module_path, output_json_path)
        print(f"Applied tuned presets to: {candidate_module_path}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
