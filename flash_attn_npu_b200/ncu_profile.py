"""Hardware counters for `profiling()` from Nsight Compute.

The reference's `profiling()` (flash_attention_forward.py:1218-1289) collects Ascend AiCore
metric groups with torch_npu's profiler, one pass per group, and summarises them into
`result_dir/profile_summary.json`.  On B200 the counters come from `ncu`: one child process runs
the module's one-launch command (`flash_attention_forward.py tune ...`) under

    ncu --clock-control none --metrics <groups> -k regex:fa_fwd_sm100 -c 1 --csv --page raw

and the raw page is parsed into the same {group: {metric: value}} shape.  The child command is
first run once without ncu and must exit 0 (a kernel that faults is never profiled).  Workloads
whose inputs exceed `MAX_MULTIPASS_BYTES` get `LARGE_INPUT_GROUPS` only -- the launch duration
`gpu__time_duration.sum`, which ncu collects in one pass.  Every other metric (the clock rate
included) needs replay passes that save and restore the program's device memory, so those stay
on inputs below the cap.
"""
from __future__ import annotations

import csv
import io
import shutil
import subprocess
from pathlib import Path

KERNEL_REGEX = "regex:fa_fwd_sm100"

METRIC_GROUPS: dict[str, list[str]] = {
    "Timing": ["gpu__time_duration.sum", "sm__cycles_elapsed.avg.per_second"],
    "SpeedOfLight": ["sm__throughput.avg.pct_of_peak_sustained_elapsed",
                     "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
                     "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed"],
    "Memory": ["dram__bytes_read.sum", "dram__bytes_write.sum"],
    "Pipes": ["sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
              "sm__inst_executed_pipe_xu.avg.pct_of_peak_sustained_active",
              "sm__pipe_fma_cycles_active.avg.pct_of_peak_sustained_active",
              "sm__pipe_alu_cycles_active.avg.pct_of_peak_sustained_active"],
    "Issue": ["sm__inst_executed.avg.per_cycle_active",
              "sm__warps_active.avg.pct_of_peak_sustained_active",
              "smsp__average_warps_issue_stalled_long_scoreboard_per_issue_active.ratio",
              "launch__registers_per_thread", "launch__grid_size"],
}
# Above the cap only the launch duration is collected (one pass, nothing saved or restored).
LARGE_INPUT_GROUPS: dict[str, list[str]] = {"Timing": ["gpu__time_duration.sum"]}
MAX_MULTIPASS_BYTES = 2 << 30


def groups_for_input_bytes(in_bytes: int) -> dict[str, list[str]]:
    """Metric groups one capture may collect for a workload whose q, k, v take `in_bytes`."""
    return METRIC_GROUPS if in_bytes <= MAX_MULTIPASS_BYTES else LARGE_INPUT_GROUPS


def ncu_path() -> str | None:
    found = shutil.which("ncu")
    if found:
        return found
    cand = Path("/usr/local/cuda/bin/ncu")
    return str(cand) if cand.exists() else None


def parse_raw_csv(text: str) -> list[dict[str, float | str]]:
    """Rows of `ncu --csv --page raw` (header, units, one row per profiled launch)."""
    lines = [ln for ln in text.splitlines() if ln.startswith('"')]
    if len(lines) < 3:
        return []
    rows = list(csv.reader(io.StringIO("\n".join(lines))))
    header, data = rows[0], rows[2:]
    out = []
    for r in data:
        rec: dict[str, float | str] = {}
        for name, val in zip(header, r):
            v = val.replace(",", "")
            try:
                rec[name] = float(v)
            except ValueError:
                rec[name] = val
        out.append(rec)
    return out


def group_summary(row: dict, groups: dict[str, list[str]]) -> dict[str, dict[str, float]]:
    return {g: {m: row[m] for m in ms if m in row and isinstance(row[m], float)}
            for g, ms in groups.items()}


def profile(child_argv: list[str], groups: dict[str, list[str]] | None = None,
            timeout_s: float = 600.0, cwd: str | None = None) -> dict:
    """Run `child_argv` plainly, then once under ncu; return {"groups": ..., "command": ...}.

    Raises RuntimeError when ncu is missing, the plain run fails, or ncu reports no launch.
    """
    groups = groups or METRIC_GROUPS
    ncu = ncu_path()
    if ncu is None:
        raise RuntimeError("ncu not found")
    plain = subprocess.run(child_argv, capture_output=True, text=True, timeout=timeout_s, cwd=cwd)
    if plain.returncode != 0:
        raise RuntimeError(f"plain run failed (rc={plain.returncode}): {plain.stderr[-500:]}")
    metrics = sorted({m for ms in groups.values() for m in ms})
    cmd = [ncu, "--clock-control", "none", "--metrics", ",".join(metrics), "-k", KERNEL_REGEX,
           "-c", "1", "--csv", "--page", "raw", *child_argv]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout_s, cwd=cwd)
    rows = parse_raw_csv(res.stdout)
    if res.returncode != 0 or not rows:
        raise RuntimeError(f"ncu failed (rc={res.returncode}): {(res.stderr or res.stdout)[-500:]}")
    return {"groups": group_summary(rows[0], groups), "command": " ".join(cmd)}
