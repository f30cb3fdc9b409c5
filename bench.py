#!/usr/bin/env python3
"""Benchmark: attention forward TFLOP/s on B200 (headline workload cfg4).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload cfg4]

Metric: "attention fwd TFLOP/s and % of B200 bf16 peak at S=8K,D=128;
1/2/4/8 GPUs".  Workload cfg4: B=16, H=16, S=8192, D=128, bf16, non-causal,
sm_scale=1/sqrt(128), q/k/v ~ N(0,1) from seed 3 (synthetic; no dataset).  One step is one
forward pass over the whole batch.  With N GPUs (torchrun, one process per GPU) the 256
(b, h) slices are split into contiguous ranges, one per rank, with no communication on the
hot path; total work is fixed, so scaling is "strong".  `value` = whole-job FLOPs per step
(4*B*H*S^2*D) / the max over ranks of the device time per step.

Timing: W untimed warm-up steps, then K steps bracketed by barrier + cuda.synchronize on both
sides, CUDA events on the launching stream.  Inputs (3 x 512 MiB at N=1) are larger than the
126 MB L2, so no flush is needed between steps.  `e2e` times the public host-buffer call
(`flash_attention_forward.attention_host`) on pinned host q, k, v: every step copies q, k, v
to the device and out, lse back, with the (b, h) slices streamed in chunks so that the copies
overlap the kernels.

`--impl reference` times the reference's CPU attention path (the oracle restatement of
evaluate_attention.py:134-143 in oracle/attention_ref.py) on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

import torch  # noqa: E402

FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}


# ----------------------------------------------------------------------------- helpers
def _dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return {"bf16_tflops": float(d["bf16_tflops"]),
                    "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained",
                                                         d["bf16_tflops"])),
                    "hbm_gbs": float(d.get("hbm_gbs", 0.0))}, "measured"
        except Exception:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def load_traffic(workload: str):
    """DRAM bytes per launch of the kernel from a committed ncu summary (None if absent)."""
    p = REPO / "profiles" / f"fa_fwd_{workload}_traffic.json"
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        return float(d["dram_bytes_per_launch_full"])
    except Exception:
        return None


class ClockSampler:
    """Samples SM clock and throttle reasons with nvidia-smi while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int, interval_ms: int = 50):
        self.idx = device_index
        self.interval_ms = interval_ms
        self.proc = None
        self.lines = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 f"-i", str(self.idx), f"-lms", str(self.interval_ms)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self._t:
            self._t.join(timeout=2)
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sms:
            return None
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes),
                "reasons": sorted(reasons), "samples": len(sms)}


def cpu_reference_rate(cfg, budget_s: float, q=None, k=None, v=None, rows=2048):
    """Time the CPU oracle on (b, h) slices of the workload: each sample is the first `rows`
    query rows of one slice against all of its keys.  Returns (TFLOP/s, description, threads).
    """
    from oracle.attention_ref import attention_ref_torch
    from flash_attn_npu_b200 import inputs as fa_inputs

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    if q is None:
        g = torch.Generator().manual_seed(cfg.seed)
        shp = (cfg.seqlen, cfg.head_dim)
        q, k, v = (torch.randn(shp, generator=g).to(cfg.dtype) for _ in range(3))
        slices = [(q, k, v)]
    else:
        slices = [(q[b, h], k[b, h], v[b, h]) for b in range(cfg.batch) for h in range(cfg.heads)]
    rows = min(rows, cfg.seqlen)
    # causal sample = the first `rows` rows (a rows x rows triangle); else rows x all keys
    flops_one = (2.0 * rows * rows * cfg.head_dim if cfg.causal
                 else 4.0 * rows * cfg.seqlen * cfg.head_dim)
    done, t_total, i = 0, 0.0, 0
    attention_ref_torch(slices[0][0][:rows], slices[0][1], slices[0][2], False, cfg.sm_scale)
    while t_total < budget_s or done == 0:
        qs, ks, vs = slices[i % len(slices)]
        t0 = time.perf_counter()
        if cfg.causal:
            attention_ref_torch(qs[:rows], ks[:rows], vs[:rows], True, cfg.sm_scale)
        else:
            attention_ref_torch(qs[:rows], ks, vs, False, cfg.sm_scale)
        t_total += time.perf_counter() - t0
        done += 1
        i += 1
    rate = done * flops_one / t_total / 1e12
    desc = (f"{done} samples of {rows} query rows x {cfg.seqlen} keys (one (b,h) slice each), "
            f"fp32 torch CPU, {t_total:.1f} s")
    return rate, desc, threads, t_total / done


def library_rate(q, k, v, cfg, stream, steps):
    """TFLOP/s of torch.nn.functional.scaled_dot_product_attention with the cuDNN backend on
    the bench's own device inputs ([n, 1, S, D] slices), timed like the headline.  Context
    only; {"unavailable": ...} if the backend refuses the shape."""
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel
    try:
        with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
            def run():
                return F.scaled_dot_product_attention(q, k, v, is_causal=cfg.causal,
                                                      scale=cfg.sm_scale)
            for _ in range(3):
                run()
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(steps):
                run()
            e1.record(stream)
            torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
    except Exception as exc:  # noqa: BLE001
        return {"kernel": "torch sdpa (cuDNN)", "unavailable": type(exc).__name__}
    flops = fa_flops_local(q, cfg)
    return {"kernel": "torch.nn.functional.scaled_dot_product_attention, cuDNN backend",
            "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms}


def kernel_label(cfg, fam):
    """Which kernel the workload's default tile runs on (one launch per step either way)."""
    from flash_attn_npu_b200 import tiling
    tc = tiling.TileConfig.from_preset(fam.get_tile_config(cfg.batch, cfg.heads, cfg.seqlen,
                                                          cfg.head_dim, cfg.causal, cfg.dtype))
    if tiling.persistent_kernel_serves(cfg.head_dim, cfg.dtype, tc, cfg.sm_scale):
        return "fa_fwd_ws_kernel (persistent, one launch per step)"
    return "fa_fwd_sm100_kernel (one CTA per tile, one launch per step)"


XU_EX2_PER_CLK_PER_SM = 16


def xu_roofline(n_slices, cfg, ms, clocks, dev):
    """Exponentials per second against the exp2 unit's throughput: one exp per (query, key)
    pair, S^2 per (b, h) slice, S (S + 1) / 2 under a causal mask."""
    S = cfg.seqlen
    exps = n_slices * (S * (S + 1) / 2 if cfg.causal else S * S)
    mhz = (clocks or {}).get("sm_mhz") or (clocks or {}).get("sm_max_mhz") or 1965.0
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    peak = XU_EX2_PER_CLK_PER_SM * sms * mhz * 1e6 / 1e12
    achieved = exps / (ms * 1e-3) / 1e12
    return {"bound": "xu", "achieved": achieved, "peak": peak, "unit": "Texp/s",
            "frac": achieved / peak, "exps_per_launch": exps,
            "peak_source": f"{XU_EX2_PER_CLK_PER_SM} ex2/clk/SM x {sms} SMs x {mhz:.0f} MHz"}


def fa_flops_local(q, cfg):
    n = q.shape[0] * q.shape[1]
    f = 4.0 * n * cfg.seqlen * cfg.seqlen * cfg.head_dim
    return f * 0.5 if cfg.causal else f


# ----------------------------------------------------------------------------- arms
def run_reference(args, cfg, world, rank):
    """Reference arm: the reference's CPU attention path on the host cores (rank 0 only)."""
    if rank != 0:
        return 0
    torch.set_num_threads(os.cpu_count() or 1)
    from oracle.attention_ref import attention_ref_torch

    g = torch.Generator().manual_seed(cfg.seed)
    shp = (cfg.seqlen, cfg.head_dim)
    q, k, v = (torch.randn(shp, generator=g).to(cfg.dtype) for _ in range(3))
    rows = min(args.ref_rows, cfg.seqlen)
    flops = (2.0 * rows * rows * cfg.head_dim if cfg.causal
             else 4.0 * rows * cfg.seqlen * cfg.head_dim)

    def step():
        if cfg.causal:
            attention_ref_torch(q[:rows], k[:rows], v[:rows], True, cfg.sm_scale)
        else:
            attention_ref_torch(q[:rows], k, v, False, cfg.sm_scale)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    value = flops / dt / 1e12
    threads = torch.get_num_threads()
    keys = f"keys [0,{rows}) (causal)" if cfg.causal else f"all {cfg.seqlen} keys"
    sample = (f"per step: query rows [0,{rows}) of one (b,h) slice of {cfg.name} against "
              f"{keys} (fp32 torch CPU restatement of evaluate_attention.py:134-143)")
    line = {
        "impl": "reference",
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {**cfg.describe(), "parallelism": "host cores, rank 0 only"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


METRIC = "attention fwd TFLOP/s and % of B200 bf16 peak at S=8K,D=128; 1/2/4/8 GPUs"


def run_ours(args, cfg, world, rank, local):
    import flash_attention_forward as fam
    from flash_attn_npu_b200 import inputs as fa_inputs
    from flash_attn_npu_b200 import sharding
    from oracle.attention_ref import attention_ref_torch

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    # inputs: drawn on the CPU generator (identical bits on every rank), this rank's slices.
    # Every rank draws the full tensors, so with N ranks on one host each takes 1/N of the
    # cores for it instead of all of them oversubscribing the host.
    threads = torch.get_num_threads()
    if world > 1:
        torch.set_num_threads(max(1, (os.cpu_count() or 1) // world))
    q_cpu, k_cpu, v_cpu = fa_inputs.make_inputs(cfg, "cpu")
    torch.set_num_threads(threads)
    n_slices = cfg.batch * cfg.heads
    start, stop = sharding.shard_range(n_slices, world, rank)
    n_local = stop - start

    def local_view(t):
        return t.reshape(n_slices, 1, cfg.seqlen, cfg.head_dim)[start:stop]

    q_h = local_view(q_cpu).contiguous().pin_memory()
    k_h = local_view(k_cpu).contiguous().pin_memory()
    v_h = local_view(v_cpu).contiguous().pin_memory()
    q, k, v = (t.to(dev) for t in (q_h, k_h, v_h))
    local_flops = fa_inputs.attention_flops(n_local, 1, cfg.seqlen, cfg.head_dim, cfg.causal)
    total_flops = cfg.flops()
    stream = torch.cuda.current_stream(dev)

    def step():
        return fam._launch_kernel(q, k, v, cfg.causal, cfg.sm_scale)

    def barrier():
        if dist is not None:
            dist.barrier()

    # ---- warm-up
    for _ in range(args.warmup):
        out, lse = step()
    torch.cuda.synchronize(dev)

    # ---- timed region (device time, max over ranks)
    sampler = ClockSampler(local).start() if rank == 0 and not args.no_clocks else None
    if sampler is not None:
        time.sleep(0.3)  # let nvidia-smi start sampling
    barrier()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        out, lse = step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clocks = sampler.stop() if sampler is not None else None
    local_ms = e0.elapsed_time(e1) / args.steps
    ms = local_ms
    if dist is not None:
        t = torch.tensor([local_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    value = total_flops / (ms * 1e-3) / 1e12

    # ---- end-to-end through the public call with host buffers
    e2e_steps = max(1, args.e2e_steps)
    out_h = torch.empty(q_h.shape, dtype=q_h.dtype).pin_memory()
    lse_h = torch.empty((n_local, 1, cfg.seqlen), dtype=torch.float32).pin_memory()

    def e2e_step():
        # host q, k, v in; host out, lse back -- every byte crosses the host link each step
        fam.attention_host(q_h, k_h, v_h, cfg.causal, cfg.sm_scale, device=dev, out=out_h,
                           lse=lse_h, return_lse=True)

    # the host link's floor for the same bytes: q, k, v in while out, lse go back on a second
    # stream, no kernel (full duplex), best of 3
    qd_l, kd_l, vd_l, od_l = (torch.empty_like(t, device=dev) for t in (q_h, k_h, v_h, q_h))
    ld_l = torch.empty(lse_h.shape, dtype=torch.float32, device=dev)
    back = torch.cuda.Stream(dev)

    def link_only():
        back.wait_stream(stream)
        with torch.cuda.stream(back):
            out_h.copy_(od_l, non_blocking=True)
            lse_h.copy_(ld_l, non_blocking=True)
        qd_l.copy_(q_h, non_blocking=True)
        kd_l.copy_(k_h, non_blocking=True)
        vd_l.copy_(v_h, non_blocking=True)
        stream.wait_stream(back)

    # With N ranks on one host all of them copy at once (barrier first), as in the timed
    # end-to-end steps, so the floor includes their contention for the host.  Each round's
    # time is the max over ranks (the round in which all of them copied together); the floor
    # is the best such round.
    link_ms = float("inf")
    for _ in range(4):
        barrier()
        torch.cuda.synchronize(dev)
        l0 = torch.cuda.Event(enable_timing=True)
        l1 = torch.cuda.Event(enable_timing=True)
        l0.record(stream)
        link_only()
        l1.record(stream)
        torch.cuda.synchronize(dev)
        round_ms = l0.elapsed_time(l1)
        if dist is not None:
            t = torch.tensor([round_ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            round_ms = t.item()
        link_ms = min(link_ms, round_ms)
    del qd_l, kd_l, vd_l, od_l, ld_l

    e2e_step()
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    s0 = torch.cuda.Event(enable_timing=True)
    s1 = torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    s1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = s0.elapsed_time(s1) / e2e_steps
    if dist is not None:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = t.item()
    h2d = sum(t.numel() * t.element_size() for t in (q_h, k_h, v_h))
    d2h = out_h.numel() * out_h.element_size() + lse_h.numel() * 4
    # the streamed host path runs the same kernel per chunk: its results equal the device run's
    e2e_equal = bool(torch.equal(out_h, out.cpu()) and torch.equal(lse_h, lse.cpu()))

    # ---- verification (after timing): gather to rank 0, check sampled slices vs the oracle
    verify = None
    if not args.no_verify:
        out_all = lse_all = None
        if dist is not None:
            out_all = sharding.gather_shards(out, n_slices, world, rank)
            lse_all = sharding.gather_shards(lse, n_slices, world, rank)
        else:
            out_all, lse_all = out, lse
        if rank == 0:
            torch.backends.cuda.matmul.allow_tf32 = False
            picks = sorted({0, n_slices - 1, n_slices // 3, (2 * n_slices) // 3})
            worst_o = worst_m = worst_l = 0.0
            lse_ok = True
            for s in picks:
                b, h = divmod(s, cfg.heads)
                ro, rl = attention_ref_torch(q_cpu[b, h].to(dev), k_cpu[b, h].to(dev),
                                             v_cpu[b, h].to(dev), cfg.causal, cfg.sm_scale)
                err = (out_all[s, 0].float() - ro).abs()
                worst_o = max(worst_o, err.max().item())
                worst_m = max(worst_m, err.mean().item())
                lerr = (lse_all[s, 0] - rl).abs()
                worst_l = max(worst_l, lerr.max().item())
                # the parity tests' LSE bar: 1e-4 plus 2e-6 * |lse| (the relative term only
                # matters for rows with |lse| in the hundreds, e.g. cfg5's outliers, where one
                # fp32 ulp is already ~3e-5 and the fp32 oracle itself sits that far from fp64)
                lse_ok = lse_ok and bool((lerr <= 1e-4 + 2e-6 * rl.abs()).all())
            verify = {"slices": picks, "max_abs": worst_o, "mean_abs": worst_m,
                      "lse_max_abs": worst_l, "lse_bar": "1e-4 + 2e-6*|lse|",
                      "ok": (worst_o <= 2e-2 and worst_m <= 2e-3 and lse_ok and e2e_equal),
                      "e2e_bitwise_equal_rank0": e2e_equal,
                      "gathered_with": "nccl p2p" if dist is not None else "local"}

    # ---- context: the library attention kernel torch ships for this GPU (cuDNN through
    # scaled_dot_product_attention), same inputs, same timing method (rank 0, N = 1 only)
    library = None
    if rank == 0 and world == 1 and not args.no_library:
        library = library_rate(q, k, v, cfg, stream, args.steps)

    # ---- CPU baseline (rank 0, N = 1 only)
    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, desc, threads, _ = cpu_reference_rate(cfg, args.cpu_budget)
        cpu_baseline = {"value": rate, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                        "sample": desc}

    if rank == 0:
        peaks, peak_src = load_peaks()
        achieved = local_flops / (local_ms * 1e-3) / 1e12
        traffic = load_traffic(cfg.name)
        if traffic is not None and world > 1:
            traffic = traffic * n_local / n_slices
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16" if cfg.dtype == torch.bfloat16 else str(cfg.dtype).replace("torch.", ""),
            "data": "synthetic",
            "config": {**cfg.describe(), "global_batch": cfg.batch, "seq_len": cfg.seqlen,
                       "parallelism": f"bh-shard x{world}" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (no flush needed)",
                       "tile": fam.get_tile_config(cfg.batch, cfg.heads, cfg.seqlen,
                                                   cfg.head_dim, cfg.causal, cfg.dtype)},
            "pct_of_peak": 100.0 * value / (world * peaks["bf16_tflops"]),
            "e2e": {"value": total_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world, "steps": e2e_steps,
                    "link_floor_ms": link_ms,
                    "link_frac": link_ms / e2e_ms,
                    "path": "flash_attention_forward.attention_host: pinned host q, k, v in, "
                            "host out, lse back, copies overlapped with the kernels"},
            "gpu_launches": args.steps * world,
            "roofline": {"bound": "tensor", "achieved": achieved,
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": achieved / peaks["bf16_tflops"],
                         "frac_sustained": achieved / peaks["bf16_tflops_sustained"],
                         "peak_source": f"{peak_src} bf16 dense (burst)",
                         "traffic": traffic,
                         "kernel": kernel_label(cfg, fam)},
            # second limit of this kernel: the exp2 unit (16 ex2.approx results per clock per SM,
            # measured on B200), against the median SM clock sampled during the timed region
            # (nvidia-smi's figure, above the effective clock under the power cap, so this
            # fraction is a lower bound)
            "roofline_xu": xu_roofline(n_local, cfg, local_ms, clocks, dev),
            "clocks": clocks,
            "cpu_baseline": cpu_baseline,
            "context_library_kernel": library,
            "verify": verify,
        }
        print(json.dumps(line), flush=True)

    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="cfg4",
                    help="cfg2 | cfg3 | cfg4 | cfg5 (see flash_attn_npu_b200/inputs.py)")
    ap.add_argument("--e2e-steps", type=int, default=5, dest="e2e_steps")
    ap.add_argument("--cpu-budget", type=float, default=10.0, dest="cpu_budget",
                    help="seconds of CPU-oracle work for cpu_baseline")
    ap.add_argument("--ref-rows", type=int, default=1024, dest="ref_rows",
                    help="query rows per reference-arm step")
    ap.add_argument("--no-verify", action="store_true", dest="no_verify")
    ap.add_argument("--no-cpu-baseline", action="store_true", dest="no_cpu_baseline")
    ap.add_argument("--no-clocks", action="store_true", dest="no_clocks")
    ap.add_argument("--no-library", action="store_true", dest="no_library",
                    help="skip the context timing of torch's cuDNN attention kernel")
    args = ap.parse_args(argv)
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    from flash_attn_npu_b200 import inputs as fa_inputs
    cfg = fa_inputs.CONFIGS[args.workload]
    world, rank, local = _dist_env()
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    if args.impl == "reference":
        return run_reference(args, cfg, world, rank)
    return run_ours(args, cfg, world, rank, local)


if __name__ == "__main__":
    sys.exit(main())
