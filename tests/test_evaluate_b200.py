"""The restated evaluator (evaluate_attention_b200.py): its statistics and score on the CPU, its
correctness suite on the GPU."""
from __future__ import annotations

import json
import statistics

import pytest

import evaluate_attention_b200 as ev
from flash_attn_npu_b200 import inputs as fa_inputs


def test_sample_stats_known_series():
    xs = [5.0, 1.0, 4.0, 2.0, 3.0, 100.0, 6.0, 7.0, 8.0, 9.0]
    s = ev.sample_stats(xs, 0.1)
    assert s["min_us"] == 1.0 and s["max_us"] == 100.0 and s["iters"] == 10
    assert s["median_us"] == statistics.median(xs)
    # 10 % of 10 samples: one cut from each end -> mean of 2..9
    assert s["trimmed_avg_us"] == pytest.approx(sum(range(2, 10)) / 8)
    # linear-interpolated quantiles over the sorted series 1..9, 100
    assert s["p10_us"] == pytest.approx(1.9)
    assert s["p90_us"] == pytest.approx(9.0 + 0.1 * 91.0)
    # a trim ratio that would remove everything keeps the middle element
    assert ev.sample_stats([3.0, 1.0, 2.0], 0.5)["trimmed_avg_us"] == 2.0


def test_case_score_caps_at_full_points():
    assert ev.case_score(10.0, 100.0, 50.0) == (2.0, 10.0)
    sp, sc = ev.case_score(10.0, 80.0, 100.0)
    assert sp == pytest.approx(0.8) and sc == pytest.approx(8.0)
    assert ev.case_score(10.0, None, 50.0) == (None, 0.0)
    assert ev.case_score(10.0, 50.0, 0.0) == (None, 0.0)


def test_reports_round_trip(tmp_path):
    shape_c = fa_inputs.EVALUATOR_CORRECTNESS_CASES[0]
    shape_p = fa_inputs.EVALUATOR_PERFORMANCE_CASES[0]
    cor = [ev.CaseResult(shape_c, 0, passed=True, max_abs_diff=1e-3, score=40.0 / 18)]
    st = ev.sample_stats([10.0, 11.0, 12.0], 0.1)
    perf = [ev.CaseResult(shape_p, 18, passed=True, max_abs_diff=2e-3, baseline=st,
                          candidate=st, speedup=1.0, score=10.0),
            ev.CaseResult(shape_p, 19, error="RuntimeError: boom")]
    summary = {"config": {"candidate_module": "m.py", "device": "cpu", "dtype": "float16",
                          "speed_metric": "median_us"},
               "correctness": ev.summarize("correctness", cor, ev.CORRECTNESS_POINTS),
               "performance": ev.summarize("performance", perf, ev.PERFORMANCE_POINTS)}
    summary["total_score"] = summary["correctness"]["score"] + summary["performance"]["score"]
    j, t = ev.write_reports(tmp_path, summary)
    back = json.loads(j.read_text())
    assert back["performance"]["passed"] == 1 and back["performance"]["total"] == 2
    assert back["performance"]["mean_speedup"] == 1.0
    assert back["total_score"] == pytest.approx(40.0 / 18 + 10.0)
    text = t.read_text()
    assert "RuntimeError: boom" in text and "speedup=1.0000" in text


def test_cli_defaults_follow_the_reference_evaluator():
    a = ev.build_parser().parse_args([])
    assert (a.sm_scale, a.atol, a.rtol, a.warmup, a.iters, a.speed_metric, a.trim_ratio) == \
        (0.5, 1e-2, 1e-2, 5, 30, "median_us", 0.1)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_correctness_suite_passes_on_gpu(dtype, tmp_path, cuda_device):
    s = ev.main(["--mode", "correctness", "--dtype", dtype, "--report-dir", str(tmp_path)])
    cor = s["correctness"]
    assert cor["passed"] == cor["total"] == len(fa_inputs.EVALUATOR_CORRECTNESS_CASES), \
        [c for c in cor["cases"] if not c["passed"]]
    assert cor["score"] == pytest.approx(ev.CORRECTNESS_POINTS)
