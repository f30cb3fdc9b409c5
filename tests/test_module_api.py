"""Host-side behaviour of the drop-in module, the tuner and the torch_npu shim (no GPU needed)."""
from __future__ import annotations

import importlib.util
import json
import os
import shutil
import sys
from pathlib import Path

import pytest
import torch

from conftest import REPO
import flash_attention_forward as fam
import tune_flash_attention_forward as tuner
from flash_attn_npu_b200 import tiling
from oracle.attention_ref import attention_ref_torch

def _reference_dir() -> Path:
    """Where the reference checkout lives: $FA_REFERENCE_DIR, else BASELINE.json's
    `reference_path` (absent on machines without the checkout; the test then skips)."""
    if os.environ.get("FA_REFERENCE_DIR"):
        return Path(os.environ["FA_REFERENCE_DIR"])
    try:
        return Path(json.loads((REPO / "BASELINE.json").read_text())["reference_path"])
    except Exception:
        return REPO / "_no_reference_checkout"


REFERENCE = _reference_dir()
SHIM = REPO / "flash_attn_npu_b200" / "npu_shim"


# ---------------------------------------------------------------- module surface
def test_reference_module_surface():
    """Every name the reference evaluator, tuner and profiler scripts touch exists."""
    for name in ("DEVICE", "attention", "_launch_kernel", "get_tiling", "get_tiling_source",
                 "_describe_runtime", "_get_persistent_programs", "_make_inputs",
                 "PROFILE_OP_NAME", "RESULT_DIR_NAME", "DEFAULT_TILING_PRESETS", "profiling",
                 "profile_once", "_validate_inputs", "_build_grid", "_resolve_tiling", "main"):
        assert hasattr(fam, name), name
    assert fam.DEVICE == "cuda"
    src = (REPO / "flash_attention_forward.py").read_text()
    assert src.count(tuner.PRESET_BEGIN) == 1 and src.count(tuner.PRESET_END) == 1


def test_validation_matches_reference_rules():
    q = torch.randn(1, 2, 8, 64)
    with pytest.raises(ValueError, match="4D"):
        fam.attention(q[0], q[0], q[0], False, 0.5)
    with pytest.raises(ValueError, match="same shape"):
        fam.attention(q, q[:, :1], q, False, 0.5)
    with pytest.raises(ValueError, match="HEAD_DIM"):
        x = torch.randn(1, 2, 8, 48)
        fam.attention(x, x, x, False, 0.5)
    with pytest.raises(ValueError, match="together"):
        fam._resolve_tiling(1, 2, 8, 64, False, bm=128)
    with pytest.raises(ValueError, match="CUDA"):
        fam.attention(q, q, q, False, 0.5)  # no CPU fallback: CPU tensors are rejected


def test_tiling_defaults_and_sources():
    assert fam.get_tiling(16, 16, 8192, 128, False) == (256, 128)
    assert fam.get_tiling(1, 1, 64, 64, True) == (128, 128)
    assert fam.get_tiling(1, 8, 2048, 256, False) == (128, 64)   # heuristic
    assert fam.get_tiling_source(16, 16, 8192, 128, False) == "fallback"
    # the tuned presets block drives the evaluator's performance shapes
    assert fam.get_tiling_source(128, 8, 2048, 256, False) == "preset"
    assert fam.get_tiling(128, 8, 2048, 256, False) == fam.DEFAULT_TILING_PRESETS[
        (128, 8, 2048, 256, False)][:2]
    rt = fam._describe_runtime(16, 16, 8192, 128, False)
    assert rt["selected_config"] == {"BLOCK_M": 256, "BLOCK_N": 128}
    assert rt["total_tiles"] == 32 * 256 and rt["stage"] == 1
    # cfg4 runs on the persistent kernel: a 4-deep K/V ring, one CTA per SM looping over tiles
    assert rt["pipeline"]["NUM_STAGES"] == 4
    assert rt["kernel"] == "persistent"
    assert rt["launched_programs"] == min(rt["total_tiles"], fam._sm_count())
    assert fam._build_grid(16, 16, 8192, 256) == (8192, 1, 1)
    # so does the same shape with a causal mask
    rtc = fam._describe_runtime(16, 16, 8192, 128, True)
    assert rtc["kernel"] == "persistent"
    assert rtc["launched_programs"] == min(rtc["total_tiles"], fam._sm_count())
    # head_dim 256 launches one CTA per tile
    rt256 = fam._describe_runtime(1, 8, 2048, 256, False)
    assert rt256["kernel"] == "one CTA per tile"
    assert rt256["launched_programs"] == rt256["total_tiles"]


def test_persistent_programs_env(monkeypatch):
    monkeypatch.setenv("PERSISTENT_PROGRAMS", "148")
    assert fam._get_persistent_programs() == 148
    # it sizes the persistent kernel's grid ...
    rt = fam._describe_runtime(4, 16, 4096, 128, True)
    assert rt["pipeline"]["PERSISTENT_CTAS"] == 148 and rt["launched_programs"] == 148
    monkeypatch.setenv("PERSISTENT_PROGRAMS", "20")
    assert fam._describe_runtime(4, 16, 4096, 64, False)["launched_programs"] == 20
    # ... and is refused, not silently dropped, where one CTA per tile is launched
    with pytest.raises(ValueError, match="PERSISTENT_PROGRAMS"):
        fam._describe_runtime(1, 8, 2048, 256, False)
    monkeypatch.setenv("PERSISTENT_PROGRAMS", "0")
    with pytest.raises(ValueError):
        fam._get_persistent_programs()


def test_tile_config_presets_roundtrip():
    assert tiling.TileConfig.from_preset((128, 64)) == tiling.TileConfig(128, 64)
    c = tiling.TileConfig.from_preset((256, 128, 4, 148))
    assert c.as_preset() == (256, 128, 4, 148)
    assert tiling.TileConfig.from_preset(c.as_dict()) == c
    with pytest.raises(ValueError):
        tiling.TileConfig.from_preset((1, 2, 3))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [16, 32, 64, 128, 256])
def test_candidates_fit_the_hardware(head_dim, dtype):
    cands = tiling.candidates(head_dim, dtype)
    assert cands
    for c in cands:
        g = tiling.geometry(head_dim, dtype, c)
        assert g["tmem_columns"] <= 512
        assert g["smem_fixed"] + c.num_stages * g["kv_tile_bytes"] <= tiling.SMEM_LIMIT
        assert 2 <= c.num_stages <= tiling.MAX_STAGES
    if head_dim == 256:
        assert all(c.block_m == 128 for c in cands)


# ---------------------------------------------------------------- tuner
def test_tuner_candidate_generation_matches_kernel_family():
    cands = tuner._generate_tiling_candidates((128, 8, 4096, 128, False), "float16")
    bms = {c["BLOCK_M"] for c in cands}
    assert bms == {128, 256}
    assert all(set(c) == {"BLOCK_M", "BLOCK_N", "NUM_STAGES", "PERSISTENT_CTAS"} for c in cands)
    short = tuner._generate_tiling_candidates((4, 4, 64, 64, True), "bfloat16")
    assert {c["BLOCK_M"] for c in short} == {128}
    key = tuner.ShapeKey.from_cli("128,8,1024,128,true")
    assert key.as_tuple() == (128, 8, 1024, 128, True)
    assert key.key() == "128:8:1024:128:1" and tuner.ShapeKey.from_key(key.key()) == key
    assert tuner.ShapeKey.from_record(key.record()) == key
    with pytest.raises(ValueError):
        tuner.ShapeKey.from_cli("1,2,3")
    with pytest.raises(ValueError):
        tuner.ShapeKey.from_cli("1,2,3,4,maybe")


def test_tuner_json_merge(tmp_path):
    out = tmp_path / "tuned.json"
    old = {"meta": {}, "tuned_configs": {"1:1:64:64:0": {"BLOCK_M": 128, "BLOCK_N": 64}},
           "results": [{"Z": 1, "H": 1, "N_CTX": 64, "HEAD_DIM": 64, "causal": False, "x": 1}]}
    out.write_text(json.dumps(old))
    new = {"meta": {"dtype": "float16"},
           "tuned_configs": {"2:2:128:64:1": {"BLOCK_M": 256, "BLOCK_N": 128, "NUM_STAGES": 4,
                                              "PERSISTENT_CTAS": 0}},
           "results": [{"Z": 2, "H": 2, "N_CTX": 128, "HEAD_DIM": 64, "causal": True, "x": 2}]}
    merged = tuner.merge_into_existing(out, new)
    assert set(merged["tuned_configs"]) == {"1:1:64:64:0", "2:2:128:64:1"}
    assert [r["x"] for r in merged["results"]] == [1, 2]
    # a re-tuned shape replaces its row in place
    again = {"tuned_configs": {"1:1:64:64:0": {"BLOCK_M": 256, "BLOCK_N": 128}},
             "results": [{"Z": 1, "H": 1, "N_CTX": 64, "HEAD_DIM": 64, "causal": False, "x": 3}]}
    merged2 = tuner.merge_tuned_payloads(merged, again)
    assert [r["x"] for r in merged2["results"]] == [3, 2]
    assert merged2["tuned_configs"]["1:1:64:64:0"]["BLOCK_M"] == 256
    assert tuner.merge_into_existing(tmp_path / "absent.json", new) is new


def test_presets_block_rewrite_roundtrip(tmp_path):
    mod_path = tmp_path / "flash_attention_forward.py"
    shutil.copy(REPO / "flash_attention_forward.py", mod_path)
    tuned = tmp_path / "tuned.json"
    tuned.write_text(json.dumps({"tuned_configs": {
        "16:16:8192:128:0": {"BLOCK_M": 256, "BLOCK_N": 128, "NUM_STAGES": 4,
                             "PERSISTENT_CTAS": 0},
        "128:8:1024:128:1": {"BLOCK_M": 128, "BLOCK_N": 64}}}))
    tuner.write_presets(mod_path, tuned)
    spec = importlib.util.spec_from_file_location("fa_rewritten", mod_path)
    m = importlib.util.module_from_spec(spec)
    sys.path.insert(0, str(REPO))
    spec.loader.exec_module(m)
    assert m.DEFAULT_TILING_PRESETS[(16, 16, 8192, 128, False)] == (256, 128, 4, 0)
    assert m.get_tiling(128, 8, 1024, 128, True) == (128, 64)
    assert m.get_tiling_source(128, 8, 1024, 128, True) == "preset"
    assert m.get_tile_config(16, 16, 8192, 128, False)["NUM_STAGES"] == 4
    # a second rewrite replaces the block instead of appending
    tuner.write_presets(mod_path, tuned)
    assert mod_path.read_text().count(tuner.PRESET_BEGIN) == 1


def test_reference_style_presets_are_accepted(tmp_path):
    """A block written by the reference tuner (2-tuples) still drives the module."""
    mod_path = tmp_path / "flash_attention_forward.py"
    src = (REPO / "flash_attention_forward.py").read_text()
    begin = src.index(tuner.PRESET_BEGIN)
    end = src.index(tuner.PRESET_END) + len(tuner.PRESET_END)
    block = (tuner.PRESET_BEGIN + "\nDEFAULT_TILING_PRESETS = {\n"
             "    (128, 8, 4096, 128, False): (128, 128),\n}\n" + tuner.PRESET_END)
    mod_path.write_text(src[:begin] + block + src[end:])
    spec = importlib.util.spec_from_file_location("fa_refstyle", mod_path)
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    assert m.get_tiling(128, 8, 4096, 128, False) == (128, 128)


# ---------------------------------------------------------------- torch_npu shim
@pytest.fixture()
def shim(monkeypatch):
    monkeypatch.syspath_prepend(str(SHIM))
    sys.modules.pop("torch_npu", None)
    import torch_npu
    yield torch_npu
    sys.modules.pop("torch_npu", None)


def test_shim_answers_vendor_op_like_the_fp32_reference(shim, monkeypatch):
    torch.manual_seed(0)
    q, k, v = (torch.randn(2, 3, 70, 32) for _ in range(3))
    mask = torch.triu(torch.ones(70, 70, dtype=torch.bool), diagonal=1)
    monkeypatch.setenv("FA_SHIM_BASELINE", "sdpa")
    out = shim.npu_fusion_attention(q, k, v, 3, atten_mask=mask, scale=0.5, keep_prob=1.0,
                                    input_layout="BNSD", pre_tockens=70, next_tockens=0)[0]
    ref = attention_ref_torch(q, k, v, True, 0.5)[0]
    assert (out - ref).abs().max().item() < 1e-5
    out_nc = shim.npu_fusion_attention(q, k, v, 3, scale=0.5, input_layout="BNSD")[0]
    assert (out_nc - attention_ref_torch(q, k, v, False, 0.5)[0]).abs().max().item() < 1e-5
    assert hasattr(torch.npu, "synchronize") and hasattr(torch.npu, "empty_cache")


def test_shim_raise_mode_and_unsupported_layout(shim, monkeypatch):
    q = torch.randn(1, 1, 8, 16)
    monkeypatch.setenv("FA_SHIM_BASELINE", "raise")
    with pytest.raises(RuntimeError):
        shim.npu_fusion_attention(q, q, q, 1, scale=1.0, input_layout="BNSD")
    monkeypatch.setenv("FA_SHIM_BASELINE", "sdpa")
    with pytest.raises(RuntimeError):
        shim.npu_fusion_attention(q, q, q, 1, scale=1.0, input_layout="BSH")


@pytest.mark.skipif(not (REFERENCE / "evaluate_attention.py").exists(),
                    reason="reference checkout not present")
def test_reference_evaluator_runs_through_the_shim(shim, monkeypatch):
    """The unchanged reference evaluator imports through the shim; its vendor-op path and its
    fp32 fallback agree (evaluate_attention.py:104-156)."""
    spec = importlib.util.spec_from_file_location("ref_eval", REFERENCE / "evaluate_attention.py")
    ev = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ev)
    q, k, v = ev._make_inputs("cpu", torch.float32, 1, 2, 64, 64, 0)
    monkeypatch.setenv("FA_SHIM_BASELINE", "sdpa")
    base = ev._reference_attention(None, q, k, v, 2, True, 0.5)
    monkeypatch.setenv("FA_SHIM_BASELINE", "raise")
    fallback = ev._reference_attention(None, q, k, v, 2, True, 0.5)
    assert (base - fallback).abs().max().item() < 1e-5
    assert tuple(ev.PERFORMANCE_CASES) == tuple(tuner.DEFAULT_SHAPES)


def test_validate_inputs_fp8_v_rules():
    """A float8_e5m2 v is accepted with 16-bit q/k (the reference's fp8_v mode); the CPU tensors
    then fail only the device rule.  fp32 q/k or head_dim < 32 with an fp8 v are refused."""
    from flash_attn_npu_b200 import ops
    q = torch.zeros(1, 1, 8, 64, dtype=torch.bfloat16)
    v8 = torch.zeros(1, 1, 8, 64).to(torch.float8_e5m2)
    with pytest.raises(ValueError, match="CUDA"):
        ops.validate_inputs(q, q, v8)
    with pytest.raises(ValueError, match="same dtype"):
        ops.validate_inputs(q.float(), q.float(), v8)
    q16 = torch.zeros(1, 1, 8, 16, dtype=torch.float16)
    with pytest.raises(ValueError, match="HEAD_DIM >= 32"):
        ops.validate_inputs(q16, q16, torch.zeros(1, 1, 8, 16).to(torch.float8_e5m2))
    assert ops.is_v_fp8(q, v8) and not ops.is_v_fp8(q.float(), v8)


def test_ncu_raw_csv_parser_and_groups():
    """`ncu --csv --page raw` output (header, units, one row per launch) -> metric groups."""
    from flash_attn_npu_b200 import ncu_profile
    text = ('==PROF== Connected to process\n'
            '"ID","Kernel Name","gpu__time_duration.sum","dram__bytes_read.sum","launch__grid_size"\n'
            '"","","nsecond","byte",""\n'
            '"0","fa_fwd_sm100_kernel","1,234","5,000,000","148"\n')
    rows = ncu_profile.parse_raw_csv(text)
    assert rows[0]["gpu__time_duration.sum"] == 1234.0
    assert rows[0]["dram__bytes_read.sum"] == 5e6
    g = ncu_profile.group_summary(rows[0], {"Timing": ["gpu__time_duration.sum"],
                                            "Memory": ["dram__bytes_read.sum", "missing"]})
    assert g == {"Timing": {"gpu__time_duration.sum": 1234.0},
                 "Memory": {"dram__bytes_read.sum": 5e6}}
    assert ncu_profile.parse_raw_csv("no csv here") == []
    # above the size cap a capture asks for the launch duration alone (one pass)
    big = ncu_profile.groups_for_input_bytes(ncu_profile.MAX_MULTIPASS_BYTES + 1)
    assert big == {"Timing": ["gpu__time_duration.sum"]}
    assert ncu_profile.groups_for_input_bytes(1 << 20) == ncu_profile.METRIC_GROUPS
