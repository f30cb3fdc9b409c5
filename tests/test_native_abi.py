"""The C-ABI library loads, exports every symbol include/*.h declares, and answers its host-only
queries consistently with the Python tile model -- all without a GPU."""
from __future__ import annotations

import ctypes
import re
import subprocess

import pytest
import torch

from conftest import REPO
from flash_attn_npu_b200 import _native, tiling

HEADERS = sorted((REPO / "include").glob("*.h"))


def _declared_functions():
    names = set()
    for h in HEADERS:
        text = h.read_text()
        for m in re.finditer(r"FA_API\s+[\w\s\*]+?\b(fa_\w+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_header_declares_expected_entry_points():
    names = _declared_functions()
    assert "fa_fwd_sm100" in names
    assert set(_native.EXPORTED_SYMBOLS) <= names


def test_library_exports_every_declared_symbol(native_lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(_native.library_path())],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = _declared_functions() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    for name in _declared_functions():
        assert hasattr(native_lib, name)


def test_version_and_status_strings(native_lib):
    assert _native.load().fa_fwd_sm100_version() >= 1000
    for code in range(0, -10, -1):
        s = _native.status_string(code)
        assert s and s != "unknown status"
    assert _native.status_string(-99) == "unknown status"


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("head_dim", [16, 32, 64, 128, 256])
def test_stage_limits_match_python_model(native_lib, dtype, head_dim):
    code = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}[dtype]
    for bm in (128, 256):
        for bn in (64, 128):
            cfg = tiling.TileConfig(bm, bn)
            py = tiling.max_stages(head_dim, dtype, cfg)
            c = _native.max_stages(head_dim, code, bm, bn)
            assert py == c, (head_dim, dtype, bm, bn, py, c)
            assert _native.supported(head_dim, code, bm, bn) == (py >= 2)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("head_dim", [16, 32, 64, 128])
@pytest.mark.parametrize("seqlen", [64, 8192])
def test_default_tile_matches_python_heuristic(native_lib, dtype, head_dim, seqlen):
    code = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}[dtype]
    if dtype == torch.float32 and head_dim < 32:
        # tf32 MN-major V needs 128-byte rows: fp32 at head_dim 16 has no kernel
        with pytest.raises(_native.NativeError):
            _native.default_tile(head_dim, code, False, seqlen)
        assert not tiling.is_supported(head_dim, dtype, tiling.heuristic(seqlen, head_dim, False, dtype))
        return
    cfg = _native.default_tile(head_dim, code, False, seqlen)
    h = tiling.heuristic(seqlen, head_dim, False, dtype)
    assert (cfg.block_m, cfg.block_n) == (h.block_m, h.block_n)
    assert tiling.is_supported(head_dim, dtype, h)


def test_unsupported_head_dim_rejected(native_lib):
    with pytest.raises(_native.NativeError) as ei:
        _native.default_tile(48, 1, False, 128)
    assert ei.value.code == _native.FA_ERR_UNSUPPORTED_HEAD_DIM
    assert not _native.supported(48, 1, 128, 128)


def _args(**kw):
    base = dict(q_ptr=256, k_ptr=256, v_ptr=256, o_ptr=256, lse_ptr=256, batch=2, heads=3,
                seqlen=100, head_dim=64, q_stride=(3 * 100 * 64, 100 * 64, 64),
                k_stride=(3 * 100 * 64, 100 * 64, 64), v_stride=(3 * 100 * 64, 100 * 64, 64),
                o_stride=(3 * 100 * 64, 100 * 64, 64), dtype_code=1, causal=False,
                sm_scale=0.125)
    base.update(kw)
    return _native.make_args(**base)


def test_struct_size_is_checked(native_lib):
    a = _args()
    lib = _native.load()
    a.struct_size = ctypes.sizeof(_native.FaFwdArgs) - 8
    assert lib.fa_fwd_sm100(ctypes.byref(a), None) == _native.FA_ERR_INVALID_ARG
    a.struct_size = ctypes.sizeof(_native.FaFwdArgs)
    # with the right size the host checks pass and the call stops at the device check
    rc = lib.fa_fwd_sm100(ctypes.byref(a), None)
    if torch.cuda.is_available():
        pytest.skip("device present; host-only path not exercised")
    assert rc == _native.FA_ERR_DEVICE


def test_host_validation_codes(native_lib):
    lib = _native.load()
    cases = [
        (_args(head_dim=48), _native.FA_ERR_UNSUPPORTED_HEAD_DIM),
        (_args(dtype_code=7), _native.FA_ERR_UNSUPPORTED_DTYPE),
        (_args(seqlen=0), _native.FA_ERR_INVALID_ARG),
        (_args(q_ptr=None), _native.FA_ERR_INVALID_ARG),
        (_args(sm_scale=float("nan")), _native.FA_ERR_INVALID_ARG),
    ]
    for a, want in cases:
        assert lib.fa_fwd_sm100(ctypes.byref(a), None) == want


def test_grid_size(native_lib):
    # non-causal default tile for D=64 bf16, S=100: BLOCK_M=128 (S <= 128) -> 1 q-block x 6
    assert _native.grid_size(_args()) == 6
    assert _native.grid_size(_args(seqlen=1000)) == 4 * 6  # BLOCK_M=256
    a = _args(seqlen=1000, block_m=128, block_n=64)
    assert _native.grid_size(a) == 8 * 6
    assert _native.grid_size(_args(head_dim=40)) == -1


def test_fp8_v_flag_validation(native_lib):
    """FA_FLAG_V_FP8_E5M2: 16-bit q/k only, head_dim >= 32; unknown flag bits are rejected."""
    lib = _native.load()
    fl = _native.FA_FLAG_V_FP8_E5M2
    cases = [
        (_args(dtype_code=2, flags=fl), _native.FA_ERR_UNSUPPORTED_DTYPE),
        (_args(head_dim=16, q_stride=(3 * 100 * 16, 100 * 16, 16),
               k_stride=(3 * 100 * 16, 100 * 16, 16), v_stride=(3 * 100 * 16, 100 * 16, 16),
               o_stride=(3 * 100 * 16, 100 * 16, 16), flags=fl), _native.FA_ERR_UNSUPPORTED_HEAD_DIM),
        (_args(flags=8), _native.FA_ERR_INVALID_ARG),
    ]
    for a, want in cases:
        assert lib.fa_fwd_sm100(ctypes.byref(a), None) == want
    # the default tile exists for every fp8-V head dim and both 16-bit types
    for d in (32, 64, 128, 256):
        for code in (0, 1):
            a = _args(head_dim=d, dtype_code=code, flags=fl, q_stride=(3 * 100 * d, 100 * d, d),
                      k_stride=(3 * 100 * d, 100 * d, d), v_stride=(3 * 100 * d, 100 * d, d),
                      o_stride=(3 * 100 * d, 100 * d, d))
            assert _native.grid_size(a) > 0, (d, code)
    # tiles outside the fp8-V set are refused before any launch
    a = _args(flags=fl, seqlen=1000, block_m=256, block_n=64)
    assert _native.grid_size(a) == -1
