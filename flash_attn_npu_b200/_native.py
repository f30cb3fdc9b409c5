"""ctypes binding to the sm_100a C-ABI library `libfa_sm100.so` (include/fa_fwd_sm100.h).

Only plain pointers, sizes and a stream handle cross this boundary; PyTorch is used by the
callers for device memory and the current stream.  If the library is missing the functions
here raise immediately -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("FA_SM100_LIB", PKG_DIR / "libfa_sm100.so"))

FA_DTYPE_FP16 = 0
FA_DTYPE_BF16 = 1
FA_DTYPE_FP32 = 2

FA_FLAG_FP32_TF32 = 1
FA_FLAG_V_FP8_E5M2 = 2
FA_FLAG_ONE_CTA_PER_TILE = 4

FA_OK = 0
FA_ERR_INVALID_ARG = -1
FA_ERR_UNSUPPORTED_HEAD_DIM = -2
FA_ERR_UNSUPPORTED_DTYPE = -3
FA_ERR_MISALIGNED = -4
FA_ERR_UNSUPPORTED_TILE = -5
FA_ERR_TENSOR_MAP = -6
FA_ERR_LAUNCH = -7
FA_ERR_DEVICE = -8
FA_ERR_DEVICE_TIMEOUT = -9

# Every symbol include/fa_fwd_sm100.h declares (checked by the tests).
EXPORTED_SYMBOLS = (
    "fa_fwd_sm100",
    "fa_fwd_sm100_default_tile",
    "fa_fwd_sm100_supported",
    "fa_fwd_sm100_max_stages",
    "fa_fwd_sm100_grid_size",
    "fa_fwd_sm100_status_string",
    "fa_fwd_sm100_version",
)


class FaTileConfig(ctypes.Structure):
    _fields_ = [
        ("block_m", ctypes.c_int32),
        ("block_n", ctypes.c_int32),
        ("num_stages", ctypes.c_int32),
        ("persistent_ctas", ctypes.c_int32),
    ]


class FaFwdArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_int32),
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("lse", ctypes.c_void_p),
        ("batch", ctypes.c_int64),
        ("heads", ctypes.c_int64),
        ("seqlen", ctypes.c_int64),
        ("head_dim", ctypes.c_int64),
        ("q_stride", ctypes.c_int64 * 3),
        ("k_stride", ctypes.c_int64 * 3),
        ("v_stride", ctypes.c_int64 * 3),
        ("o_stride", ctypes.c_int64 * 3),
        ("dtype", ctypes.c_int32),
        ("causal", ctypes.c_int32),
        ("sm_scale", ctypes.c_float),
        ("tile", FaTileConfig),
        ("dev_status", ctypes.c_void_p),
        ("flags", ctypes.c_int32),
    ]


class NativeError(RuntimeError):
    """Raised for a non-zero status from the C ABI."""

    def __init__(self, code: int, message: str):
        super().__init__(f"fa_fwd_sm100 error {code}: {message}")
        self.code = code


_lib = None
_lock = threading.Lock()


def library_path() -> Path:
    return LIB_PATH


def load() -> ctypes.CDLL:
    """Load (once) and return the native library; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"sm_100a library not found at {LIB_PATH}; build it with "
                "`python -m flash_attn_npu_b200.build` (no CPU fallback exists)")
        lib = ctypes.CDLL(str(LIB_PATH))
        lib.fa_fwd_sm100.argtypes = [ctypes.POINTER(FaFwdArgs), ctypes.c_void_p]
        lib.fa_fwd_sm100.restype = ctypes.c_int
        lib.fa_fwd_sm100_default_tile.argtypes = [
            ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64,
            ctypes.POINTER(FaTileConfig)]
        lib.fa_fwd_sm100_default_tile.restype = ctypes.c_int
        lib.fa_fwd_sm100_supported.argtypes = [
            ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]
        lib.fa_fwd_sm100_supported.restype = ctypes.c_int
        lib.fa_fwd_sm100_max_stages.argtypes = [
            ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]
        lib.fa_fwd_sm100_max_stages.restype = ctypes.c_int
        lib.fa_fwd_sm100_grid_size.argtypes = [ctypes.POINTER(FaFwdArgs)]
        lib.fa_fwd_sm100_grid_size.restype = ctypes.c_int64
        lib.fa_fwd_sm100_status_string.argtypes = [ctypes.c_int]
        lib.fa_fwd_sm100_status_string.restype = ctypes.c_char_p
        lib.fa_fwd_sm100_version.argtypes = []
        lib.fa_fwd_sm100_version.restype = ctypes.c_int
        _lib = lib
        return lib


def status_string(code: int) -> str:
    return load().fa_fwd_sm100_status_string(int(code)).decode()


def default_tile(head_dim: int, dtype_code: int, causal: bool, seqlen: int) -> FaTileConfig:
    cfg = FaTileConfig()
    rc = load().fa_fwd_sm100_default_tile(int(head_dim), int(dtype_code), int(bool(causal)),
                                          int(seqlen), ctypes.byref(cfg))
    if rc != FA_OK:
        raise NativeError(rc, status_string(rc))
    return cfg


def supported(head_dim: int, dtype_code: int, block_m: int, block_n: int,
              num_stages: int = 0) -> bool:
    return bool(load().fa_fwd_sm100_supported(int(head_dim), int(dtype_code), int(block_m),
                                              int(block_n), int(num_stages)))


def max_stages(head_dim: int, dtype_code: int, block_m: int, block_n: int) -> int:
    return int(load().fa_fwd_sm100_max_stages(int(head_dim), int(dtype_code), int(block_m),
                                              int(block_n)))


def make_args(*, q_ptr, k_ptr, v_ptr, o_ptr, lse_ptr, batch, heads, seqlen, head_dim,
              q_stride, k_stride, v_stride, o_stride, dtype_code, causal, sm_scale,
              block_m=0, block_n=0, num_stages=0, persistent_ctas=0,
              status_ptr=None, flags=0) -> FaFwdArgs:
    a = FaFwdArgs()
    a.struct_size = ctypes.sizeof(FaFwdArgs)
    a.q, a.k, a.v, a.o, a.lse = q_ptr, k_ptr, v_ptr, o_ptr, lse_ptr
    a.batch, a.heads, a.seqlen, a.head_dim = int(batch), int(heads), int(seqlen), int(head_dim)
    for name, st in (("q_stride", q_stride), ("k_stride", k_stride), ("v_stride", v_stride),
                     ("o_stride", o_stride)):
        arr = getattr(a, name)
        for i in range(3):
            arr[i] = int(st[i])
    a.dtype = int(dtype_code)
    a.causal = int(bool(causal))
    a.sm_scale = float(sm_scale)
    a.tile = FaTileConfig(int(block_m), int(block_n), int(num_stages), int(persistent_ctas))
    a.dev_status = status_ptr
    a.flags = int(flags)
    return a


def grid_size(args: FaFwdArgs) -> int:
    return int(load().fa_fwd_sm100_grid_size(ctypes.byref(args)))


def launch(args: FaFwdArgs, stream_handle: int) -> None:
    """Enqueue the forward pass on `stream_handle` (a cudaStream_t as int)."""
    rc = load().fa_fwd_sm100(ctypes.byref(args), ctypes.c_void_p(stream_handle))
    if rc != FA_OK:
        raise NativeError(rc, status_string(rc))
