"""Build the sm_100a shared library `libfa_sm100.so` in-tree with nvcc.

The library is a plain C-ABI shared object (see include/fa_fwd_sm100.h); it has no PyTorch
dependency, so it is compiled directly with nvcc rather than through torch's extension
machinery.  The five head-dimension translation units compile in parallel.

Usage:  python -m flash_attn_npu_b200.build [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = REPO_DIR / "_build" / "fa_sm100"
LIB_NAME = "libfa_sm100.so"
LIB_PATH = PKG_DIR / LIB_NAME

# Test builds of the same sources.  "shortwait": every pipeline wait gives up as soon as its
# first non-suspending probe finds the phase incomplete (FA_WAIT_TIMEOUT_NS = 0, no spin
# polls), while the teardown drains keep their long limit -- the library the bounded-wait test
# launches to see the timeout status come back.
VARIANTS = {
    "shortwait": ["-DFA_WAIT_TIMEOUT_NS=0ull", "-DFA_WAIT_SPIN_POLLS=0",
                  "-DFA_WAIT_POLL_NONBLOCKING"],
}


def variant_path(variant: str) -> Path:
    return PKG_DIR / f"libfa_sm100_{variant}.so"

SOURCES = [
    "fa_fwd_api.cu",
    "fa_fwd_fp32.cu",
    "fa_fwd_d16.cu",
    "fa_fwd_d32.cu",
    "fa_fwd_d64.cu",
    "fa_fwd_d128.cu",
    "fa_fwd_d256.cu",
]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the sm_100a library cannot be built")
    return cand


def _inputs_digest(extra_flags: list[str]) -> str:
    h = hashlib.sha256()
    for p in sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
                    + list(INCLUDE.glob("*.h"))):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(ARCH_FLAGS + COMMON_FLAGS + extra_flags).encode())
    return h.hexdigest()


def _stamp_path(lib_path: Path = LIB_PATH) -> Path:
    return lib_path.with_name(lib_path.name + ".sha256")


def is_up_to_date(extra_flags: list[str] | None = None, lib_path: Path = LIB_PATH) -> bool:
    stamp = _stamp_path(lib_path)
    return lib_path.exists() and stamp.exists() and stamp.read_text().strip() == _inputs_digest(
        extra_flags or [])


def _compile_one(nvcc: str, src: str, extra: list[str], verbose: bool,
                 build_dir: Path = BUILD_DIR) -> Path:
    obj = build_dir / (Path(src).stem + ".o")
    cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, *extra, "-I", str(INCLUDE), "-c", str(CSRC / src),
           "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr)
    return obj


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None,
          variant: str | None = None) -> Path:
    """Compile every CUDA source for sm_100a and link `libfa_sm100.so` next to this file
    (or, with `variant`, the test library `libfa_sm100_<variant>.so`)."""
    extra = list(extra_flags or [])
    lib_path, build_dir = LIB_PATH, BUILD_DIR
    if variant is not None:
        extra = VARIANTS[variant] + extra
        lib_path = variant_path(variant)
        build_dir = BUILD_DIR.with_name(f"fa_sm100_{variant}")
    if not force and is_up_to_date(extra, lib_path):
        return lib_path
    nvcc = nvcc_path()
    build_dir.mkdir(parents=True, exist_ok=True)
    workers = min(len(SOURCES), max(1, os.cpu_count() or 1))
    with cf.ThreadPoolExecutor(max_workers=workers) as ex:
        objs = list(ex.map(lambda s: _compile_one(nvcc, s, extra, verbose, build_dir), SOURCES))
    tmp = lib_path.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *[str(o) for o in objs]]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, lib_path)
    _stamp_path(lib_path).write_text(_inputs_digest(extra) + "\n")
    return lib_path


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill report")
    ap.add_argument("--variant", choices=sorted(VARIANTS), default=None,
                    help="build a test variant of the library instead of the product")
    args = ap.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose, variant=args.variant)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
