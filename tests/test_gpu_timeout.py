"""The kernel's bounded waits, exercised the allowed way: no fault, no hang, no barrier taken out.

The test library `libfa_sm100_shortwait.so` is the product source built with a pipeline-wait
limit of zero (`python -m flash_attn_npu_b200.build --variant shortwait`): any mbarrier wait
that is not satisfied after its first polls gives up, records FA_ERR_DEVICE_TIMEOUT in the
status word and raises the CTA's abort flag; every role then drains its own in-flight TMA
loads and MMAs (that limit stays long) and the CTA exits.  On a launch of 1024 query blocks
some wait is certain to give up.  Both kernels are exercised: the persistent one (grid = one CTA
per SM, each looping over tiles) and the one-CTA-per-tile one.  The child process checks that

  - the launch returns and the stream synchronizes (nothing hangs),
  - the status word reads FA_ERR_DEVICE_TIMEOUT,
  - the CUDA context is still usable: a launch of the product library in the same process
    right after it matches the oracle.
"""
from __future__ import annotations

import ctypes
import json
import os
import subprocess
import sys

import pytest
import torch

from conftest import REPO

pytestmark = pytest.mark.gpu


def _child_main(kernel: str, head_dim: int) -> None:
    from flash_attn_npu_b200 import _native, build, ops
    from oracle.attention_ref import attention_ref_torch

    lib = ctypes.CDLL(str(build.variant_path("shortwait")))
    lib.fa_fwd_sm100.argtypes = [ctypes.POINTER(_native.FaFwdArgs), ctypes.c_void_p]
    lib.fa_fwd_sm100.restype = ctypes.c_int
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(11)
    B, H, S, D = 4, 16, 4096, head_dim
    q, k, v = (torch.randn((B, H, S, D), generator=g).to(torch.bfloat16).to(dev)
               for _ in range(3))
    out = torch.empty_like(q)
    lse = torch.empty((B, H, S), device=dev, dtype=torch.float32)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    st = (H * S * D, S * D, D)
    args = _native.make_args(q_ptr=q.data_ptr(), k_ptr=k.data_ptr(), v_ptr=v.data_ptr(),
                             o_ptr=out.data_ptr(), lse_ptr=lse.data_ptr(), batch=B, heads=H,
                             seqlen=S, head_dim=D, q_stride=st, k_stride=st, v_stride=st,
                             o_stride=st, dtype_code=_native.FA_DTYPE_BF16, causal=False,
                             sm_scale=D ** -0.5, status_ptr=status.data_ptr(),
                             block_m=256, block_n=128,
                             persistent_ctas=(torch.cuda.get_device_properties(dev)
                                              .multi_processor_count
                                              if kernel == "persistent" else 0),
                             flags=(_native.FA_FLAG_ONE_CTA_PER_TILE
                                    if kernel == "one_cta_per_tile" else 0))
    rc = lib.fa_fwd_sm100(ctypes.byref(args),
                          ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    torch.cuda.synchronize(dev)
    timed_out = int(status.item())
    # the context is still usable: the product library on a fresh problem
    qs, ks, vs = (t[:1, :2, :700].contiguous() for t in (q, k, v))
    o2, l2 = ops.forward(qs, ks, vs, True, D ** -0.5)
    ro, rl = attention_ref_torch(qs.cpu(), ks.cpu(), vs.cpu(), True, D ** -0.5)
    torch.cuda.synchronize(dev)
    print("RESULT " + json.dumps({
        "rc": rc, "status": timed_out,
        "after_max_abs": (o2.float().cpu() - ro).abs().max().item(),
        "after_mean_abs": (o2.float().cpu() - ro).abs().mean().item(),
        "after_lse_abs": (l2.cpu() - rl).abs().max().item()}), flush=True)


# head_dim 64 runs the persistent kernel's separate-P protocol (S read -> next S, P V -> next P
# store), head_dim 128 the one with P over S
@pytest.mark.parametrize("kernel,head_dim", [("persistent", 128), ("persistent", 64),
                                             ("one_cta_per_tile", 128)])
def test_pipeline_wait_timeout_reports_status_and_context_survives(kernel, head_dim, native_lib,
                                                                    cuda_device):
    from flash_attn_npu_b200 import _native, build
    build.build(variant="shortwait")  # no-op when up to date
    res = subprocess.run([sys.executable, __file__, "child", kernel, str(head_dim)],
                         cwd=str(REPO),
                         env=dict(os.environ), capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr[-3000:]
    line = [ln for ln in res.stdout.splitlines() if ln.startswith("RESULT ")][-1]
    r = json.loads(line[len("RESULT "):])
    assert r["rc"] == _native.FA_OK
    assert r["status"] == _native.FA_ERR_DEVICE_TIMEOUT
    assert r["after_max_abs"] <= 2e-2 and r["after_mean_abs"] <= 2e-3
    assert r["after_lse_abs"] <= 1e-4


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "child":
        sys.path.insert(0, str(REPO))
        _child_main(sys.argv[2], int(sys.argv[3]))
