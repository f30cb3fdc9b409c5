"""`torch.ops.flash_attn_b200.fwd`: fake implementation on the CPU (meta / FakeTensorMode),
and on the GPU bit-equality with `ops.forward`, the operator checks and CUDA-graph replay."""
from __future__ import annotations

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from flash_attn_npu_b200 import ops, torch_op  # noqa: F401  (registers the operator)

FWD = torch.ops.flash_attn_b200.fwd


# ----------------------------------------------------------------------------- CPU
@pytest.mark.parametrize("shape,dtype", [((2, 3, 100, 64), torch.bfloat16),
                                         ((1, 1, 7, 256), torch.float16),
                                         ((2, 2, 33, 32), torch.float32)])
def test_fake_shapes_on_meta(shape, dtype):
    q = torch.empty(shape, dtype=dtype, device="meta")
    out, lse = FWD(q, q, q, True, 0.1, 0, 0, 0, 0)
    assert out.shape == q.shape and out.dtype == dtype and out.stride() == q.stride()
    assert lse.shape == shape[:3] and lse.dtype == torch.float32 and lse.is_contiguous()


def test_fake_keeps_bshd_layout_and_fixes_unaligned():
    q = torch.empty(2, 100, 3, 64, dtype=torch.float16, device="meta").transpose(1, 2)
    out, _ = FWD(q, q, q, False, 0.125)
    assert out.stride() == q.stride()
    # a 65-element row stride (130 bytes) cannot be a TMA stride: the output is contiguous
    base = torch.empty(1, 2, 40, 65, dtype=torch.float16, device="meta")[..., :64]
    out, _ = FWD(base, base, base, False, 0.125)
    assert out.is_contiguous()


def test_fake_validates_and_runs_under_fake_mode():
    with FakeTensorMode():
        q = torch.empty(1, 2, 64, 32, dtype=torch.float16)
        out, lse = FWD(q, q, q, False, 0.1)
        assert out.shape == q.shape and lse.shape == (1, 2, 64)
    bad = torch.empty(1, 2, 64, 48, dtype=torch.float16, device="meta")
    with pytest.raises(ValueError):
        FWD(bad, bad, bad, False, 0.1)
    v8 = torch.empty(1, 2, 64, 64, dtype=torch.float8_e5m2, device="meta")
    q = torch.empty(1, 2, 64, 64, dtype=torch.bfloat16, device="meta")
    out, _ = FWD(q, q, v8, False, 0.1)
    assert out.dtype == torch.bfloat16


# ----------------------------------------------------------------------------- GPU
def _inputs(shape, dtype, dev, seed=0):
    g = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(shape, generator=g).to(dtype).to(dev) for _ in range(3))


@pytest.mark.gpu
@pytest.mark.parametrize("causal", [False, True])
def test_op_bit_equal_to_ops_forward(causal, cuda_device):
    q, k, v = _inputs((2, 4, 700, 128), torch.bfloat16, cuda_device)
    ref_o, ref_l = ops.forward(q, k, v, causal, 0.09)
    out, lse = FWD(q, k, v, causal, 0.09, 0, 0, 0, 0)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_o) and torch.equal(lse, ref_l)


@pytest.mark.gpu
def test_opcheck_schema_and_fake(cuda_device):
    q, k, v = _inputs((1, 2, 256, 64), torch.float16, cuda_device)
    torch.library.opcheck(FWD, (q, k, v, True, 0.125, 0, 0, 0, 0),
                          test_utils=("test_schema", "test_faketensor"))


@pytest.mark.gpu
def test_cuda_graph_replay(cuda_device):
    """Captured once, replayed on new inputs written into the captured buffers."""
    q, k, v = _inputs((2, 3, 512, 128), torch.bfloat16, cuda_device, seed=1)
    s = torch.cuda.Stream(cuda_device)
    s.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(s):
        for _ in range(2):
            FWD(q, k, v, False, 0.1, 0, 0, 0, 0)
    torch.cuda.current_stream(cuda_device).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        g_out, g_lse = FWD(q, k, v, False, 0.1, 0, 0, 0, 0)
    for seed in (2, 3):
        nq, nk, nv = _inputs((2, 3, 512, 128), torch.bfloat16, cuda_device, seed=seed)
        q.copy_(nq), k.copy_(nk), v.copy_(nv)
        graph.replay()
        ref_o, ref_l = ops.forward(nq, nk, nv, False, 0.1)
        torch.cuda.synchronize()
        assert torch.equal(g_out, ref_o) and torch.equal(g_lse, ref_l)
    del graph
