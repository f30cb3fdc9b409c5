"""Host-buffer path (`flash_attn_npu_b200.host_stream`): chunk planning and argument checks
on the CPU, and bit-equality with the device-resident launch on the GPU."""
from __future__ import annotations

import pytest
import torch

import flash_attention_forward as faf
from flash_attn_npu_b200 import host_stream, ops


# ----------------------------------------------------------------------------- CPU
@pytest.mark.parametrize("n,slice_bytes,target,cs", [
    (256, 6 << 20, 96 << 20, None), (7, 1000, 3000, None), (5, 10, 10 ** 9, None),
    (10, 1 << 30, 96 << 20, None), (13, 1, 1, 4), (1, 5, 5, 3)])
def test_plan_chunks_cover_every_slice_once(n, slice_bytes, target, cs):
    chunks = host_stream.plan_chunks(n, slice_bytes, target, chunk_slices=cs)
    covered = [s for a, b in chunks for s in range(a, b)]
    assert covered == list(range(n))
    sizes = [b - a for a, b in chunks]
    assert all(x > 0 for x in sizes)
    assert all(x >= y for x, y in zip(sizes, sizes[1:]))  # never grows: the tail is split finer
    full = min(n, max(1, target // slice_bytes)) if cs is None else min(n, cs)
    assert sizes[0] == full
    n_full = -(-n // full)
    if n_full > 1:  # the last uniform chunk became at most 4 pieces
        assert all(x == full for x in sizes[:n_full - 1])
        assert 1 <= len(sizes) - (n_full - 1) <= 4
    else:
        assert sizes == [n]


def test_plan_chunks_edges():
    assert host_stream.plan_chunks(0, 100) == []
    chunks = host_stream.plan_chunks(256, 6 << 20)  # 16-slice chunks, the last one in four
    assert chunks[-5:] == [(224, 240), (240, 244), (244, 248), (248, 252), (252, 256)]
    assert host_stream.plan_chunks(10, 1, 4, tail_split=1) == [(0, 4), (4, 8), (8, 10)]
    with pytest.raises(ValueError):
        host_stream.plan_chunks(4, 100, chunk_slices=0)


def _host(shape=(1, 2, 64, 64), dtype=torch.float16):
    return tuple(torch.randn(shape).to(dtype) for _ in range(3))


def test_forward_host_argument_checks():
    q, k, v = _host()
    with pytest.raises(ValueError):
        host_stream.forward_host(q, k, v[:, :, :32], False, 0.125, device="cuda:0")
    with pytest.raises(ValueError):
        host_stream.forward_host(q[0], k[0], v[0], False, 0.125, device="cuda:0")
    with pytest.raises(ValueError):
        host_stream.forward_host(q, k, v.float(), False, 0.125, device="cuda:0")
    with pytest.raises(ValueError):
        host_stream.forward_host(q, k, v, False, 0.125, device="cpu")
    with pytest.raises(ValueError):  # out of the wrong shape
        host_stream.forward_host(q, k, v, False, 0.125, device="cuda:0",
                                 out=torch.empty(1, 2, 64, 32, dtype=q.dtype))
    with pytest.raises(ValueError):  # lse of the wrong dtype
        host_stream.forward_host(q, k, v, False, 0.125, device="cuda:0",
                                 out=torch.empty_like(q),
                                 lse=torch.empty(1, 2, 64, dtype=torch.float16))
    with pytest.raises(ValueError):  # head dim the kernels do not build
        q2, k2, v2 = _host((1, 1, 8, 48))
        faf.attention_host(q2, k2, v2, False, 0.125, device="cuda:0")


# ----------------------------------------------------------------------------- GPU
def _device_run(q, k, v, causal, scale, dev, bm=None, bn=None):
    qd, kd, vd = (t.to(dev) for t in (q, k, v))
    o, l = faf._launch_kernel(qd, kd, vd, causal, scale, bm=bm, bn=bn)
    torch.cuda.synchronize(dev)
    return o.cpu(), l.cpu()


@pytest.mark.gpu
@pytest.mark.parametrize("shape,dtype,causal,chunk", [
    ((2, 3, 300, 64), torch.float16, True, 1),
    ((2, 3, 300, 64), torch.float16, True, 4),
    ((2, 3, 300, 64), torch.float16, False, None),
    ((3, 5, 1024, 128), torch.bfloat16, False, 2),
    ((1, 4, 777, 256), torch.bfloat16, True, 3),
    ((2, 2, 512, 32), torch.float32, False, 3),
], ids=str)
def test_forward_host_bit_equal_to_device_launch(shape, dtype, causal, chunk, cuda_device):
    g = torch.Generator().manual_seed(17)
    q, k, v = (torch.randn(shape, generator=g).to(dtype).pin_memory() for _ in range(3))
    scale = shape[-1] ** -0.5
    ref_o, ref_l = _device_run(q, k, v, causal, scale, cuda_device)
    o, l = host_stream.forward_host(q, k, v, causal, scale, device=cuda_device,
                                    chunk_slices=chunk)
    assert o.device.type == "cpu" and l.device.type == "cpu"
    assert torch.equal(o, ref_o)
    assert torch.equal(l, ref_l)


@pytest.mark.gpu
def test_attention_host_module_api_preallocated_and_async(cuda_device):
    g = torch.Generator().manual_seed(5)
    shape = (4, 4, 640, 128)
    q, k, v = (torch.randn(shape, generator=g).to(torch.bfloat16).pin_memory() for _ in range(3))
    out = torch.empty(shape, dtype=torch.bfloat16).pin_memory()
    lse = torch.empty(shape[:3], dtype=torch.float32).pin_memory()
    ref_o, ref_l = _device_run(q, k, v, False, 0.1, cuda_device, bm=128, bn=128)
    o, l = faf.attention_host(q, k, v, False, 0.1, BM=128, BN=128, return_lse=True,
                              device=cuda_device, out=out, lse=lse)
    assert o.data_ptr() == out.data_ptr() and l.data_ptr() == lse.data_ptr()
    assert torch.equal(o, ref_o) and torch.equal(l, ref_l)

    out.zero_()
    host_stream.forward_host(q, k, v, False, 0.1, device=cuda_device, out=out, lse=lse,
                             block_m=128, block_n=128, chunk_slices=3, synchronize=False)
    torch.cuda.current_stream(cuda_device).synchronize()
    assert torch.equal(out, ref_o)


@pytest.mark.gpu
def test_forward_host_fp8_v(cuda_device):
    g = torch.Generator().manual_seed(8)
    q, k = (torch.randn(2, 3, 400, 128, generator=g).to(torch.float16) for _ in range(2))
    v = torch.randn(2, 3, 400, 128, generator=g).to(torch.float8_e5m2)
    ref_o, ref_l = _device_run(q, k, v, True, 0.09, cuda_device)
    o, l = faf.attention_host(q, k, v, True, 0.09, return_lse=True, device=cuda_device)
    assert o.dtype == torch.float16
    assert torch.equal(o, ref_o) and torch.equal(l, ref_l)


@pytest.mark.gpu
def test_forward_host_empty_and_unsupported_tile(cuda_device):
    q, k, v = _host((0, 2, 64, 64))
    o, l = host_stream.forward_host(q, k, v, False, 0.125, device=cuda_device)
    assert o.shape == q.shape and l.shape == (0, 2, 64)
    q, k, v = _host((1, 2, 64, 64))
    with pytest.raises(ValueError):
        host_stream.forward_host(q, k, v, False, 0.125, device=cuda_device, block_m=96,
                                 block_n=64)
    # the device stays usable after the launch error
    o, _ = host_stream.forward_host(q, k, v, False, 0.125, device=cuda_device)
    assert torch.isfinite(o.float()).all()
