"""Attention over host-resident q, k, v: (b, h) slices streamed through the GPU.

The reference's entry point takes device tensors (flash_attention_forward.py:1197); a caller
holding its inputs in host memory would copy q, k, v over, run the kernel and copy out, lse
back, one after the other -- on a B200 the three host copies take ~4x the kernel's time at
S=8192, D=128.  Attention is independent per (b, h) slice, so `forward_host` splits the
flattened B*H slices into chunks and runs three streams over a ring of device buffers:

    h2d stream:     copy q, k, v of chunk c         (waits until chunk c-NBUF's kernel is done)
    compute stream: kernel on chunk c               (waits for chunk c's copies and for chunk
                                                     c-NBUF's results to have left the device)
    d2h stream:     copy out, lse of chunk c back   (waits for chunk c's kernel)

so the host->device copies, the kernels and the device->host copies overlap, and a whole call
costs about one pass over the host link instead of the sum of the three.  The kernel launches
are the same `ops.forward` calls on contiguous [n, 1, S, D] chunks, so the results are
bit-identical to one launch over the whole batch.  Host tensors should be pinned
(`Tensor.pin_memory()`); pageable memory works but the copies then block the host.
"""
from __future__ import annotations

import torch

from . import ops

NBUF = 3                      # device buffers in the ring
TARGET_CHUNK_BYTES = 96 << 20  # q + k + v bytes per chunk

_streams: dict[int, tuple] = {}


def plan_chunks(n_slices: int, slice_bytes: int, target_bytes: int = TARGET_CHUNK_BYTES,
                chunk_slices: int | None = None, tail_split: int = 4) -> list[tuple[int, int]]:
    """[start, stop) slice ranges: `chunk_slices` per chunk, or as many as fit `target_bytes`
    (at least one), with the remainder in the last chunk.  When there is more than one chunk
    the last one is cut into `tail_split` smaller pieces: the last chunk's kernel and copy-out
    are the only part of the pipeline no copy-in overlaps."""
    if n_slices <= 0:
        return []
    if chunk_slices is None:
        chunk_slices = max(1, target_bytes // max(1, slice_bytes))
    if chunk_slices <= 0:
        raise ValueError("chunk_slices must be positive")
    cs = min(chunk_slices, n_slices)
    chunks = [(s, min(s + cs, n_slices)) for s in range(0, n_slices, cs)]
    if len(chunks) > 1 and tail_split > 1:
        a, b = chunks.pop()
        piece = max(1, -(-(b - a) // tail_split))
        chunks += [(s, min(s + piece, b)) for s in range(a, b, piece)]
    return chunks


def _side_streams(device: torch.device):
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _streams:
        _streams[idx] = tuple(torch.cuda.Stream(device=idx) for _ in range(3))
    return _streams[idx]


def _check_host(name: str, t: torch.Tensor) -> None:
    if t.device.type != "cpu":
        raise ValueError(f"{name} must be a host (CPU) tensor, got {t.device}")


def forward_host(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool,
                 sm_scale: float, *, device: torch.device | str | int | None = None,
                 out: torch.Tensor | None = None, lse: torch.Tensor | None = None,
                 block_m: int = 0, block_n: int = 0, num_stages: int = 0,
                 persistent_ctas: int = 0, chunk_slices: int | None = None,
                 synchronize: bool = True):
    """Attention forward of host tensors q, k, v [Z, H, N_CTX, D] on a CUDA device.

    Returns host tensors (out [Z, H, N_CTX, D] in q's dtype, fp32 lse [Z, H, N_CTX]); `out` and
    `lse` may be given preallocated (pinned, contiguous).  The same dtype, head-dim and tile
    rules as `ops.forward` apply.  With `synchronize=False` the call returns once the work is
    queued: the results are valid after the current stream of `device` has been synchronised.
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        _check_host(name, t)
    ops.validate_layout(q, k, v)
    z, h, n_ctx, head_dim = q.shape
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("device must be a CUDA device")
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())

    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    elif out.shape != q.shape or out.dtype != q.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous host tensor matching q in shape and dtype")
    if lse is None:
        lse = torch.empty((z, h, n_ctx), dtype=torch.float32, pin_memory=True)
    elif lse.shape != (z, h, n_ctx) or lse.dtype != torch.float32 or not lse.is_contiguous():
        raise ValueError("lse must be a contiguous float32 host tensor of shape [Z, H, N_CTX]")
    _check_host("out", out)
    _check_host("lse", lse)

    n = z * h
    if n == 0 or n_ctx == 0:
        return out, lse
    qf, kf, vf = (t.contiguous().view(n, 1, n_ctx, head_dim) for t in (q, k, v))
    of = out.view(n, 1, n_ctx, head_dim)
    lf = lse.view(n, 1, n_ctx)
    slice_bytes = n_ctx * head_dim * (q.element_size() + k.element_size() + v.element_size())
    chunks = plan_chunks(n, slice_bytes, chunk_slices=chunk_slices)
    cs = chunks[0][1] - chunks[0][0]
    nbuf = min(NBUF, len(chunks))

    with torch.cuda.device(device):
        caller = torch.cuda.current_stream(device)
        s_in, s_mma, s_out = _side_streams(device)
        bufs = []
        for _ in range(nbuf):
            bufs.append((torch.empty((cs, 1, n_ctx, head_dim), dtype=q.dtype, device=device),
                         torch.empty((cs, 1, n_ctx, head_dim), dtype=k.dtype, device=device),
                         torch.empty((cs, 1, n_ctx, head_dim), dtype=v.dtype, device=device),
                         torch.empty((cs, 1, n_ctx, head_dim), dtype=q.dtype, device=device),
                         torch.empty((cs, 1, n_ctx), dtype=torch.float32, device=device)))
        start = torch.cuda.Event()
        start.record(caller)  # the buffers were allocated on the caller's stream
        for s in (s_in, s_mma, s_out):
            s.wait_event(start)

        in_free = [None] * nbuf   # event: the kernel that last read buffer b is done
        out_free = [None] * nbuf  # event: the copy-out that last read buffer b is done
        try:
            _run_chunks(chunks, bufs, nbuf, (qf, kf, vf, of, lf), (s_in, s_mma, s_out),
                        in_free, out_free, causal, sm_scale,
                        dict(block_m=block_m, block_n=block_n, num_stages=num_stages,
                             persistent_ctas=persistent_ctas))
        finally:
            # The caller's stream resumes after all queued side-stream work (also when a
            # launch raised part-way); the ring buffers are freed on it, so the allocator
            # cannot hand them out while a copy or kernel still uses them.
            for s in (s_in, s_mma, s_out):
                ev = torch.cuda.Event()
                ev.record(s)
                caller.wait_event(ev)
            del bufs
        if synchronize:
            caller.synchronize()
    return out, lse


def _run_chunks(chunks, bufs, nbuf, host, streams, in_free, out_free, causal, sm_scale, tile):
    qf, kf, vf, of, lf = host
    s_in, s_mma, s_out = streams
    for c, (a, b_) in enumerate(chunks):
        m = b_ - a
        slot = c % nbuf
        qd, kd, vd, od, ld = (t[:m] for t in bufs[slot])
        with torch.cuda.stream(s_in):
            if in_free[slot] is not None:
                s_in.wait_event(in_free[slot])
            qd.copy_(qf[a:b_], non_blocking=True)
            kd.copy_(kf[a:b_], non_blocking=True)
            vd.copy_(vf[a:b_], non_blocking=True)
            loaded = torch.cuda.Event()
            loaded.record(s_in)
        with torch.cuda.stream(s_mma):
            s_mma.wait_event(loaded)
            if out_free[slot] is not None:
                s_mma.wait_event(out_free[slot])
            ops.forward(qd, kd, vd, causal, sm_scale, out=od, lse=ld, **tile)
            done = torch.cuda.Event()
            done.record(s_mma)
            in_free[slot] = done
        with torch.cuda.stream(s_out):
            s_out.wait_event(done)
            of[a:b_].copy_(od, non_blocking=True)
            lf[a:b_].copy_(ld, non_blocking=True)
            freed = torch.cuda.Event()
            freed.record(s_out)
            out_free[slot] = freed
