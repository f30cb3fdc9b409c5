"""CPU oracle for the attention forward -- TEST INFRASTRUCTURE ONLY.

Only tests/, `__graft_entry__.smoke()` and bench.py's CPU-baseline leg may import this module,
and only as the checker (or as the timed CPU baseline).  The product path
(`flash_attention_forward.py`, `flash_attn_npu_b200/`) never calls it; without the CUDA
library the product raises.

What it restates
----------------
The reference's hardware-independent attention path, `_torch_attention_reference` in
ZyEng-Art/flash_attn_npu evaluate_attention.py:134-143:

    scores = (q.float() @ k.float().T) * sm_scale          # :135
    causal: scores.masked_fill(triu(ones, diagonal=1), -inf)  # :136-141
    probs  = softmax(scores, dim=-1, dtype=float32)          # :142
    out    = (probs @ v.float()).to(q.dtype)                 # :143

The evaluator uses it as the correctness oracle whenever the vendor op is unavailable
(evaluate_attention.py:151-156).  The reference kernel additionally emits the per-row
logsumexp `M = m + log(l)` (flash_attention_forward.py:1022, 1031); here that is
`logsumexp(scores, -1)` of the same fp32 scores.  The oracle returns fp32 (it skips the final
`.to(q.dtype)` so parity can be measured before rounding).

Pinning
-------
tests/golden/*.npz hold inputs and outputs produced by importing the reference evaluator
itself (script: tests/golden/make_golden.py); tests/test_oracle.py checks this restatement
against every fixture.
"""
from __future__ import annotations

import numpy as np
import torch


def attention_ref_torch(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool,
                        sm_scale: float) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 attention + natural-log LSE on whatever device the inputs live on.

    Follows evaluate_attention.py:135-143 line by line (matmul in fp32, -inf causal mask,
    fp32 softmax, fp32 P.V).  Works on [..., S, D] tensors.
    """
    qf, kf, vf = q.float(), k.float(), v.float()
    scores = torch.matmul(qf, kf.transpose(-2, -1)) * sm_scale
    if causal:
        mask = torch.triu(torch.ones((q.shape[-2], k.shape[-2]), device=q.device,
                                     dtype=torch.bool), diagonal=1)
        scores = scores.masked_fill(mask, float("-inf"))
    lse = torch.logsumexp(scores, dim=-1)
    probs = torch.softmax(scores, dim=-1, dtype=torch.float32)
    out = torch.matmul(probs, vf)
    return out, lse


def attention_ref_sliced(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool,
                         sm_scale: float, slices=None):
    """Per-(b, h) evaluation, so S x S fp32 scores never exceed one slice at a time.

    `slices` is an iterable of (b, h) pairs (default: all).  Returns dicts keyed by (b, h).
    """
    z, h = q.shape[0], q.shape[1]
    if slices is None:
        slices = [(b, hh) for b in range(z) for hh in range(h)]
    outs, lses = {}, {}
    for b, hh in slices:
        o, l = attention_ref_torch(q[b, hh], k[b, hh], v[b, hh], causal, sm_scale)
        outs[(b, hh)] = o
        lses[(b, hh)] = l
    return outs, lses


def attention_ref_numpy(q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool,
                        sm_scale: float, acc_dtype=np.float64) -> tuple[np.ndarray, np.ndarray]:
    """Same restatement in numpy (default float64 accumulation) for [B, H, S, D] arrays.

    A second, independent evaluation of evaluate_attention.py:135-143 used to bound the
    fp32 torch oracle's own rounding.
    """
    qa, ka, va = (np.asarray(x, dtype=acc_dtype) for x in (q, k, v))
    scores = np.matmul(qa, np.swapaxes(ka, -1, -2)) * acc_dtype(sm_scale)
    if causal:
        s = scores.shape[-1]
        mask = np.triu(np.ones((s, s), dtype=bool), k=1)
        scores = np.where(mask, -np.inf, scores)
    m = np.max(scores, axis=-1, keepdims=True)
    e = np.exp(scores - m)
    l = np.sum(e, axis=-1, keepdims=True)
    out = np.matmul(e / l, va)
    lse = (m + np.log(l))[..., 0]
    return out, lse


# ----------------------------------------------------------------------------- fp8 V
# The reference's fp8_v mode (flash_attention_forward.py:704 and :737, selected at :996 / :1017
# when V is float8e5): Q and K stay 16-bit, P is rounded to float8 e5m2 before the P.V dot, the
# running sum l keeps the unrounded fp32 p.  Two restatements, both on CPU in fp32:
#   - attention_ref_fp8v_online: the reference's stable online softmax (:698-724) over key
#     blocks of `block_n` -- m_ij = max(m_i, rowmax), p = exp(qk - m_ij), alpha = exp(m_i - m_ij),
#     l = l*alpha + sum(p), acc = acc*alpha + fp8(p) @ v -- so P is rounded at the running max;
#   - attention_kernel_order_fp8v: the same product with the exponent base the sm_100a kernel
#     uses (base moves only when a block's max passes it by more than 8 in log2 units), so P is
#     rounded at exactly the values the kernel rounds; it pins the kernel's fp8 rounding, while
#     the online form bounds how far two valid orders of the same fp8 product can differ.

def _masked_scores(q, k, causal, sm_scale):
    s = (q.float() @ k.float().transpose(-1, -2)) * sm_scale
    if causal:
        n = s.shape[-1]
        s = s.masked_fill(torch.triu(torch.ones(n, n, dtype=torch.bool), diagonal=1), float("-inf"))
    return s


def attention_ref_fp8v_online(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool,
                              sm_scale: float, block_n: int = 128):
    """Reference-order fp8-V attention on CPU; returns fp32 (out, lse)."""
    s = _masked_scores(q, k, causal, sm_scale)
    vf = v.float()
    n = s.shape[-1]
    m = torch.full(s.shape[:-1], float("-inf"))
    l = torch.zeros(s.shape[:-1])
    acc = torch.zeros(*s.shape[:-1], vf.shape[-1])
    for j0 in range(0, n, block_n):
        blk = s[..., j0:j0 + block_n]
        m_new = torch.maximum(m, blk.amax(-1))
        p = torch.exp(blk - m_new[..., None])
        alpha = torch.exp(m - m_new)
        l = l * alpha + p.sum(-1)
        p8 = p.to(torch.float8_e5m2).float()
        acc = acc * alpha[..., None] + p8 @ vf[..., j0:j0 + block_n, :]
        m = m_new
    return acc / l[..., None], m + torch.log(l)


def attention_kernel_order_fp8v(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool,
                                sm_scale: float, block_n: int = 128, threshold: float = 8.0):
    """fp8-V attention with the sm_100a kernel's exponent bases; returns fp32 (out, lse)."""
    x = _masked_scores(q, k, causal, sm_scale) * 1.4426950408889634  # log2 units
    vf = v.float()
    n = x.shape[-1]
    m = torch.full(x.shape[:-1], float("-inf"))
    l = torch.zeros(x.shape[:-1])
    acc = torch.zeros(*x.shape[:-1], vf.shape[-1])
    for j0 in range(0, n, block_n):
        xb = x[..., j0:j0 + block_n]
        mt = xb.amax(-1)
        need = mt > m + threshold
        m_new = torch.where(need, mt, m)
        alpha = torch.where(need, torch.exp2(m - m_new), torch.ones_like(m))
        l = l * alpha
        acc = acc * alpha[..., None]
        m = m_new
        base = torch.where(torch.isinf(m), torch.zeros_like(m), m)
        p = torch.exp2(xb - base[..., None])
        l = l + p.sum(-1)
        acc = acc + p.to(torch.float8_e5m2).float() @ vf[..., j0:j0 + block_n, :]
    lse = (m + torch.log2(l)) * 0.6931471805599453
    return acc / l[..., None], lse
