"""Variable-length (packed) non-causal attention.

Replaces the reference's FlashAttention-4 wrappers (pan/utils/flash_attention.py:18-243): the packed
training path attends within each ``cu_seqlens`` segment, returns the output and the per-row
log-sum-exp, and its backward gives ``dq, dk, dv``.  ``q, k, v`` are ``[L, H, D]`` bf16; the output
is ``[L, H, D]``.  Rows beyond the last boundary are padding: their output is zero and they
contribute nothing.

CUDA tensors run the tcgen05 kernels of ``csrc/attention_sm100.cu``; CPU tensors run PyTorch's
math attention per segment.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence

import torch
import torch.nn.functional as F

from ._ext import ext


_ITEM_CACHE: dict = {}


def work_items(lens: Sequence[int], rows_per_item: int, device) -> torch.Tensor:
    """int32 ``[n, 4]`` work list ``(segment start, segment length, first tile row, 0)``: one entry
    per ``rows_per_item`` rows of every non-empty segment.  Cached per (lens, tile, device)."""
    key = (tuple(int(n) for n in lens), rows_per_item, str(device))
    t = _ITEM_CACHE.get(key)
    if t is None:
        rows, start = [], 0
        for n in key[0]:
            for r0 in range(0, n, rows_per_item):
                rows.append((start, n, r0, 0))
            start += n
        t = torch.tensor(rows if rows else [(0, 0, 0, 0)][:0], dtype=torch.int32).reshape(-1, 4)
        if torch.device(device).type == "cuda":
            t = t.pin_memory()
        t = t.to(device, non_blocking=True)
        if len(_ITEM_CACHE) > 256:
            _ITEM_CACHE.clear()
        _ITEM_CACHE[key] = t
    return t


class _VarlenAttnCUDA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, lens, scale):
        n_valid = int(sum(lens))
        o, lse = ext().attn_fwd(q, k, v, work_items(lens, 256, q.device), n_valid, scale)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.lens, ctx.scale, ctx.n_valid = lens, scale, n_valid
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        items = work_items(ctx.lens, 128, q.device)
        dq, dk, dv = ext().attn_bwd(do.contiguous(), q, k, v, o, lse, items, items, ctx.n_valid, ctx.scale)
        return dq, dk, dv, None, None


def varlen_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens: torch.Tensor,
                     lens: Sequence[int], max_seqlen: Optional[int] = None,
                     scale: Optional[float] = None) -> torch.Tensor:
    """Attention within each segment of ``cu_seqlens``; ``lens`` are the host segment lengths."""
    D = q.shape[-1]
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    max_seqlen = int(max(lens)) if max_seqlen is None else int(max_seqlen)
    if q.is_cuda:
        return _VarlenAttnCUDA.apply(q.contiguous(), k.contiguous(), v.contiguous(),
                                     [int(n) for n in lens], float(scale))
    out = torch.zeros_like(q)
    pieces = []
    start = 0
    for n in lens:
        n = int(n)
        if n == 0:
            continue
        qs, ks, vs = (t[start:start + n].transpose(0, 1).unsqueeze(0) for t in (q, k, v))
        o = F.scaled_dot_product_attention(qs.float(), ks.float(), vs.float(), scale=scale)
        pieces.append((start, n, o[0].transpose(0, 1).to(q.dtype)))
        start += n
    if not pieces:
        return out
    rows = [p[2] for p in pieces]
    tail = q.shape[0] - start
    if tail:
        rows.append(q.new_zeros(tail, *q.shape[1:]))
    return torch.cat(rows, 0)


@torch.no_grad()
def attention_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, lens: Sequence[int],
                      scale: Optional[float] = None):
    """Forward only: ``(o, lse)`` of :func:`varlen_attention` (``lse`` is ``None`` on the CPU, whose
    backward recomputes the attention).  With :func:`kept_attention` this is selective activation
    checkpointing: the checkpointed forward keeps ``o`` / ``lse`` and the recompute before the
    backward skips the attention forward (reference: train.py:817-845, which keeps the FA4 forward
    outputs under ``use_dedicated_gradient_checkpointing``)."""
    D = q.shape[-1]
    scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    lens = [int(n) for n in lens]
    if q.is_cuda:
        o, lse = ext().attn_fwd(q.contiguous(), k.contiguous(), v.contiguous(), work_items(lens, 256, q.device),
                                int(sum(lens)), scale)
        return o, lse
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32)
    return varlen_attention(q, k, v, cu, lens, scale=scale), None


class _KeptAttn(torch.autograd.Function):
    """Attention whose forward output was kept: returns ``o``; the backward is the attention
    backward of ``q, k, v`` (the fused kernel with the kept ``o`` / ``lse`` on CUDA, a recomputation
    through the math path on the CPU)."""

    @staticmethod
    def forward(ctx, q, k, v, o, lse, lens, scale):
        ctx.save_for_backward(q, k, v, o, *(() if lse is None else (lse,)))
        ctx.lens, ctx.scale, ctx.has_lse = lens, scale, lse is not None
        return o.view_as(o)

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, *rest = ctx.saved_tensors
        if ctx.has_lse:
            items = work_items(ctx.lens, 128, q.device)
            dq, dk, dv = ext().attn_bwd(do.contiguous(), q, k, v, o, rest[0], items, items, int(sum(ctx.lens)),
                                        ctx.scale)
            return dq, dk, dv, None, None, None, None
        cu = torch.tensor([0] + list(torch.tensor(ctx.lens).cumsum(0).tolist()), dtype=torch.int32)
        with torch.enable_grad():
            qd, kd, vd = (t.detach().requires_grad_(True) for t in (q, k, v))
            out = varlen_attention(qd, kd, vd, cu, ctx.lens, scale=ctx.scale)
            dq, dk, dv = torch.autograd.grad(out, (qd, kd, vd), do)
        return dq, dk, dv, None, None, None, None


def kept_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor, lse: Optional[torch.Tensor],
                   lens: Sequence[int], scale: Optional[float] = None) -> torch.Tensor:
    """:func:`varlen_attention` of ``q, k, v`` given its kept forward ``(o, lse)`` from
    :func:`attention_forward` on the same inputs."""
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else float(scale)
    return _KeptAttn.apply(q.contiguous(), k.contiguous(), v.contiguous(), o, lse, [int(n) for n in lens], scale)


def dense_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                    mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Self-attention over ``[B, S, H, D]`` where ``mask`` (``[B, S]``, True = valid) gates both
    queries and keys; masked query rows return zeros (reference attention.py:27-53)."""
    B, S, H, D = q.shape
    if mask is None:
        mask = torch.ones(B, S, dtype=torch.bool, device=q.device)
    mask = mask.to(device=q.device, dtype=torch.bool)
    idx = torch.nonzero(mask.flatten(), as_tuple=False).flatten()
    lens = mask.sum(-1).tolist()
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device=q.device)
    qf, kf, vf = (t.reshape(B * S, H, D).index_select(0, idx) for t in (q, k, v))
    o = varlen_attention(qf, kf, vf, cu, lens)
    out = q.new_zeros(B * S, H, D)
    out.index_copy_(0, idx, o[: idx.numel()])
    return out.view(B, S, H, D)
