"""Grouped QKV projection with per-head RMS q/k norm, RoPE and the concat -> interleave permute.

One autograd node, like the reference's ``gmlp::grouped_qkv_proj_fwd`` custom op
(pan/models/transformers/modules/mlp_ops.py:283-420 with the Triton kernels K13-K16 of
triton_kernels.py:1170-1668):

1. ``raw = x_mod @ W[mod]^T + b[mod]`` per modality (video rows, then text rows, concat layout);
2. for Q and K, per token and head: ``z = raw * w[mod] * rsqrt(mean(raw^2) + eps)`` and RoPE
   ``y = z * cos + rotate_half(z) * sin`` in fp32, rounded once to bf16;
3. every row (Q, K and V) is stored at its interleave position ``interleave_to_concat[p]``.

On CUDA, step 1 is the tcgen05 grouped GEMM and steps 2-3 one kernel (``csrc/qkv_ops.cu``) whose
backward also produces the q/k affine gradients.  Outputs are ``[L, H, D]``; padding rows are zero.
"""
from __future__ import annotations

from typing import Sequence, Tuple

import torch
import torch.nn.functional as F

from ._ext import ext
from .gemm import grouped_mm_nt, mm_nn, mm_tn
from .packed import segment_sum
from ..models.rope import rotate_half


class _QKVProjCUDA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, qw, kw, cos, sin, itc, bounds, heads, eps):
        L = x.shape[0]
        wc = w.to(torch.bfloat16).contiguous()
        bc = b.to(torch.bfloat16).contiguous()
        raw = torch.empty(L, wc.shape[1], dtype=torch.bfloat16, device=x.device)
        grouped_mm_nt(x, wc, bounds, raw, bias=bc)
        q, k, v = ext().qkv_post_fwd(raw, qw.float().contiguous(), kw.float().contiguous(), cos, sin, itc,
                                     bounds[1], bounds[2], heads, eps)
        ctx.save_for_backward(x, wc, raw, qw, kw, cos, sin, itc)
        ctx.bounds, ctx.heads, ctx.eps = list(bounds), heads, eps
        ctx.dtypes = (w.dtype, b.dtype, qw.dtype, kw.dtype)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        x, wc, raw, qw, kw, cos, sin, itc = ctx.saved_tensors
        bounds = ctx.bounds
        draw, dqw, dkw = ext().qkv_post_bwd(dq.contiguous(), dk.contiguous(), dv.contiguous(), raw,
                                            qw.float().contiguous(), kw.float().contiguous(), cos, sin, itc,
                                            bounds[1], bounds[2], ctx.heads, ctx.eps)
        gx = torch.zeros_like(x)
        gw = torch.zeros(wc.shape, dtype=torch.float32, device=x.device)
        for g in range(len(bounds) - 1):
            r0, r1 = bounds[g], bounds[g + 1]
            if r1 <= r0:
                continue
            mm_nn(draw[r0:r1], wc[g], out=gx[r0:r1])
            mm_tn(draw[r0:r1], x[r0:r1], out=gw[g])
        gb = segment_sum(draw, bounds)
        wdt, bdt, qdt, kdt = ctx.dtypes
        return (gx, gw.to(wdt), gb.to(bdt), dqw.to(qdt), dkw.to(kdt),
                None, None, None, None, None, None)


def qkv_project(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, q_weight: torch.Tensor,
                k_weight: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                interleave_to_concat: torch.Tensor, bounds: Sequence[int], heads: int,
                eps: float = 1e-6) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Returns ``q, k, v`` ``[L, H, D]`` in interleave layout.

    ``weight`` is ``[2, 3*hidden, hidden]``, ``bias`` ``[2, 3*hidden]``, ``q_weight``/``k_weight``
    ``[2*D]`` (video affine then text affine), ``cos``/``sin`` ``[L, D]`` (or ``[L, 1, D]``) fp32 in
    interleave layout, ``bounds = [0, n_video, n_video + n_text]``.
    """
    L, hidden = x.shape
    D = hidden // heads
    cos2 = cos.reshape(cos.shape[0], -1)
    sin2 = sin.reshape(sin.shape[0], -1)
    if x.is_cuda:
        return _QKVProjCUDA.apply(x.to(torch.bfloat16).contiguous(), weight, bias, q_weight, k_weight,
                                  cos2.float().contiguous(), sin2.float().contiguous(),
                                  interleave_to_concat.to(torch.int32).contiguous(), list(bounds), heads, eps)
    nv, na = bounds[1], bounds[2]
    outs_q, outs_k, outs_v = [], [], []
    for g, (r0, r1) in enumerate(((0, nv), (nv, na))):
        raw = F.linear(x[r0:r1], weight[g].to(x.dtype), bias[g].to(x.dtype))
        q, k, v = raw.view(r1 - r0, 3, heads, D).unbind(1)
        for t, w, acc in ((q, q_weight, outs_q), (k, k_weight, outs_k)):
            tf = t.float()
            r = torch.rsqrt(tf.pow(2).mean(-1, keepdim=True) + eps)
            acc.append(tf * w[g * D:(g + 1) * D].float() * r)
        outs_v.append(v)
    pad = L - na
    zf = x.new_zeros(pad, heads, D, dtype=torch.float32)
    qz = torch.cat(outs_q + [zf], 0)
    kz = torch.cat(outs_k + [zf], 0)
    vz = torch.cat(outs_v + [zf.to(x.dtype)], 0)
    itc = interleave_to_concat.long()
    # rows in concat order -> rope tables of their interleave position
    c = cos2.index_select(0, itc).unsqueeze(1).float()
    s = sin2.index_select(0, itc).unsqueeze(1).float()
    qr = (qz * c + rotate_half(qz) * s).to(x.dtype)
    kr = (kz * c + rotate_half(kz) * s).to(x.dtype)
    # scatter concat rows to interleave rows: out[itc[p]] = row p
    inv = torch.empty_like(itc)
    inv[itc] = torch.arange(L, device=itc.device)
    return qr.index_select(0, inv), kr.index_select(0, inv), vz.index_select(0, inv)
