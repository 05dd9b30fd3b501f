"""GEMM entry points and the GEMM-shaped autograd ops of the model.

All CUDA GEMMs run the persistent tcgen05/TMEM/TMA kernel of ``csrc/gemm_sm100.cu``:

``D[M, N] (+)= A[M, K] @ B[N, K]^T`` where each operand is stored either K-major (row-major with
K contiguous) or MN-major (its M/N index contiguous).  That one kernel covers the three products of
a linear layer:

* forward ``Y = X W^T``            — A = X (K-major), B = W (K-major);
* input grad ``dX = dY W``         — A = dY (K-major), B = W viewed as ``[K=N_out, N=K_in]`` (MN-major);
* weight grad ``dW = dY^T X``      — A = dY^T (MN-major), B = X^T (MN-major).

Epilogues: optional bias (bf16/fp32), GELU-tanh with the pre-activation written alongside,
fp32 or bf16 output, accumulate into the output.  Grouped variants take up to four row groups,
each with its own weight/bias, which is how the per-modality (video/text) projections of the
reference's ``gmlp`` custom ops (pan/models/transformers/modules/mlp_ops.py:59-660) run as one
launch.

CPU tensors take the plain PyTorch path with identical semantics.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch
import torch.nn.functional as F

from ._ext import ext
from .packed import segment_sum


# --------------------------------------------------------------------------------------------
# raw products
# --------------------------------------------------------------------------------------------

def _check_cuda_gemm(*ts):
    for t in ts:
        if t is not None and t.dtype not in (torch.bfloat16,):
            raise TypeError(f"sm_100a GEMM operands must be bf16, got {t.dtype}")


def mm_nt(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None,
          bias: Optional[torch.Tensor] = None, gelu_pre: Optional[torch.Tensor] = None,
          accumulate: bool = False, out_dtype=None) -> torch.Tensor:
    """``a[M,K] @ b[N,K]^T`` (+bias, GELU-tanh writing the pre-activation to ``gelu_pre``)."""
    M, N = a.shape[0], b.shape[0]
    if a.is_cuda:
        _check_cuda_gemm(a, b)
        if out is None:
            out = torch.empty(M, N, dtype=out_dtype or a.dtype, device=a.device)
        ext().gemm(a, b, out, True, True, bias, gelu_pre, accumulate)
        return out
    y = a.float() @ b.float().t()
    if bias is not None:
        y = y + bias.float()
    if gelu_pre is not None:
        gelu_pre.copy_(y)
        y = F.gelu(y, approximate="tanh")
    return _finish(y, out, accumulate, out_dtype or a.dtype)


def mm_nn(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None,
          accumulate: bool = False, out_dtype=None) -> torch.Tensor:
    """``a[M,K] @ b[K,N]``."""
    M, N = a.shape[0], b.shape[1]
    if a.is_cuda:
        _check_cuda_gemm(a, b)
        if out is None:
            out = torch.empty(M, N, dtype=out_dtype or a.dtype, device=a.device)
        ext().gemm(a, b, out, True, False, None, None, accumulate)
        return out
    return _finish(a.float() @ b.float(), out, accumulate, out_dtype or a.dtype)


def mm_tn(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None,
          accumulate: bool = False, out_dtype=None) -> torch.Tensor:
    """``a[K,M]^T @ b[K,N]`` (weight gradients: reduction over the token dim)."""
    M, N = a.shape[1], b.shape[1]
    if a.is_cuda:
        _check_cuda_gemm(a, b)
        if out is None:
            out = torch.empty(M, N, dtype=out_dtype or torch.float32, device=a.device)
        ext().gemm(a, b, out, False, False, None, None, accumulate)
        return out
    return _finish(a.float().t() @ b.float(), out, accumulate, out_dtype or torch.float32)


def _finish(y, out, accumulate, dtype):
    if out is None:
        return y.to(dtype)
    if accumulate:
        out.add_(y.to(out.dtype))
    else:
        out.copy_(y)
    return out


def grouped_mm_nt(a: torch.Tensor, w: torch.Tensor, bounds: Sequence[int], out: torch.Tensor,
                  bias: Optional[torch.Tensor] = None, gelu_pre: Optional[torch.Tensor] = None,
                  n_cols: Optional[Sequence[int]] = None) -> torch.Tensor:
    """Rows ``bounds[g]:bounds[g+1]`` of ``out`` get ``a[rows] @ w[g]^T (+ bias[g])``.

    ``w`` is ``[G, N, K]`` (or a list of ``[N_g, K]`` weights, with ``n_cols`` their widths).
    """
    G = len(bounds) - 1
    if a.is_cuda:
        ws = [w[g] for g in range(G)] if isinstance(w, torch.Tensor) else list(w)
        bs = [None] * G if bias is None else ([bias[g] for g in range(G)] if isinstance(bias, torch.Tensor) else list(bias))
        ext().gemm_grouped_nt(a, ws, out, bs, gelu_pre, list(bounds))
        return out
    for g in range(G):
        r0, r1 = bounds[g], bounds[g + 1]
        if r1 <= r0:
            continue
        wg = w[g]
        ng = wg.shape[0]
        y = a[r0:r1].float() @ wg.float().t()
        if bias is not None:
            y = y + bias[g].float()
        if gelu_pre is not None:
            gelu_pre[r0:r1, :ng] = y.to(gelu_pre.dtype)
            y = F.gelu(y, approximate="tanh")
        out[r0:r1, :ng] = y.to(out.dtype)
    return out


# --------------------------------------------------------------------------------------------
# autograd ops
# --------------------------------------------------------------------------------------------

def _pad_k(t: torch.Tensor, k_pad: int) -> torch.Tensor:
    """Zero-pad the last dim to ``k_pad`` (TMA needs 16-byte row strides)."""
    if t.shape[-1] == k_pad:
        return t.contiguous()
    out = t.new_zeros(*t.shape[:-1], k_pad)
    out[..., : t.shape[-1]] = t
    return out


class _LinearCUDA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b):
        shp = x.shape
        K = shp[-1]
        k_pad = (K + 7) // 8 * 8
        x2 = _pad_k(x.reshape(-1, K), k_pad)
        wc = _pad_k(w.to(torch.bfloat16), k_pad)
        bc = None if b is None else b.to(torch.bfloat16).contiguous()
        y = mm_nt(x2, wc, bias=bc)
        ctx.save_for_backward(x2, wc)
        ctx.shp = shp
        ctx.K = K
        ctx.w_dtype = w.dtype
        ctx.has_b = b is not None
        ctx.b_dtype = None if b is None else b.dtype
        return y.reshape(*shp[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x2, wc = ctx.saved_tensors
        g2 = gy.reshape(-1, gy.shape[-1]).contiguous().to(torch.bfloat16)
        K = ctx.K
        gx = mm_nn(g2, wc)[:, :K].reshape(ctx.shp) if ctx.needs_input_grad[0] else None
        gw = mm_tn(g2, x2, out_dtype=torch.float32)[:, :K].to(ctx.w_dtype) if ctx.needs_input_grad[1] else None
        gb = segment_sum(g2, [0, g2.shape[0]])[0].to(ctx.b_dtype) if ctx.has_b and ctx.needs_input_grad[2] else None
        return gx, gw, gb


def linear(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x @ w^T + b``; CUDA inputs compute in bf16 on the sm_100a GEMM with fp32 accumulation."""
    if x.is_cuda:
        return _LinearCUDA.apply(x.to(torch.bfloat16), w, b)
    return F.linear(x, w.to(x.dtype), None if b is None else b.to(x.dtype))


def _rows_outside_zeroed(t: torch.Tensor, bounds: Sequence[int]) -> torch.Tensor:
    """``t`` (fresh, uninitialised) with the rows outside ``[bounds[0], bounds[-1])`` zeroed; the
    grouped GEMMs write every row inside the bounds."""
    if bounds[0] > 0:
        t[:bounds[0]].zero_()
    if bounds[-1] < t.shape[0]:
        t[bounds[-1]:].zero_()
    return t


class _GroupedLinearCUDA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, bounds):
        G = len(bounds) - 1
        wc = w.to(torch.bfloat16).contiguous()
        bc = b.to(torch.bfloat16).contiguous()
        out = _rows_outside_zeroed(torch.empty(x.shape[0], wc.shape[1], dtype=torch.bfloat16, device=x.device),
                                   bounds)
        grouped_mm_nt(x, wc, bounds, out, bias=bc)
        ctx.save_for_backward(x, wc)
        ctx.bounds = list(bounds)
        ctx.w_dtype, ctx.b_dtype = w.dtype, b.dtype
        return out

    @staticmethod
    def backward(ctx, gy):
        x, wc = ctx.saved_tensors
        bounds = ctx.bounds
        gy = gy.contiguous()
        gx = _rows_outside_zeroed(torch.empty_like(x), bounds)
        gw = torch.zeros(wc.shape, dtype=torch.float32, device=x.device)
        for g in range(len(bounds) - 1):
            r0, r1 = bounds[g], bounds[g + 1]
            if r1 <= r0:
                continue
            mm_nn(gy[r0:r1], wc[g], out=gx[r0:r1])
            mm_tn(gy[r0:r1], x[r0:r1], out=gw[g])
        gb = segment_sum(gy, bounds)
        return gx, gw.to(ctx.w_dtype), gb.to(ctx.b_dtype), None


def grouped_linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, bounds: Sequence[int]) -> torch.Tensor:
    """Per-group linear: rows ``bounds[g]:bounds[g+1]`` use ``w[g]``/``b[g]``; other rows are zero.

    ``w`` is ``[G, N, K]`` and ``b`` is ``[G, N]``.  This is the reference's ``grouped_out_proj``
    without the gather (the attention kernel already writes its output in concat order).
    """
    if x.is_cuda:
        return _GroupedLinearCUDA.apply(x.to(torch.bfloat16).contiguous(), w, b, list(bounds))
    out = x.new_zeros(x.shape[0], w.shape[1])
    parts = []
    for g in range(len(bounds) - 1):
        r0, r1 = bounds[g], bounds[g + 1]
        parts.append(F.linear(x[r0:r1], w[g].to(x.dtype), b[g].to(x.dtype)))
    tail = x.shape[0] - bounds[-1]
    parts.append(x.new_zeros(tail, w.shape[1]))
    return torch.cat(parts, 0) if parts else out


FFN_ROW_CHUNK = 16384


def _chunks(r0: int, r1: int, size: int):
    for a in range(r0, r1, size):
        yield a, min(a + size, r1)


class _GroupedFFNCUDA(torch.autograd.Function):
    """Per-modality GELU-tanh MLP.  Forward stores only the bf16 pre-activation; GELU is recomputed
    in the backward's dGELU epilogue.  Rows are processed in chunks so the [rows, hidden] temporaries
    (post-activation, its gradient) stay small at 100k-token batches."""

    @staticmethod
    def forward(ctx, x, bounds, *params):
        G = len(bounds) - 1
        wu = [params[4 * g + 0].to(torch.bfloat16) for g in range(G)]
        bu = [params[4 * g + 1].to(torch.bfloat16) for g in range(G)]
        wd = [params[4 * g + 2].to(torch.bfloat16) for g in range(G)]
        bd = [params[4 * g + 3].to(torch.bfloat16) for g in range(G)]
        L = x.shape[0]
        hidden = max(w.shape[0] for w in wu)
        pre = torch.empty(L, hidden, dtype=torch.bfloat16, device=x.device)
        out = _rows_outside_zeroed(torch.empty(L, wd[0].shape[0], dtype=torch.bfloat16, device=x.device), bounds)
        E = ext()
        for g in range(G):
            hid = wu[g].shape[0]
            for a, b in _chunks(bounds[g], bounds[g + 1], FFN_ROW_CHUNK):
                post = torch.empty(b - a, hid, dtype=torch.bfloat16, device=x.device)
                E.gemm(x[a:b], wu[g], post, True, True, bu[g], pre[a:b, :hid], False)
                E.gemm(post, wd[g], out[a:b], True, True, bd[g], None, False)
        ctx.save_for_backward(x, pre, *wu, *wd)
        ctx.bounds, ctx.G = list(bounds), G
        ctx.dtypes = [p.dtype for p in params]
        return out

    @staticmethod
    def backward(ctx, gy):
        saved = ctx.saved_tensors
        G, bounds = ctx.G, ctx.bounds
        x, pre = saved[0], saved[1]
        wu, wd = saved[2:2 + G], saved[2 + G:2 + 2 * G]
        gy = gy.contiguous()
        gx = _rows_outside_zeroed(torch.empty_like(x), bounds)
        grads = []
        E = ext()
        dev = x.device
        for g in range(G):
            hid, H = wu[g].shape[0], wd[g].shape[0]
            gwu = torch.zeros(hid, x.shape[1], dtype=torch.float32, device=dev)
            gwd = torch.zeros(H, hid, dtype=torch.float32, device=dev)
            gbu = torch.zeros(hid, dtype=torch.float32, device=dev)
            gbd = torch.zeros(H, dtype=torch.float32, device=dev)
            for a, b in _chunks(bounds[g], bounds[g + 1], FFN_ROW_CHUNK):
                gyg = gy[a:b]
                dpre = torch.empty(b - a, hid, dtype=torch.bfloat16, device=dev)
                post = torch.empty(b - a, hid, dtype=torch.bfloat16, device=dev)
                E.gemm_dgelu(gyg, wd[g], pre[a:b, :hid], dpre, post)   # d pre = (gy Wd) * gelu'(pre)
                E.gemm(gyg, post, gwd, False, False, None, None, True)  # gWd += gy^T post
                gbd += segment_sum(gyg, [0, b - a])[0]
                E.gemm(dpre, wu[g], gx[a:b], True, False, None, None, False)  # gx = dpre Wu
                E.gemm(dpre, x[a:b], gwu, False, False, None, None, True)    # gWu += dpre^T x
                gbu += segment_sum(dpre, [0, b - a])[0]
            grads += [gwu, gbu, gwd, gbd]
        grads = [gr.to(dt) for gr, dt in zip(grads, ctx.dtypes)]
        return (gx, None, *grads)


def grouped_ffn(x: torch.Tensor, bounds: Sequence[int], params: Sequence[torch.Tensor]) -> torch.Tensor:
    """GELU-tanh MLP per row group; ``params`` = ``[w_up, b_up, w_down, b_down] * G``."""
    if x.is_cuda:
        return _GroupedFFNCUDA.apply(x.to(torch.bfloat16).contiguous(), list(bounds), *params)
    G = len(bounds) - 1
    parts = []
    for g in range(G):
        r0, r1 = bounds[g], bounds[g + 1]
        wu, bu, wd, bd = params[4 * g: 4 * g + 4]
        h = F.gelu(F.linear(x[r0:r1], wu.to(x.dtype), bu.to(x.dtype)), approximate="tanh")
        parts.append(F.linear(h, wd.to(x.dtype), bd.to(x.dtype)))
    parts.append(x.new_zeros(x.shape[0] - bounds[-1], params[2].shape[0]))
    return torch.cat(parts, 0)
