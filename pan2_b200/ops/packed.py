"""Fused elementwise ops over packed ``[L, C]`` token matrices (autograd-aware).

Semantics match the reference's Triton ops in pan/models/transformers/modules/triton_kernels.py:

* ``ln_stats`` is ``[L, 2]`` fp32 ``(sum_c x, sum_c x^2)`` of a tensor whose affine-free LayerNorm
  (eps 1e-6) is fused into the next :func:`ln_modulate` (triton_kernels.py:255-285).  It carries no
  gradient; the consumer's backward is the exact LayerNorm backward w.r.t. ``x``.
* :func:`ln_modulate` ``= LN(x) * (1 + scale[seg]) + shift[seg]`` (K4-K6, triton_kernels.py:288-436).
* :func:`gate_residual` ``= y * gate[seg] + residual`` and emits ``ln_stats`` of the result (K7/K8,
  triton_kernels.py:558-667).
* :func:`simple_concat` builds the concat layout ``[video | text + text_type_vec | pad]`` with
  ``ln_stats`` (K9/K10, triton_kernels.py:753-869).
* :func:`concat_mse_sums` returns ``(sum (pred - target)^2, count)`` over the video rows (K11/K12,
  triton_kernels.py:986-1073); the caller averages across ranks.
* :func:`segment_sum` sums rows per segment in fp32 (K1, triton_kernels.py:69-139).

Segments are given as host lists of row boundaries (``bounds[s] .. bounds[s+1]``); rows outside the
last boundary are padding.  CUDA tensors run the sm_100a kernels of ``csrc/packed_ops.cu``; CPU
tensors run plain PyTorch with the same math.
"""
from __future__ import annotations

from typing import Optional, Sequence, Tuple

import torch

from ._ext import ext

LN_EPS = 1e-6


def _seg_index(bounds: Sequence[int], total: int, device) -> torch.Tensor:
    """Per-row segment id (``-1`` on padding rows), CPU path helper."""
    idx = torch.full((total,), -1, dtype=torch.long, device=device)
    for s in range(len(bounds) - 1):
        idx[bounds[s]:bounds[s + 1]] = s
    return idx


_BOUNDS_CACHE: dict = {}


def _bounds_tensor(bounds: Sequence[int], device) -> torch.Tensor:
    """Device int32 copy of host boundaries, cached: building it from a Python list would be a
    pageable host-to-device copy, which synchronises the host with the GPU on every call."""
    key = (tuple(int(b) for b in bounds), str(device))
    t = _BOUNDS_CACHE.get(key)
    if t is None:
        host = torch.tensor(key[0], dtype=torch.int32)
        if torch.device(device).type == "cuda":
            host = host.pin_memory()
        t = host.to(device, non_blocking=True)
        if len(_BOUNDS_CACHE) > 4096:
            _BOUNDS_CACHE.clear()
        _BOUNDS_CACHE[key] = t
    return t


# --------------------------------------------------------------------------------------------
# ln_stats
# --------------------------------------------------------------------------------------------

def ln_stats_of(x: torch.Tensor, n_rows: Optional[int] = None) -> torch.Tensor:
    """``(sum x, sum x^2)`` per row in fp32; rows at or beyond ``n_rows`` are zero."""
    n_rows = x.shape[0] if n_rows is None else n_rows
    xf = x.float()
    st = torch.stack([xf.sum(-1), xf.pow(2).sum(-1)], dim=-1)
    if n_rows < x.shape[0]:
        st[n_rows:] = 0
    return st


# --------------------------------------------------------------------------------------------
# ln_modulate
# --------------------------------------------------------------------------------------------

class _LnModulateCUDA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, ln_stats, shift, scale, bounds_t, n_seg, zero_grad_outside):
        out = ext().ln_modulate_fwd(x, ln_stats, shift.contiguous(), scale.contiguous(), bounds_t, n_seg)
        ctx.save_for_backward(x, ln_stats, scale, bounds_t)
        ctx.n_seg = n_seg
        return out

    @staticmethod
    def backward(ctx, gout):
        x, ln_stats, scale, bounds_t = ctx.saved_tensors
        gx, gshift, gscale = ext().ln_modulate_bwd(gout.contiguous(), x, ln_stats, scale.contiguous(),
                                                   bounds_t, ctx.n_seg)
        return gx, None, gshift.to(scale.dtype), gscale.to(scale.dtype), None, None, None


def ln_modulate(x: torch.Tensor, ln_stats: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor,
                bounds: Sequence[int], bounds_t: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``LayerNorm(x) * (1 + scale[seg]) + shift[seg]`` over the segments ``bounds``.

    ``shift``/``scale`` are ``[n_seg, C]``.  Padding rows of the output are zero and get a zero
    gradient.
    """
    n_seg = len(bounds) - 1
    assert shift.shape[0] >= n_seg and scale.shape[0] >= n_seg
    if x.is_cuda:
        if bounds_t is None:
            bounds_t = _bounds_tensor(bounds, x.device)
        return _LnModulateCUDA.apply(x.contiguous(), ln_stats, shift, scale, bounds_t, n_seg, True)
    L, C = x.shape
    seg = _seg_index(bounds, L, x.device)
    valid = seg >= 0
    xf = x.float()
    n = torch.nn.functional.layer_norm(xf, (C,), eps=LN_EPS)
    segc = seg.clamp(min=0)
    y = n * (1 + scale.float()[segc]) + shift.float()[segc]
    y = torch.where(valid[:, None], y, torch.zeros_like(y))
    return y.to(x.dtype)


# --------------------------------------------------------------------------------------------
# gate + residual (+ ln_stats)
# --------------------------------------------------------------------------------------------

class _GateResidualCUDA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, gate, residual, bounds_t, n_seg):
        out, stats = ext().gate_residual_fwd(y, gate.contiguous(), residual, bounds_t, n_seg)
        ctx.save_for_backward(y, gate, bounds_t)
        ctx.n_seg = n_seg
        ctx.mark_non_differentiable(stats)
        return out, stats

    @staticmethod
    def backward(ctx, gout, _gstats):
        y, gate, bounds_t = ctx.saved_tensors
        gout = gout.contiguous()
        gy, ggate = ext().gate_bwd(gout, y, gate.contiguous(), bounds_t, ctx.n_seg)
        return gy, ggate.to(gate.dtype), gout, None, None


def gate_residual(y: torch.Tensor, gate: torch.Tensor, residual: torch.Tensor, bounds: Sequence[int],
                  bounds_t: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """``out = y * gate[seg] + residual`` and ``ln_stats(out)``; padding rows keep the residual."""
    n_seg = len(bounds) - 1
    if y.is_cuda:
        if bounds_t is None:
            bounds_t = _bounds_tensor(bounds, y.device)
        return _GateResidualCUDA.apply(y.contiguous(), gate, residual.contiguous(), bounds_t, n_seg)
    L, C = y.shape
    seg = _seg_index(bounds, L, y.device)
    valid = (seg >= 0)[:, None]
    g = gate.float()[seg.clamp(min=0)]
    out = torch.where(valid, y.float() * g + residual.float(), residual.float()).to(residual.dtype)
    return out, ln_stats_of(out.detach(), bounds[-1])


# --------------------------------------------------------------------------------------------
# concat [video | text + ttv | pad]
# --------------------------------------------------------------------------------------------

class _ConcatCUDA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, vid, txt, ttv, total):
        out, stats = ext().simple_concat_fwd(vid, txt, ttv, total)
        ctx.n_video, ctx.n_text = vid.shape[0], txt.shape[0]
        ctx.has_ttv = ttv is not None
        ctx.ttv_dtype = ttv.dtype if ttv is not None else None
        ctx.mark_non_differentiable(stats)
        return out, stats

    @staticmethod
    def backward(ctx, gout, _gstats):
        gout = gout.contiguous()
        nv, nt = ctx.n_video, ctx.n_text
        gvid = gout[:nv]
        gtxt = gout[nv:nv + nt]
        gttv = None
        if ctx.has_ttv:
            gttv = ext().column_sum(gtxt).to(ctx.ttv_dtype)
        return gvid, gtxt, gttv, None


def simple_concat(vid: torch.Tensor, txt: torch.Tensor, total: int,
                  text_type_vec: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Concat layout ``[video | text + text_type_vec | zero pad]`` of ``total`` rows and its ln_stats."""
    nv, nt = vid.shape[0], txt.shape[0]
    if vid.is_cuda:
        ttv = None if text_type_vec is None else text_type_vec.to(vid.dtype).contiguous()
        return _ConcatCUDA.apply(vid.contiguous(), txt.to(vid.dtype).contiguous(), ttv, total)
    t = txt if text_type_vec is None else txt + text_type_vec.to(txt.dtype)
    pad = vid.new_zeros(total - nv - nt, vid.shape[1])
    out = torch.cat([vid, t.to(vid.dtype), pad], dim=0)
    return out, ln_stats_of(out.detach(), nv + nt)


# --------------------------------------------------------------------------------------------
# MSE over the video rows of the concat layout
# --------------------------------------------------------------------------------------------

class _MseCUDA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pred, target, n_video):
        sums = ext().mse_fwd(pred, target, n_video)   # [2] fp32: (sum sq, count)
        ctx.save_for_backward(pred, target)
        ctx.n_video = n_video
        return sums

    @staticmethod
    def backward(ctx, gsums):
        pred, target = ctx.saved_tensors
        gpred = ext().mse_bwd(pred, target, gsums.contiguous().float(), ctx.n_video)
        return gpred, None, None


def concat_mse_sums(pred: torch.Tensor, target: torch.Tensor, n_video: int) -> torch.Tensor:
    """``[sum (pred[:n_video] - target)^2, n_video * C]`` in fp32; differentiable in the first entry.

    The gradient of the count entry is ignored.
    """
    if pred.is_cuda:
        return _MseCUDA.apply(pred.contiguous(), target.contiguous(), n_video)
    d = pred[:n_video].float() - target.float()
    sq = d.pow(2).sum()
    count = torch.tensor(float(d.numel()), device=pred.device)
    return torch.stack([sq, count])


# --------------------------------------------------------------------------------------------
# segment sums
# --------------------------------------------------------------------------------------------

def segment_sum(x: torch.Tensor, bounds: Sequence[int], out_dtype=torch.float32) -> torch.Tensor:
    """``[n_seg, C]`` row sums per segment, accumulated in fp32."""
    n_seg = len(bounds) - 1
    if x.is_cuda:
        return ext().segment_sum(x.contiguous(), _bounds_tensor(bounds, x.device), n_seg).to(out_dtype)
    return torch.stack([x[bounds[s]:bounds[s + 1]].float().sum(0) for s in range(n_seg)]).to(out_dtype)


class _PermuteRowsCUDA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, index, inverse):
        ctx.save_for_backward(inverse)
        return ext().gather_rows(x.contiguous(), index)

    @staticmethod
    def backward(ctx, g):
        (inverse,) = ctx.saved_tensors
        return ext().gather_rows(g.contiguous(), inverse), None, None


def permute_rows(x: torch.Tensor, index: torch.Tensor, inverse: torch.Tensor) -> torch.Tensor:
    """``x[index]`` for a row permutation ``index`` whose inverse is ``inverse`` (differentiable:
    the gradient is gathered back with the inverse permutation)."""
    if x.is_cuda:
        return _PermuteRowsCUDA.apply(x, index.to(torch.int32), inverse.to(torch.int32))
    return x.index_select(0, index.long())


def gather_rows(x: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    """``x[index]`` for a 2-D/3-D tensor (row gather, no gradient on CUDA: use permute_rows)."""
    if x.is_cuda:
        return ext().gather_rows(x.contiguous(), index)
    return x.index_select(0, index.long())
