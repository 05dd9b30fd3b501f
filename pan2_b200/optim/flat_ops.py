"""Flat-shard optimizer primitives: CUDA tensors run ``csrc/optim_ops.cu``; CPU tensors run the same
math in PyTorch (used by the gloo multi-rank tests and the CPU oracle)."""
from __future__ import annotations

import math
from typing import Optional

import torch

from ..ops._ext import ext


def _join(hi: torch.Tensor, lo: torch.Tensor) -> torch.Tensor:
    h = hi.view(torch.int16).to(torch.int32) & 0xFFFF
    l = lo.view(torch.int16).to(torch.int32) & 0xFFFF
    return ((h << 16) | l).view(torch.float32)


def _split_into(x: torch.Tensor, hi: torch.Tensor, lo: torch.Tensor) -> None:
    b = x.float().contiguous().view(torch.int32)
    hi.view(torch.int16).copy_(((b >> 16) & 0xFFFF).to(torch.int16))
    lo.view(torch.int16).copy_((b & 0xFFFF).to(torch.int16))


def split_master(x: torch.Tensor, hi: torch.Tensor, lo: torch.Tensor) -> None:
    if x.is_cuda:
        ext().split_master(x, hi, lo)
    else:
        _split_into(x, hi, lo)


def join_master(hi: torch.Tensor, lo: torch.Tensor) -> torch.Tensor:
    if hi.is_cuda:
        out = torch.empty(hi.numel(), dtype=torch.float32, device=hi.device)
        ext().join_master(hi, lo.to(hi.device), out)
        return out
    return _join(hi, lo)


def sumsq_partial(x: torch.Tensor, partial: torch.Tensor) -> None:
    if x.is_cuda:
        ext().sumsq_partial(x, partial)
    else:
        partial.zero_()
        partial[0] = x.float().pow(2).sum()


def norm_and_clip(partials: torch.Tensor, max_norm: float, out: torch.Tensor) -> None:
    if partials.is_cuda:
        ext().norm_and_clip(partials, max_norm, out)
    else:
        n = partials.sum().sqrt()
        out[0] = n
        out[1] = min(1.0, max_norm / (n.item() + 1e-6)) if max_norm > 0 else 1.0


def muon_momentum(buf: torch.Tensor, g: torch.Tensor, clip: Optional[torch.Tensor], mu: float, out: torch.Tensor):
    if buf.is_cuda:
        ext().muon_momentum(buf, g, clip, mu, out)
        return
    gi = g.float() * (clip[0] if clip is not None else 1.0)
    buf.mul_(mu).add_(gi, alpha=1 - mu)
    out.copy_((1 - mu) * gi + mu * buf)


def muon_update(hi, lo, u, lr_t, lr_scale: float, wd: float) -> None:
    if hi.is_cuda:
        ext().muon_update(hi, lo, u, lr_t, lr_scale, wd)
        return
    lr = float(lr_t[0])
    p = _join(hi, lo) * (1 - lr * wd) - lr * lr_scale * u.float()
    _split_into(p, hi, lo)


def adamw_update(hi, lo, g, m, v, clip, lr_t, beta1, beta2, eps, wd, step: int) -> None:
    if hi.is_cuda:
        ext().adamw_update(hi, lo, g, m, v, clip, lr_t, beta1, beta2, eps, wd, step)
        return
    lr = float(lr_t[0])
    gi = g.float() * (clip[0] if clip is not None else 1.0)
    m.mul_(beta1).add_(gi, alpha=1 - beta1)
    v.mul_(beta2).addcmul_(gi, gi, value=1 - beta2)
    bc1 = 1 - beta1 ** step
    bc2 = 1 - beta2 ** step
    p = _join(hi, lo) * (1 - lr * wd)
    p = p - (lr / bc1) * m / (v.sqrt() / math.sqrt(bc2) + eps)
    _split_into(p, hi, lo)
