"""Normalisation and adaLN conditioning blocks of the MMDiT.

Parameter names and the arithmetic the checkpoints were trained with are the reference's
(pan/models/transformers/modules/layers.py:24-119): RMS normalisation runs in fp32 and the result is
rounded to the input dtype before the learned scale multiplies it (that rounding point is part of
the bf16 model); the adaLN projection is ``linear(activation(embedding))`` with ``chunks * width``
outputs, zero at initialisation so a fresh block is the identity.  The packed training path applies
modulation and gating in fused kernels (``pan2_b200.ops.packed``), not here.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn


def make_activation(name: str) -> nn.Module:
    """A fresh activation module for a config name (``silu``, ``gelu``, ``gelu_tanh``, ``relu``)."""
    if name == "silu":
        return nn.SiLU()
    if name == "gelu":
        return nn.GELU()
    if name == "gelu_tanh":
        return nn.GELU(approximate="tanh")
    if name == "relu":
        return nn.ReLU()
    raise ValueError(f"activation {name!r} is not one of silu, gelu, gelu_tanh, relu")


def rms_norm(x: torch.Tensor, weight: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    """fp32 RMS normalisation, rounded to ``x.dtype`` before the (optional) scale."""
    wide = x.to(torch.float32)
    inv_rms = torch.rsqrt(wide.square().mean(dim=-1, keepdim=True) + eps)
    normed = (wide * inv_rms).to(x.dtype)
    return normed if weight is None else normed * weight


class RMSNorm(nn.Module):
    """RMS normalisation over the last dim with an optional learned per-channel scale ``weight``."""

    def __init__(self, dim: int, eps: float = 1e-6, elementwise_affine: bool = True):
        super().__init__()
        self.dim, self.eps, self.elementwise_affine = dim, eps, elementwise_affine
        if elementwise_affine:
            self.weight = nn.Parameter(torch.ones(dim))
        else:
            self.register_parameter("weight", None)

    def reset_parameters(self) -> None:
        if self.weight is not None:
            with torch.no_grad():
                self.weight.fill_(1.0)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return rms_norm(x, self.weight, self.eps)

    def extra_repr(self) -> str:
        return f"{self.dim}, eps={self.eps}, elementwise_affine={self.elementwise_affine}"


class AdaLNProjection(nn.Module):
    """``chunks`` modulation vectors of width ``width`` from a conditioning embedding."""

    def __init__(self, width: int, chunks: int, activation: str = "silu", zero_init: bool = True):
        super().__init__()
        self.act = make_activation(activation)
        self.linear = nn.Linear(width, chunks * width, bias=True)
        if zero_init:
            with torch.no_grad():
                self.linear.weight.zero_()
                self.linear.bias.zero_()

    def forward(self, emb: torch.Tensor) -> torch.Tensor:
        return self.linear(self.act(emb))
