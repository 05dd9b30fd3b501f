"""Shared building blocks: activations, RMS normalisation and adaLN conditioning.

Semantics follow pan/models/transformers/modules/layers.py:24-119 of the reference:

* ``RMSNorm`` normalises in fp32, rounds back to the input dtype, and only then multiplies by the
  learned scale (layers.py:65-72).  The bf16 rounding point is part of the trained model.
* ``AdaLNProjection`` is ``Linear(act(emb))`` producing ``chunks * width`` values, zero-initialised
  when ``zero_init`` (layers.py:76-99).
* ``modulate(x, shift, scale) = x * (1 + scale) + shift`` and ``gate(x, g) = x * g`` with per-sample
  ``[B, C]`` conditioning broadcast over tokens (layers.py:102-119).
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.nn as nn

_ACTIVATIONS = {
    "gelu": nn.GELU,
    "gelu_tanh": lambda: nn.GELU(approximate="tanh"),
    "relu": nn.ReLU,
    "silu": nn.SiLU,
}


def activation_factory(name: str) -> Callable[[], nn.Module]:
    """Zero-argument constructor of the named activation module."""
    if name not in _ACTIVATIONS:
        raise ValueError(f"Unknown activation {name!r}; expected one of {sorted(_ACTIVATIONS)}")
    return _ACTIVATIONS[name]


def rms_norm(x: torch.Tensor, weight: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    """fp32 RMS normalisation, cast back to ``x.dtype`` before the affine scale."""
    xf = x.float()
    y = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)
    return y if weight is None else y * weight


class RMSNorm(nn.Module):
    """RMSNorm whose normalised value is rounded to the input dtype before the scale."""

    def __init__(self, dim: int, eps: float = 1e-6, elementwise_affine: bool = True):
        super().__init__()
        self.dim = dim
        self.eps = eps
        self.elementwise_affine = elementwise_affine
        self.weight = nn.Parameter(torch.ones(dim)) if elementwise_affine else None

    def reset_parameters(self) -> None:
        if self.weight is not None:
            nn.init.ones_(self.weight)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return rms_norm(x, self.weight, self.eps)

    def extra_repr(self) -> str:
        return f"{self.dim}, eps={self.eps}, elementwise_affine={self.elementwise_affine}"


class AdaLNProjection(nn.Module):
    """``linear(act(emb))`` producing ``chunks * width`` modulation values."""

    def __init__(self, width: int, chunks: int, make_act: Callable[[], nn.Module], zero_init: bool = True):
        super().__init__()
        self.act = make_act()
        self.linear = nn.Linear(width, chunks * width, bias=True)
        if zero_init:
            nn.init.zeros_(self.linear.weight)
            nn.init.zeros_(self.linear.bias)

    def forward(self, emb: torch.Tensor) -> torch.Tensor:
        return self.linear(self.act(emb))


def modulate(x: torch.Tensor, shift: Optional[torch.Tensor] = None,
             scale: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x * (1 + scale) + shift`` with ``[B, C]`` conditioning over ``[B, L, C]`` tokens."""
    if scale is not None:
        x = x * (1 + scale.unsqueeze(1))
    if shift is not None:
        x = x + shift.unsqueeze(1)
    return x


def gate(x: torch.Tensor, g: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x * g`` with a ``[B, C]`` gate broadcast over the tokens of ``[B, L, C]``."""
    return x if g is None else x * g.unsqueeze(1)
