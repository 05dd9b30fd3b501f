"""Rectified-flow training math: the noised sample, training-time draws and the time warp.

Semantics (and the arithmetic, operation for operation, so draws and warps are bit-identical) follow
pan/flow_matching.py:16-112 of the reference: time runs on ``[0, T]``; the sample at ``t`` is
``(1 - t/T) x_0 + (t/T) noise`` and the model regresses ``noise - x_0``; training times are
uniform or logit-normal, held ``1e-5`` inside ``(0, 1)``; the warp maps ``f = t/T`` to
``s f / (1 + (s - 1) f)``.  Under the ``dynamic`` rule ``log s`` is the sum of two straight-line
fits, one in the pixel area (256^2 -> 0.5, 1024^2 -> 1.15) and one in the frame count
(1 -> 0, 121 -> 1.64) of each sample, times ``rescale_factor``, and ``s`` is capped at ``max_shift``.
Those fits are training-distribution constants of the released checkpoints.
"""
from __future__ import annotations

from enum import Enum
from typing import Optional

import torch


class NoiseDraw(str, Enum):
    """Distribution of training times (config key ``flow_snr_type``)."""
    UNIFORM = "uniform"
    LOGNORM = "lognorm"


class ShiftRule(str, Enum):
    """One warp for all samples, or one per sample from its size (``train_timestep_shift_mode``)."""
    FIXED = "fixed"
    DYNAMIC = "dynamic"


MARGIN = 1e-5                      # draws stay this far from both ends of (0, 1)
_SPAN = (1.0 - MARGIN) - MARGIN


def _fit(p: tuple, q: tuple) -> tuple:
    """(slope, intercept) of the line through points ``p`` and ``q``."""
    slope = (q[1] - p[1]) / (q[0] - p[0])
    return slope, p[1] - slope * p[0]


# log-shift contributions: pixel area and frame count
_AREA_FIT = _fit((256 * 256, 0.5), (1024 * 1024, 1.15))
_FRAME_FIT = _fit((1, 0.0), (121, 1.64))


def interpolate(clean: torch.Tensor, noise: torch.Tensor, t: torch.Tensor, dim: int = 0, *,
                T: int = 1000) -> torch.Tensor:
    """Sample at times ``t`` (one per index of axis ``dim``) on the line from ``clean`` to ``noise``."""
    view = [-1 if a == dim % clean.dim() else 1 for a in range(clean.dim())]
    frac = (t / T).reshape(view)
    return (1 - frac) * clean + frac * noise


def draw_timesteps(count: int, device=None, generator: Optional[torch.Generator] = None, *,
                   distribution="lognorm", T: int = 1000, loc: float = 0.0, scale: float = 1.0,
                   default_device=None) -> torch.Tensor:
    """``count`` training times on ``[0, T]``."""
    where = device or default_device or "cpu"
    if NoiseDraw(distribution) == NoiseDraw.LOGNORM:
        z = torch.normal(mean=loc, std=scale, size=(count,), device=where, generator=generator)
        unit = 1.0 / (1.0 + torch.exp(-z))  # logistic of a normal draw
    else:
        unit = torch.rand((count,), device=where, generator=generator)
    return (unit * _SPAN + MARGIN) * T


def _dynamic_shift(latent_shapes: torch.Tensor, device, rescale_factor: float, max_shift: float,
                   frame_stride: int, pixel_stride_h: int, pixel_stride_w: Optional[int]) -> torch.Tensor:
    """Per-sample shift from ``[N, 3]`` token grids ``(t, h, w)`` (strides convert tokens to frames /
    pixels)."""
    g = latent_shapes.to(device=device, dtype=torch.float32)
    n_frames = (g[:, 0] - 1) * frame_stride + 1
    n_pixels = (g[:, 1] * pixel_stride_h) * (g[:, 2] * (pixel_stride_w or pixel_stride_h))
    log_shift = (_AREA_FIT[0] * n_pixels + _AREA_FIT[1]) + (_FRAME_FIT[0] * n_frames + _FRAME_FIT[1])
    return torch.exp(rescale_factor * log_shift).clamp(max=max_shift)


def shift_timesteps(timesteps: torch.Tensor, T: int, shift: float = 1.0, mode="fixed",
                    latent_shapes: Optional[torch.Tensor] = None, rescale_factor: float = 0.5,
                    max_shift: float = 1000.0, frame_stride: int = 4, pixel_stride_h: int = 16,
                    pixel_stride_w: Optional[int] = None) -> torch.Tensor:
    """Warp training times toward the noisy end (see the module docstring)."""
    if ShiftRule(mode) == ShiftRule.DYNAMIC:
        if latent_shapes is None:
            raise ValueError("the dynamic timestep shift needs each sample's latent grid (latent_shapes)")
        s = _dynamic_shift(latent_shapes, timesteps.device, rescale_factor, max_shift, frame_stride,
                           pixel_stride_h, pixel_stride_w)
    else:
        if shift == 1.0:
            return timesteps
        s = shift
    f = timesteps / T
    return s * f / (1 + (s - 1) * f) * T
