"""Rectified-flow training math: noising, timestep draws and the time shift.

Semantics of pan/flow_matching.py:16-112 in the reference: time runs on ``[0, T]`` (``T`` =
``num_train_timesteps``), ``x_t = (1 - t/T) x_0 + (t/T) noise`` and the model regresses the velocity
``noise - x_0``.  Draws are uniform or logit-normal, kept ``1e-5`` inside ``(0, 1)``.  The shift maps
``f = t/T`` to ``s f / (1 + (s - 1) f)``; in ``dynamic`` mode ``s`` grows log-linearly with the pixel
area (256^2 -> 0.5, 1024^2 -> 1.15) and the frame count (1 -> 0, 121 -> 1.64) of each sample, scaled by
``rescale_factor`` and clamped to ``max_shift``.
"""
from __future__ import annotations

from enum import Enum
from typing import Optional

import torch


class TimestepDistribution(str, Enum):
    UNIFORM = "uniform"
    LOGNORM = "lognorm"


class TimestepShiftMode(str, Enum):
    FIXED = "fixed"
    DYNAMIC = "dynamic"


EDGE = 1e-5


def interpolate(clean: torch.Tensor, noise: torch.Tensor, t: torch.Tensor, dim: int = 0, *, T: int = 1000):
    """Point at time ``t`` on the straight path from ``clean`` to ``noise`` (``t`` broadcast on ``dim``)."""
    shape = [1] * clean.ndim
    shape[dim] = -1
    w = (t / T).view(shape)
    return (1 - w) * clean + w * noise


def draw_timesteps(count: int, device=None, generator: Optional[torch.Generator] = None, *,
                   distribution="lognorm", T: int = 1000, loc: float = 0.0, scale: float = 1.0,
                   default_device=None) -> torch.Tensor:
    device = device or default_device or "cpu"
    distribution = TimestepDistribution(distribution)
    if distribution is TimestepDistribution.UNIFORM:
        u = torch.rand((count,), device=device, generator=generator)
    else:
        z = torch.normal(mean=loc, std=scale, size=(count,), device=device, generator=generator)
        u = torch.sigmoid(z)
    return (u * (1 - 2 * EDGE) + EDGE) * T


def _line(x, p1, p2):
    (x1, y1), (x2, y2) = p1, p2
    k = (y2 - y1) / (x2 - x1)
    return k * x + (y1 - k * x1)


def shift_timesteps(timesteps: torch.Tensor, T: int, shift: float = 1.0, mode="fixed",
                    latent_shapes: Optional[torch.Tensor] = None, rescale_factor: float = 0.5,
                    max_shift: float = 1000.0, frame_stride: int = 4, pixel_stride_h: int = 16,
                    pixel_stride_w: Optional[int] = None) -> torch.Tensor:
    mode = TimestepShiftMode(mode)
    if mode is TimestepShiftMode.FIXED:
        s = shift
    else:
        if latent_shapes is None:
            raise ValueError("latent_shapes is required when train_timestep_shift_mode=dynamic")
        g = latent_shapes.to(device=timesteps.device, dtype=torch.float32)
        frames = (g[:, 0] - 1) * frame_stride + 1
        area = (g[:, 1] * pixel_stride_h) * (g[:, 2] * (pixel_stride_w or pixel_stride_h))
        log_s = _line(area, (256 * 256, 0.5), (1024 * 1024, 1.15)) + _line(frames, (1, 0.0), (121, 1.64))
        s = torch.exp(rescale_factor * log_s).clamp(max=max_shift)
    if isinstance(s, float) and s == 1.0:
        return timesteps
    f = timesteps / T
    return s * f / (1 + (s - 1) * f) * T
