"""Multi-axis rotary position embeddings.

Same tables as pan/models/transformers/modules/rope.py:33-123 of the reference: the head dim is split
into one slice per (t, h, w) axis (``axes_dim``), each rotated by that axis' coordinate times its
position scale; ``inv_freq = theta ** -(2i/dim)``; angles in fp32; ``cos``/``sin`` with every frequency
repeated twice so that they line up with adjacent ``(x[2i], x[2i+1])`` pairs, which rotate as
``(a, b) -> (a cos - b sin, b cos + a sin)``.  Text tokens get the identity (cos=1, sin=0).
"""
from __future__ import annotations

from functools import lru_cache
from typing import Sequence, Tuple

import torch


def _per_axis(value, ndim: int, name: str) -> list:
    if isinstance(value, (int, float)):
        return [value] * ndim
    value = list(value)
    if len(value) == 1:
        return value * ndim
    if len(value) != ndim:
        raise ValueError(f"{name} must be a scalar or have one entry per axis ({ndim}), got {value}")
    return value


def _axis_tables(dim: int, positions: torch.Tensor, theta: float, scale: float):
    inv_freq = 1.0 / (theta ** (torch.arange(0, dim, 2, device=positions.device)[: dim // 2].float() / dim))
    angles = torch.outer(positions * scale, inv_freq)
    return angles.cos().repeat_interleave(2, dim=1), angles.sin().repeat_interleave(2, dim=1)


def _tables(axes_dim, coords, theta, position_scale):
    scales = _per_axis(position_scale, len(axes_dim), "position_scale")
    parts = [_axis_tables(d, coords[a], theta, scales[a]) for a, d in enumerate(axes_dim)]
    return torch.cat([c for c, _ in parts], dim=1), torch.cat([s for _, s in parts], dim=1)


@lru_cache(maxsize=64)
def rope_tables_for_grid(axes_dim: Sequence[int], grid_sizes, theta: float = 10000.0,
                         position_scale=1.0) -> Tuple[torch.Tensor, torch.Tensor]:
    """``(cos, sin)`` of shape ``[prod(grid), sum(axes_dim)]`` for a row-major (t, h, w) grid."""
    axes_dim = tuple(axes_dim)
    sizes = (grid_sizes,) * len(axes_dim) if isinstance(grid_sizes, int) else tuple(grid_sizes)
    if len(sizes) != len(axes_dim):
        raise ValueError(f"grid_sizes {sizes} must have one entry per rope axis ({len(axes_dim)})")
    axes = torch.meshgrid(*[torch.arange(n, dtype=torch.float32) for n in sizes], indexing="ij")
    return _tables(axes_dim, [a.reshape(-1) for a in axes], theta, position_scale)


def rope_tables_for_positions(axes_dim: Sequence[int], positions: torch.Tensor, theta: float = 10000.0,
                              position_scale=1.0) -> Tuple[torch.Tensor, torch.Tensor]:
    """``(cos, sin)`` from explicit ``[N, len(axes_dim)]`` coordinates."""
    axes_dim = tuple(axes_dim)
    if positions.ndim != 2 or positions.size(1) != len(axes_dim):
        raise ValueError(f"Expected positions with shape [N, {len(axes_dim)}], got {tuple(positions.shape)}")
    positions = positions.float()
    return _tables(axes_dim, [positions[:, a] for a in range(len(axes_dim))], theta, position_scale)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """Adjacent pairs ``(a, b) -> (-b, a)`` along the last dim."""
    pairs = x.unflatten(-1, (-1, 2))
    return torch.stack((-pairs[..., 1], pairs[..., 0]), dim=-1).flatten(-2)


def _broadcast(table: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    table = table.to(x.device)
    if table.ndim == 2:
        if table.shape != (x.shape[-3], x.shape[-1]):
            raise ValueError(f"RoPE table {tuple(table.shape)} does not match x {tuple(x.shape)}")
        return table.unsqueeze(1)
    return table


def apply_rope(query: torch.Tensor, key: torch.Tensor, cos_sin) -> Tuple[torch.Tensor, torch.Tensor]:
    """Rotate ``[..., S, H, D]`` query/key in fp32 and cast back."""
    cos, sin = (_broadcast(t, query) for t in cos_sin)

    def rotate(x):
        xf = x.float()
        return (xf * cos + rotate_half(xf) * sin).type_as(x)

    return rotate(query), rotate(key)
