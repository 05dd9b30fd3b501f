"""Rotary position embeddings over several coordinate axes (time, height, width).

Numerically the tables are those of the reference (pan/models/transformers/modules/rope.py:33-123):
the head dimension is cut into one slice per axis (``axes_dim``); within a slice of width ``w`` the
rotated pair ``k`` turns by ``coord * scale * theta ** -(2k / w)``, computed in fp32; ``cos`` and
``sin`` carry each pair's angle in both of its columns so that the pair ``(x[2k], x[2k + 1])``
rotates as ``(a, b) -> (a cos - b sin, b cos + a sin)``.  Text tokens rotate by nothing.

The organisation is this module's own: a :class:`RopePlan` fixes, per table column, which axis it
follows and its frequency; tables for a token grid or for explicit coordinates are one broadcast
product against that plan.  The fused QKV kernel (``csrc/qkv_ops.cu``) reads the same tables.
"""
from __future__ import annotations

from functools import lru_cache
from typing import Sequence, Tuple

import torch

Tables = Tuple[torch.Tensor, torch.Tensor]


def _one_per_axis(value, n_axes: int, what: str) -> list:
    """A scalar or a 1-sequence repeated for every axis, or a sequence with one value per axis."""
    values = [value] if isinstance(value, (int, float)) else list(value)
    if len(values) == 1:
        values = values * n_axes
    if len(values) != n_axes:
        raise ValueError(f"{what}: need 1 value or one per RoPE axis ({n_axes}); got {values}")
    return values


class RopePlan:
    """Which axis every rotated pair follows, and at what angular frequency."""

    def __init__(self, axes_dim: Sequence[int], theta: float, position_scale=1.0):
        self.axes_dim = tuple(int(d) for d in axes_dim)
        self.theta = float(theta)
        self.scales = _one_per_axis(position_scale, len(self.axes_dim), "position_scale")

    def _freqs(self, width: int, device) -> torch.Tensor:
        pairs = width // 2
        exponent = torch.arange(0, width, 2, device=device)[:pairs].float() / width
        return torch.pow(self.theta, exponent).reciprocal()

    def tables(self, coords: Sequence[torch.Tensor]) -> Tables:
        """``coords[a]``: fp32 coordinate of every token on axis ``a`` (length N each)."""
        cos_parts, sin_parts = [], []
        for axis, width in enumerate(self.axes_dim):
            at = coords[axis] * self.scales[axis]
            angle = at[:, None] * self._freqs(width, at.device)[None, :]   # [N, pairs]
            cos_parts.append(torch.repeat_interleave(angle.cos(), 2, dim=1))
            sin_parts.append(torch.repeat_interleave(angle.sin(), 2, dim=1))
        return torch.cat(cos_parts, dim=1), torch.cat(sin_parts, dim=1)


def _grid_coords(sizes: Sequence[int]) -> list:
    """fp32 coordinates of every cell of a row-major grid, one tensor per axis."""
    n = 1
    for s in sizes:
        n *= int(s)
    flat = torch.arange(n, device="cpu")
    coords, stride = [], n
    for s in sizes:
        stride //= int(s)
        coords.append(((flat // stride) % int(s)).to(torch.float32))
    return coords


@lru_cache(maxsize=64)
def rope_tables_for_grid(axes_dim: Sequence[int], grid_sizes, theta: float = 10000.0,
                         position_scale=1.0) -> Tables:
    """``(cos, sin)``, each ``[prod(grid), sum(axes_dim)]``, for a row-major (t, h, w) token grid.
    Cached: pass tuples."""
    plan = RopePlan(axes_dim, theta, position_scale)
    sizes = tuple(grid_sizes) if not isinstance(grid_sizes, int) else (grid_sizes,) * len(plan.axes_dim)
    if len(sizes) != len(plan.axes_dim):
        raise ValueError(f"grid of {len(sizes)} axes {sizes} for a RoPE plan of {len(plan.axes_dim)} axes")
    return plan.tables(_grid_coords(sizes))


def rope_tables_for_positions(axes_dim: Sequence[int], positions: torch.Tensor, theta: float = 10000.0,
                              position_scale=1.0) -> Tables:
    """``(cos, sin)`` for explicit coordinates ``positions`` of shape ``[N, len(axes_dim)]``."""
    plan = RopePlan(axes_dim, theta, position_scale)
    if positions.dim() != 2 or positions.shape[1] != len(plan.axes_dim):
        raise ValueError(f"positions must be [tokens, {len(plan.axes_dim)}]; got {list(positions.shape)}")
    pos = positions.to(torch.float32)
    return plan.tables([pos[:, a] for a in range(pos.shape[1])])


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """Every adjacent pair ``(a, b)`` of the last dim becomes ``(-b, a)``."""
    swapped = x.unflatten(-1, (x.shape[-1] // 2, 2)).flip(-1).clone()
    swapped[..., 0].neg_()
    return swapped.flatten(-2)


def _table_for(table: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """A ``[S, D]`` table gains a head axis to broadcast over ``[..., S, H, D]``; a table that already
    has one (``[S, 1, D]``) is used as it is."""
    table = table.to(x.device)
    if table.dim() != 2:
        return table
    if tuple(table.shape) != (x.shape[-3], x.shape[-1]):
        raise ValueError(f"RoPE table of shape {list(table.shape)} cannot rotate a tensor of shape {list(x.shape)}")
    return table[:, None, :]


def apply_rope(query: torch.Tensor, key: torch.Tensor, cos_sin: Tables) -> Tuple[torch.Tensor, torch.Tensor]:
    """Rotate ``[..., S, H, D]`` query and key in fp32; results keep the inputs' dtype."""
    cos = _table_for(cos_sin[0], query)
    sin = _table_for(cos_sin[1], query)
    out = []
    for t in (query, key):
        tf = t.to(torch.float32)
        out.append((tf * cos + rotate_half(tf) * sin).to(t.dtype))
    return out[0], out[1]
