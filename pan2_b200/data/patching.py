"""Patchify / RoPE-table helpers shared by the packed dataloader, the model tests and the sampler.

Token order is (t, h, w) row-major and each token's features are laid out (C, pt, ph, pw), the order
of the reference's ``VideoPatchEmbed`` / ``unpatchify`` (pan/models/transformers/pan_transformer.py:1007-1019)
and its packed dataloader (dataset/packed_dataloader.py:420-440).  Caption tokens get the identity
rotation (cos = 1, sin = 0), as in dataset/packing_dataset.py:439-442.
"""
from __future__ import annotations

from typing import Sequence, Tuple

import torch
from einops import rearrange

from ..models.rope import rope_tables_for_grid


def patchify(latent: torch.Tensor, patch_size: Sequence[int]) -> torch.Tensor:
    """``[C, T, H, W]`` -> ``[C*pt*ph*pw, N]`` flat patches (one column per token)."""
    pt, ph, pw = patch_size
    return rearrange(latent, "c (t pt) (h ph) (w pw) -> (c pt ph pw) (t h w)", pt=pt, ph=ph, pw=pw)


def unpatchify(tokens: torch.Tensor, grid: Sequence[int], patch_size: Sequence[int], channels: int) -> torch.Tensor:
    """``[N, C*pt*ph*pw]`` -> ``[C, T, H, W]``."""
    t, h, w = grid
    pt, ph, pw = patch_size
    return rearrange(tokens, "(t h w) (c pt ph pw) -> c (t pt) (h ph) (w pw)", t=t, h=h, w=w, c=channels,
                     pt=pt, ph=ph, pw=pw)


def packed_rope_tables(axes_dim, theta, position_scale, grids: Sequence[Tuple[int, int, int]],
                       caption_lens: Sequence[int], total: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Interleave-layout ``(cos, sin)`` ``[total, D]`` fp32: per sample its video grid, then identity rows."""
    D = sum(axes_dim)
    cos = torch.ones(total, D, dtype=torch.float32)
    sin = torch.zeros(total, D, dtype=torch.float32)
    pos = 0
    for grid, nt in zip(grids, caption_lens):
        c, s = rope_tables_for_grid(tuple(axes_dim), tuple(grid), theta=theta, position_scale=position_scale)
        n = c.shape[0]
        cos[pos:pos + n] = c
        sin[pos:pos + n] = s
        pos += n + int(nt)
    return cos, sin
