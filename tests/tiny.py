"""Tiny-model fixtures shared by the tests (2 blocks, hidden 256, two packed 48x5x8x8 videos)."""
from __future__ import annotations

import torch

from pan2_b200.models.transformer import PanVideoDiffusionTransformer
from pan2_b200.models.packed import build_packed_params
from pan2_b200.data.patching import patchify, packed_rope_tables

TINY_ARCH = dict(patch_size=(1, 2, 2), in_channels=97, out_channels=48, hidden_size=256, num_attention_heads=4,
                 num_layers=2, mlp_ratio=8.0, context_mlp_ratio=4.0, rope_axes_dim=(16, 24, 24), rope_theta=256,
                 rope_temporal_scale=16 / 24, text_embed_dim=4096, zero_init_modulation=False)


def tiny_model(seed=0, **over):
    torch.manual_seed(seed)
    arch = dict(TINY_ARCH)
    arch.update(over)
    return PanVideoDiffusionTransformer(**arch)


def tiny_batch(model, n_samples=2, frames=5, hw=8, text_len=32, pad=7, seed=1, dtype=torch.float32):
    """Packed batch of ``n_samples`` videos ``[97, frames, hw, hw]`` + captions; returns dict + dense views."""
    g = torch.Generator().manual_seed(seed)
    C = model.in_channels
    lat = [torch.randn(C, frames, hw, hw, generator=g) for _ in range(n_samples)]
    text = [torch.randn(text_len, model.text_embed_dim, generator=g) for _ in range(n_samples)]
    target_lat = [torch.randn(model.out_channels, frames, hw, hw, generator=g) for _ in range(n_samples)]
    t = torch.rand(n_samples, generator=g) * 1000
    ps = model.patch_size
    grids = [(frames // ps[0], hw // ps[1], hw // ps[2])] * n_samples
    vlen = [a * b * c for a, b, c in grids]
    clen = [text_len] * n_samples
    total = sum(vlen) + sum(clen) + pad
    axes, theta, scale = model.rope_settings()
    cos, sin = packed_rope_tables(axes, theta, scale, grids, clen, total)
    meta = build_packed_params(vlen, clen, total, cos, sin)
    hidden = torch.cat([patchify(x, ps) for x in lat], dim=1)[:, :, None, None]
    target = torch.cat([patchify(x, ps).t() for x in target_lat], dim=0)
    batch = dict(hidden_states=hidden.to(dtype), timestep=t, text_states=torch.cat(text, 0).to(dtype),
                 packed_seq_params=meta, target=target.to(dtype))
    dense = dict(latents=torch.stack(lat).to(dtype), timestep=t, text=torch.stack(text).to(dtype),
                 target=torch.stack(target_lat).to(dtype))
    return batch, dense
