"""Synthetic packed batches of the benchmark shapes (random latents / text embeddings).

Builds exactly what the packed dataloader hands the trainer (dataset/packed_dataloader.py:323-468 of
the reference): per clip a Wan-2.2-shaped latent ``[48, T, H, W]`` is noised along the rectified-flow
path at a logit-normal, shifted timestep; the model input is the channel concat
``[x_t (48), condition (48), mask (1)]`` patchified to ``[C*pt*ph*pw, N]``; the target is
``noise - latent``; captions are ``[n_text, 4096]`` embeddings; RoPE tables are in interleave layout
with identity rows for text.  All tensors are created on the CPU (pinned when requested).
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

import torch

from ..diffusion.flow_matching import draw_timesteps, interpolate, shift_timesteps
from ..models.packed import build_packed_params
from .patching import packed_rope_tables, patchify


def synthetic_packed_batch(n_clips: int, latent_thw: Tuple[int, int, int], text_len: int, *,
                           latent_channels: int = 48, patch_size=(1, 2, 2), text_dim: int = 4096,
                           rope_axes=(16, 56, 56), rope_theta: float = 256.0,
                           rope_scale=(16 / 24, 1.0, 1.0), pad_multiple: int = 128, shift: float = 9.0,
                           image_cond_first: bool = True, seed: int = 0, dtype=torch.bfloat16,
                           pin: bool = False, T: int = 1000) -> Dict:
    g = torch.Generator().manual_seed(seed)
    t_lat, h_lat, w_lat = latent_thw
    pt, ph, pw = patch_size
    grids = [(t_lat // pt, h_lat // ph, w_lat // pw)] * n_clips
    vlen = [a * b * c for a, b, c in grids]
    clen = [text_len] * n_clips
    n_active = sum(vlen) + sum(clen)
    total = (n_active + pad_multiple - 1) // pad_multiple * pad_multiple
    t = draw_timesteps(n_clips, "cpu", g, distribution="lognorm", T=T)
    t = shift_timesteps(t, T, shift)
    inputs, targets = [], []
    for i in range(n_clips):
        x0 = torch.randn(latent_channels, t_lat, h_lat, w_lat, generator=g)
        eps = torch.randn(latent_channels, t_lat, h_lat, w_lat, generator=g)
        xt = interpolate(x0.unsqueeze(0), eps.unsqueeze(0), t[i:i + 1], dim=0, T=T)[0]
        cond = torch.zeros_like(x0)
        mask = torch.zeros(1, t_lat, h_lat, w_lat)
        if image_cond_first and i == 0:
            cond[:, :1] = x0[:, :1]
            mask[:, :1] = 1.0
        inp = torch.cat([xt, cond, mask], 0)
        inputs.append(patchify(inp, patch_size))
        targets.append(patchify(eps - x0, patch_size).t())
    hidden = torch.cat(inputs, 1).to(dtype)[:, :, None, None].contiguous()
    target = torch.cat(targets, 0).to(dtype).contiguous()
    text = torch.randn(sum(clen), text_dim, generator=g).to(dtype)
    cos, sin = packed_rope_tables(rope_axes, rope_theta, rope_scale, grids, clen, total)
    meta = build_packed_params(vlen, clen, total, cos, sin)
    batch = dict(hidden_states=hidden, timestep=t.float(), text_states=text, target=target,
                 packed_seq_params=meta)
    if pin:
        batch = pin_batch(batch)
    return batch


def pin_batch(batch: Dict) -> Dict:
    out = {}
    for k, v in batch.items():
        if isinstance(v, torch.Tensor):
            out[k] = v.pin_memory()
        elif k == "packed_seq_params":
            out[k] = v.to("cpu")
            for name, t in out[k].tensors().items():
                setattr(out[k], name, t.pin_memory())
        else:
            out[k] = v
    return out


def batch_to_device(batch: Dict, device, non_blocking: bool = True) -> Dict:
    out = {}
    for k, v in batch.items():
        if isinstance(v, torch.Tensor):
            out[k] = v.to(device, non_blocking=non_blocking)
        elif k == "packed_seq_params":
            out[k] = v.to(device, non_blocking=non_blocking)
        else:
            out[k] = v
    return out


def batch_bytes(batch: Dict) -> int:
    n = 0
    for k, v in batch.items():
        if isinstance(v, torch.Tensor):
            n += v.numel() * v.element_size()
        elif k == "packed_seq_params":
            n += sum(t.numel() * t.element_size() for t in v.tensors().values())
    return n
