"""Synthetic packed batches of the benchmark shapes (random latents / text embeddings).

Builds exactly what the packed dataloader hands the trainer (dataset/packed_dataloader.py:323-468 of
the reference): per clip a Wan-2.2-shaped latent ``[48, T, H, W]`` is noised along the rectified-flow
path at a logit-normal, shifted timestep; the model input is the channel concat
``[x_t (48), condition (48), mask (1)]`` patchified to ``[C*pt*ph*pw, N]``; the target is
``noise - latent``; captions are ``[n_text, 4096]`` embeddings; RoPE tables are in interleave layout
with identity rows for text.  All tensors are created on the CPU (pinned when requested).
"""
from __future__ import annotations

from typing import Dict, List, Sequence, Tuple

import torch

from ..diffusion.flow_matching import draw_timesteps, interpolate, shift_timesteps
from ..models.packed import build_packed_params
from .patching import packed_rope_tables, patchify


def synthetic_packed_batch(n_clips: int, latent_thw: Tuple[int, int, int], text_len: int, *,
                           image_cond_first: bool = True, **kw) -> Dict:
    """``n_clips`` clips of one latent shape; the first carries a first-frame condition."""
    items = [(tuple(latent_thw), image_cond_first and i == 0) for i in range(n_clips)]
    return synthetic_items_batch(items, [text_len] * n_clips, **kw)


def synthetic_items_batch(items: Sequence[Tuple[Tuple[int, int, int], bool]], text_lens: Sequence[int], *,
                          latent_channels: int = 48, patch_size=(1, 2, 2), text_dim: int = 4096,
                          rope_axes=(16, 56, 56), rope_theta: float = 256.0,
                          rope_scale=(16 / 24, 1.0, 1.0), pad_multiple: int = 128, shift: float = 9.0,
                          seed: int = 0, dtype=torch.bfloat16, pin: bool = False, T: int = 1000) -> Dict:
    """One packed batch of arbitrary items: ``items[i] = ((T, H, W) latent shape, first-frame
    condition)`` (single-frame items are images), each with ``text_lens[i]`` caption tokens."""
    g = torch.Generator().manual_seed(seed)
    pt, ph, pw = patch_size
    n = len(items)
    grids = [(t_lat // pt, h_lat // ph, w_lat // pw) for (t_lat, h_lat, w_lat), _ in items]
    vlen = [a * b * c for a, b, c in grids]
    clen = [int(x) for x in text_lens]
    n_active = sum(vlen) + sum(clen)
    total = (n_active + pad_multiple - 1) // pad_multiple * pad_multiple
    t = draw_timesteps(n, "cpu", g, distribution="lognorm", T=T)
    t = shift_timesteps(t, T, shift)
    inputs, targets = [], []
    for i, ((t_lat, h_lat, w_lat), cond_first) in enumerate(items):
        x0 = torch.randn(latent_channels, t_lat, h_lat, w_lat, generator=g)
        eps = torch.randn(latent_channels, t_lat, h_lat, w_lat, generator=g)
        xt = interpolate(x0.unsqueeze(0), eps.unsqueeze(0), t[i:i + 1], dim=0, T=T)[0]
        cond = torch.zeros_like(x0)
        mask = torch.zeros(1, t_lat, h_lat, w_lat)
        if cond_first:
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


def sft_mix_items(budget_video: int, budget_joint: int, max_seq: int, text_len: int, *, seed: int = 0,
                  hw: Tuple[int, int] = (44, 80), n_images: int = 4, max_frames: int = 61,
                  image_cond_prob: float = 0.3) -> List[Tuple[Tuple[int, int, int], bool]]:
    """A mixed image + video packing of the SFT shape class: ``n_images`` single-frame items, then
    videos of seeded random lengths (5..``max_frames`` latent frames) while the token budgets and
    the sequence limit allow; first-frame conditioning drawn with ``image_cond_prob``."""
    g = torch.Generator().manual_seed(seed)
    per_frame = (hw[0] // 2) * (hw[1] // 2)
    items: List[Tuple[Tuple[int, int, int], bool]] = [((1, hw[0], hw[1]), False) for _ in range(n_images)]
    video = per_frame * n_images
    while len(items) < max_seq:
        frames = int(torch.randint(5, max_frames + 1, (1,), generator=g))
        room = min(budget_video - video, budget_joint - video - text_len * (len(items) + 1)) // per_frame
        frames = min(frames, room)
        if frames < 5:
            break
        cond = bool(torch.rand(1, generator=g) < image_cond_prob)
        items.append(((frames, hw[0], hw[1]), cond))
        video += frames * per_frame
    return items


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
