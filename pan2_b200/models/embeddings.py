"""Input embeddings: the video patch embedding and the timestep encoder.

Behaviour follows pan/models/transformers/modules/embeddings.py:26-127 of the reference:

* ``VideoPatchEmbed`` is a stride == kernel ``Conv3d``; on the packed path the dataloader has already
  cut samples into flat ``[C*pt*ph*pw, N, 1, 1]`` patches and the conv weight is applied as the
  equivalent linear map (embeddings.py:51-55).  Xavier-uniform over the flattened weight, zero bias.
* ``TimestepEncoder``: sinusoidal ``cos || sin`` embedding of ``t * exp(-ln(max_period) * i / half)``,
  ``num_channels=256``; then ``in_proj -> SiLU -> out_proj``.  The frequency table is a persistent
  buffer that is always rebuilt in fp32 on the CPU (embeddings.py:96-121), never trusted from a
  low-precision copy.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F


def patch_triple(patch_size) -> tuple:
    if isinstance(patch_size, int):
        return (patch_size, patch_size, patch_size)
    patch_size = tuple(int(p) for p in patch_size)
    if len(patch_size) != 3:
        raise ValueError(f"patch_size must be an int or a (t, h, w) triple, got {patch_size}")
    return patch_size


class VideoPatchEmbed(nn.Module):
    """Video latents -> tokens (dense ``[B,C,T,H,W]`` or packed ``[C*pt*ph*pw, N, 1, 1]`` input)."""

    def __init__(self, patch_size, in_channels: int, inner_dim: int):
        super().__init__()
        self.patch_size = patch_triple(patch_size)
        self.proj = nn.Conv3d(in_channels, inner_dim, kernel_size=self.patch_size, stride=self.patch_size)
        nn.init.xavier_uniform_(self.proj.weight.view(inner_dim, -1))
        nn.init.zeros_(self.proj.bias)

    def forward(self, hidden_states: torch.Tensor, packed: bool = False) -> torch.Tensor:
        if packed:
            patches = hidden_states.reshape(hidden_states.shape[0], -1).transpose(0, 1)  # [N, C*pt*ph*pw]
            return F.linear(patches, self.proj.weight.flatten(1).to(patches.dtype),
                            self.proj.bias.to(patches.dtype))
        out = self.proj(hidden_states)
        return out.flatten(2).transpose(1, 2)


def timestep_frequencies(num_channels: int = 256, max_period: float = 10000.0) -> torch.Tensor:
    """fp32 CPU frequency table ``exp(-ln(max_period) * i / half)`` for ``i < half``."""
    half = num_channels // 2
    exponent = -math.log(max_period) * torch.arange(0, half, dtype=torch.float32, device="cpu") / half
    return torch.exp(exponent)


def timestep_embedding(timesteps: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """Sinusoidal embedding ordered ``cos`` then ``sin``."""
    angles = timesteps[:, None].float() * freqs[None, :].to(timesteps.device)
    return torch.cat([torch.cos(angles), torch.sin(angles)], dim=-1)


class TimestepEncoder(nn.Module):
    """Timesteps -> sinusoidal embedding -> ``in_proj -> act -> out_proj``."""

    def __init__(self, time_embed_dim: int, make_act, num_channels: int = 256, max_period: int = 10000):
        super().__init__()
        self.num_channels = num_channels
        self.max_period = max_period
        self.register_buffer("freqs", timestep_frequencies(num_channels, max_period))
        self.in_proj = nn.Linear(num_channels, time_embed_dim)
        self.act = make_act()
        self.out_proj = nn.Linear(time_embed_dim, time_embed_dim)
        nn.init.normal_(self.in_proj.weight, std=0.02)
        nn.init.normal_(self.out_proj.weight, std=0.02)

    def _rebuild_freqs(self):
        device = self.freqs.device
        if device.type == "meta":
            return
        self.freqs = timestep_frequencies(self.num_channels, self.max_period).to(device)

    def _apply(self, fn, recurse=True):
        super()._apply(fn, recurse=recurse)
        self._rebuild_freqs()
        return self

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict,
                              missing_keys, unexpected_keys, error_msgs):
        key = prefix + "freqs"
        saved = state_dict.get(key)
        if isinstance(saved, torch.Tensor) and saved.shape == self.freqs.shape:
            state_dict = dict(state_dict)
            state_dict[key] = timestep_frequencies(self.num_channels, self.max_period).to(saved.device)
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict,
                                      missing_keys, unexpected_keys, error_msgs)
        self._rebuild_freqs()

    def forward(self, timestep: torch.Tensor) -> torch.Tensor:
        from ..ops.gemm import linear
        sample = timestep_embedding(timestep, self.freqs).to(self.in_proj.weight.dtype)
        h = self.act(linear(sample, self.in_proj.weight, self.in_proj.bias))
        return linear(h, self.out_proj.weight, self.out_proj.bias)
