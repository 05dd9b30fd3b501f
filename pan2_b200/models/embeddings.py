"""Input embeddings: the video patch embedding and the timestep encoder.

Parameter names, shapes and initialisation match the reference
(pan/models/transformers/modules/embeddings.py:26-127) so checkpoints interchange:

* ``VideoPatchEmbed.proj`` is a stride-equals-kernel ``Conv3d``, Xavier-uniform over its flattened
  ``[inner_dim, C*pt*ph*pw]`` weight, zero bias.  The packed path receives patches already cut by
  the loader (``[C*pt*ph*pw, N, 1, 1]``) and applies the conv as the equivalent linear map.
* ``TimestepEncoder``: the sinusoidal ``cos || sin`` embedding of ``t * exp(-ln(max_period) i / half)``
  over 256 channels, then ``in_proj -> SiLU -> out_proj``.

The sinusoid frequencies must be the fp32 values computed on the CPU (a low-precision or GPU copy puts
a phase error on the fast channels).  Here ``forward`` never reads the stored ``freqs`` buffer: it
takes the table from :func:`sinusoid_frequencies`, cached per device.  The buffer is kept only so
state dicts carry the reference's ``timestep_encoder.freqs`` key; hooks write the exact fp32 table
into every state dict produced and replace whatever a loaded state dict holds there.
"""
from __future__ import annotations

import math
from functools import lru_cache

import torch
import torch.nn as nn
import torch.nn.functional as F


def patch_triple(patch_size) -> tuple:
    """``(t, h, w)`` patch size from an int or a 3-sequence."""
    dims = (patch_size,) * 3 if isinstance(patch_size, int) else tuple(int(p) for p in patch_size)
    if len(dims) != 3:
        raise ValueError(f"patch_size {patch_size!r}: give one int or three (t, h, w)")
    return dims


class VideoPatchEmbed(nn.Module):
    """Video latents -> tokens: dense ``[B, C, T, H, W]`` or packed ``[C*pt*ph*pw, N, 1, 1]`` input."""

    def __init__(self, patch_size, in_channels: int, inner_dim: int):
        super().__init__()
        self.patch_size = patch_triple(patch_size)
        self.proj = nn.Conv3d(in_channels, inner_dim, kernel_size=self.patch_size, stride=self.patch_size)
        nn.init.xavier_uniform_(self.proj.weight.view(inner_dim, -1))
        nn.init.zeros_(self.proj.bias)

    def forward(self, hidden_states: torch.Tensor, packed: bool = False) -> torch.Tensor:
        if not packed:
            return self.proj(hidden_states).flatten(2).transpose(1, 2)
        rows = hidden_states.flatten(1).t()  # [N, C*pt*ph*pw]
        w = self.proj.weight.flatten(1).to(rows.dtype)
        return F.linear(rows, w, self.proj.bias.to(rows.dtype))


@lru_cache(maxsize=32)
def _cpu_frequencies(channels: int, max_period: float) -> torch.Tensor:
    half = channels // 2
    steps = torch.arange(half, dtype=torch.float32, device="cpu") * -math.log(max_period)
    return torch.exp(steps / half)


def sinusoid_frequencies(channels: int = 256, max_period: float = 10000.0, device=None) -> torch.Tensor:
    """``exp(-ln(max_period) * i / half)``, ``i < half``, evaluated in fp32 on the CPU."""
    table = _cpu_frequencies(int(channels), float(max_period))
    return table if device is None else table.to(device)


def timestep_embedding(timesteps: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """``cos(t f) || sin(t f)`` for every timestep."""
    phase = torch.outer(timesteps.float(), freqs.to(timesteps.device))
    return torch.cat((phase.cos(), phase.sin()), dim=-1)


class TimestepEncoder(nn.Module):
    """Timesteps -> sinusoidal embedding -> ``in_proj -> act -> out_proj``."""

    def __init__(self, time_embed_dim: int, activation: str = "silu", num_channels: int = 256,
                 max_period: int = 10000):
        super().__init__()
        from .layers import make_activation
        self.num_channels, self.max_period = num_channels, max_period
        self.register_buffer("freqs", sinusoid_frequencies(num_channels, max_period).clone().to(
            torch.empty(0).device))  # the module's construction device (meta under a meta context)
        self.in_proj = nn.Linear(num_channels, time_embed_dim)
        self.act = make_activation(activation)
        self.out_proj = nn.Linear(time_embed_dim, time_embed_dim)
        nn.init.normal_(self.in_proj.weight, std=0.02)
        nn.init.normal_(self.out_proj.weight, std=0.02)
        self._register_state_dict_hook(TimestepEncoder._exact_on_save)
        self._register_load_state_dict_pre_hook(self._exact_on_load)

    @staticmethod
    def _exact_on_save(module, state_dict, prefix, local_metadata):
        key = prefix + "freqs"
        if key in state_dict:
            state_dict[key] = sinusoid_frequencies(module.num_channels, module.max_period, state_dict[key].device)
        return state_dict

    def _exact_on_load(self, state_dict, prefix, *args):
        key = prefix + "freqs"
        if isinstance(state_dict.get(key), torch.Tensor) and state_dict[key].shape == self.freqs.shape:
            state_dict[key] = sinusoid_frequencies(self.num_channels, self.max_period, state_dict[key].device)

    def forward(self, timestep: torch.Tensor) -> torch.Tensor:
        from ..ops.gemm import linear
        table = sinusoid_frequencies(self.num_channels, self.max_period, timestep.device)
        emb = timestep_embedding(timestep, table).to(self.in_proj.weight.dtype)
        h = self.act(linear(emb, self.in_proj.weight, self.in_proj.bias))
        return linear(h, self.out_proj.weight, self.out_proj.bias)
