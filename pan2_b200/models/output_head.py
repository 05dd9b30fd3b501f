"""Output head: adaLN-modulated affine-free LayerNorm and the projection back to latent patches.

Same parameters and math as pan/models/transformers/modules/output_head.py:21-62: ``norm`` is
``LayerNorm(eps=1e-6, affine=False)``, ``proj`` is ``Linear(hidden, prod(patch) * C_out)`` (Kaiming
normal, zero bias), ``modulation`` is an ``AdaLNProjection`` chunked as ``(shift, scale)`` — that order
is what the checkpoints store.  The packed path fuses the LayerNorm through ``ln_stats`` and projects
only the video rows.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from .layers import AdaLNProjection
from ..ops.gemm import linear
from ..ops.packed import ln_modulate


class OutputHead(nn.Module):
    def __init__(self, inner_dim, patch_size, out_channels, activation: str = "silu", zero_init_modulation: bool = True):
        super().__init__()
        patch_numel = patch_size * patch_size if isinstance(patch_size, int) else math.prod(patch_size)
        self.norm = nn.LayerNorm(inner_dim, elementwise_affine=False, eps=1e-6)
        self.proj = nn.Linear(inner_dim, patch_numel * out_channels, bias=True)
        nn.init.kaiming_normal_(self.proj.weight)
        nn.init.zeros_(self.proj.bias)
        self.modulation = AdaLNProjection(inner_dim, 2, activation, zero_init=zero_init_modulation)

    def modulation_rows(self, temb: torch.Tensor):
        a = self.modulation.act(temb)
        shift, scale = linear(a, self.modulation.linear.weight, self.modulation.linear.bias).chunk(2, dim=1)
        return shift, scale

    def forward(self, hidden_states, temb):
        """Dense path: ``[B, N, hidden]`` -> ``[B, N, prod(patch) * C_out]``."""
        shift, scale = self.modulation_rows(temb)
        h = self.norm(hidden_states.float()).to(hidden_states.dtype)
        h = h * (1 + scale)[:, None, :].to(h.dtype) + shift[:, None, :].to(h.dtype)
        return linear(h, self.proj.weight, self.proj.bias)

    def forward_packed(self, x, temb, ln_stats, video_bounds, n_video):
        """Packed path: LayerNorm fused via ``ln_stats``, per-video modulation, video rows only."""
        shift, scale = self.modulation_rows(temb)
        # modulate only the video rows; text / padding rows are outside the segments
        h = ln_modulate(x, ln_stats, shift.to(x.dtype), scale.to(x.dtype), video_bounds)
        return linear(h[:n_video], self.proj.weight, self.proj.bias)
