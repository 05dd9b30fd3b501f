"""Caption encoder ("token refiner"): pre-norm self-attention blocks over the projected captions.

Same structure and parameter names as pan/models/transformers/modules/caption_encoder.py:30-153:
``attn_norm`` RMSNorm(1e-5) -> bias-free fused ``qkv`` -> per-head ``q_norm``/``k_norm`` RMSNorm ->
attention -> ``attn_out``; then ``ffn_norm`` -> SwiGLU ``w2(w3(x) * silu(w1(x)))``.  Captions run either
packed (``cu_seqlens`` + host ``lens``) or padded (``mask`` ``[B, L]``; position 0 is always visible).
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from .layers import RMSNorm
from ..ops.attention import dense_attention, varlen_attention
from ..ops.gemm import linear


class SwiGLUFeedForward(nn.Module):
    """Bias-free SwiGLU: ``w2(w3(x) * silu(w1(x)))``."""

    def __init__(self, dim: int, inner_dim: int):
        super().__init__()
        self.w1 = nn.Linear(dim, inner_dim, bias=False)
        self.w3 = nn.Linear(dim, inner_dim, bias=False)
        self.w2 = nn.Linear(inner_dim, dim, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        gate = F.silu(linear(x, self.w1.weight))
        return linear(linear(x, self.w3.weight) * gate, self.w2.weight)


def _init_residual_output(layer: nn.Linear, zero_init: bool, init_std: Optional[float]) -> None:
    if init_std is not None and init_std < 0:
        raise ValueError(f"residual init std must be non-negative, got {init_std}")
    if init_std is None and not zero_init:
        return
    if init_std is None:
        nn.init.zeros_(layer.weight)
    else:
        nn.init.normal_(layer.weight, mean=0.0, std=init_std)
    if layer.bias is not None:
        nn.init.zeros_(layer.bias)


class CaptionEncoderBlock(nn.Module):
    def __init__(self, *, dim: int, num_attention_heads: int, mlp_ratio: float = 4.0, qk_norm: bool = True,
                 eps: float = 1e-5, zero_residual_init: bool = False, residual_init_std: Optional[float] = None):
        super().__init__()
        self.heads = num_attention_heads
        head_dim = dim // num_attention_heads
        # attribute order = parameter / initializer order
        self.attn_norm = RMSNorm(dim, eps=eps)
        self.qkv = nn.Linear(dim, 3 * dim, bias=False)
        self.qkv.weight._muon_chunks_dim_0 = 3 * num_attention_heads
        self.q_norm = RMSNorm(head_dim, eps=eps) if qk_norm else nn.Identity()
        self.k_norm = RMSNorm(head_dim, eps=eps) if qk_norm else nn.Identity()
        self.attn_out = nn.Linear(dim, dim, bias=False)
        self.ffn_norm = RMSNorm(dim, eps=eps)
        self.ffn = SwiGLUFeedForward(dim, int(dim * mlp_ratio))
        _init_residual_output(self.attn_out, zero_residual_init, residual_init_std)
        _init_residual_output(self.ffn.w2, zero_residual_init, residual_init_std)

    def attention(self, x, mask=None, cu_seqlens=None, lens=None, max_seqlen=None):
        q, k, v = linear(x, self.qkv.weight).chunk(3, dim=-1)
        q, k, v = (t.unflatten(-1, (self.heads, -1)) for t in (q, k, v))
        q = self.q_norm(q).to(v.dtype)
        k = self.k_norm(k).to(v.dtype)
        if cu_seqlens is None:
            o = dense_attention(q, k, v, mask)
        else:
            o = varlen_attention(q, k, v, cu_seqlens, lens, max_seqlen)
        return linear(o.flatten(-2), self.attn_out.weight)

    def forward(self, x, attention_mask=None, cu_seqlens=None, lens=None, max_seqlen=None):
        if cu_seqlens is not None and attention_mask is not None:
            raise ValueError("Pass either attention_mask (padded) or cu_seqlens (packed), not both")
        x = x + self.attention(self.attn_norm(x), attention_mask, cu_seqlens, lens, max_seqlen)
        x = x + self.ffn(self.ffn_norm(x))
        return x


class CaptionEncoder(nn.Module):
    def __init__(self, dim: int, num_attention_heads: int, num_layers: int = 4, **block_kwargs):
        super().__init__()
        self.blocks = nn.ModuleList([CaptionEncoderBlock(dim=dim, num_attention_heads=num_attention_heads, **block_kwargs)
                                     for _ in range(num_layers)])

    def forward(self, x, mask=None, cu_seqlens=None, lens: Optional[Sequence[int]] = None, max_seqlen=None):
        if mask is not None:
            mask = mask.bool() | (torch.arange(mask.shape[1], device=mask.device) == 0)
        for block in self.blocks:
            x = block(x, attention_mask=mask, cu_seqlens=cu_seqlens, lens=lens, max_seqlen=max_seqlen)
        return x
