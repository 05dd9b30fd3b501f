"""Caption encoder (token refiner): pre-norm self-attention blocks over the projected captions.

Parameter names, shapes and creation order match the reference's caption encoder
(pan/models/transformers/modules/caption_encoder.py:30-153), so checkpoints load and seeded
initialisation matches: ``attn_norm`` -> bias-free fused ``qkv`` -> per-head ``q_norm`` / ``k_norm``
-> attention -> ``attn_out``, then ``ffn_norm`` -> SwiGLU ``w2(w3(x) * silu(w1(x)))``.

Captions run packed (``cu_seqlens`` and host ``lens``: the varlen tcgen05 attention) or padded
(``mask`` ``[B, L]``; the first position of every caption stays visible so an all-padding caption
still has a key).
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
    """Bias-free SwiGLU ``w2(w3(x) * silu(w1(x)))`` (``w1``, ``w3``, ``w2`` created in that order)."""

    def __init__(self, dim: int, inner_dim: int):
        super().__init__()
        self.w1 = nn.Linear(dim, inner_dim, bias=False)
        self.w3 = nn.Linear(dim, inner_dim, bias=False)
        self.w2 = nn.Linear(inner_dim, dim, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        value = linear(x, self.w3.weight)
        return linear(value * F.silu(linear(x, self.w1.weight)), self.w2.weight)


def reinit_branch_output(layer: nn.Linear, zero: bool, std: Optional[float]) -> None:
    """Re-initialise a residual branch's output projection: normal with ``std`` when given, zero
    when ``zero``; left as constructed otherwise.  A bias, if any, becomes zero."""
    if std is None and not zero:
        return
    if std is not None and not std >= 0:
        raise ValueError(f"residual_init_std={std} is negative")
    with torch.no_grad():
        if std is None:
            layer.weight.zero_()
        else:
            layer.weight.normal_(0.0, std)
        if layer.bias is not None:
            layer.bias.zero_()


class CaptionEncoderBlock(nn.Module):
    def __init__(self, *, dim: int, num_attention_heads: int, mlp_ratio: float = 4.0, qk_norm: bool = True,
                 eps: float = 1e-5, zero_residual_init: bool = False, residual_init_std: Optional[float] = None):
        super().__init__()
        self.heads = num_attention_heads
        d_head = dim // num_attention_heads
        norm_or_id = (lambda: RMSNorm(d_head, eps=eps)) if qk_norm else nn.Identity
        self.attn_norm = RMSNorm(dim, eps=eps)
        self.qkv = nn.Linear(dim, 3 * dim, bias=False)
        self.qkv.weight._muon_chunks_dim_0 = 3 * num_attention_heads  # Muon: a row block per (q|k|v, head)
        self.q_norm = norm_or_id()
        self.k_norm = norm_or_id()
        self.attn_out = nn.Linear(dim, dim, bias=False)
        self.ffn_norm = RMSNorm(dim, eps=eps)
        self.ffn = SwiGLUFeedForward(dim, int(dim * mlp_ratio))
        for out in (self.attn_out, self.ffn.w2):
            reinit_branch_output(out, zero_residual_init, residual_init_std)

    def forward(self, x, attention_mask=None, cu_seqlens=None, lens=None, max_seqlen=None):
        packed = cu_seqlens is not None
        if packed and attention_mask is not None:
            raise ValueError("a caption batch is packed (cu_seqlens) or padded (attention_mask), not both")
        h = self.attn_norm(x)
        q, k, v = linear(h, self.qkv.weight).unflatten(-1, (3, self.heads, -1)).unbind(-3)
        q = self.q_norm(q).to(v.dtype)
        k = self.k_norm(k).to(v.dtype)
        o = varlen_attention(q, k, v, cu_seqlens, lens, max_seqlen) if packed else dense_attention(q, k, v,
                                                                                                  attention_mask)
        x = x + linear(o.flatten(-2), self.attn_out.weight)
        return x + self.ffn(self.ffn_norm(x))


class CaptionEncoder(nn.Module):
    def __init__(self, dim: int, num_attention_heads: int, num_layers: int = 4, **block_kwargs):
        super().__init__()
        self.blocks = nn.ModuleList(CaptionEncoderBlock(dim=dim, num_attention_heads=num_attention_heads,
                                                        **block_kwargs) for _ in range(num_layers))

    def forward(self, x, mask=None, cu_seqlens=None, lens: Optional[Sequence[int]] = None, max_seqlen=None):
        if mask is not None:
            mask = mask.bool().clone()
            mask[:, 0] = True  # every caption keeps one visible key
        for block in self.blocks:
            x = block(x, attention_mask=mask, cu_seqlens=cu_seqlens, lens=lens, max_seqlen=max_seqlen)
        return x
