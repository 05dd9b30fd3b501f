"""State-dict key conversions: legacy per-modality block keys -> the grouped layout.

Same mapping as the reference's ``JointAttentionBlock._convert_grouped_state_dict`` /
``_load_from_state_dict`` (pan/models/transformers/pan_transformer.py:288-409): separate video/text
``linear1_qkv``/``q_norm``/``attn_out``/``ffn`` tensors are stacked video-first into
``qkv_proj``/``out_proj``/``ffn.*``, and an old ``text_modulation.linear`` projection of a learned
``text_empty_embedding`` is folded into the direct ``text_modulation`` vector.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F


def convert_legacy_block_keys(state_dict: dict, prefix: str, text_modulation_timestep_dependent: bool,
                              text_linear_weight_shape: Optional[torch.Size] = None) -> None:
    P = prefix

    def stack(new, old_v, old_t):
        if P + new not in state_dict and P + old_v in state_dict:
            state_dict[P + new] = torch.cat([state_dict.pop(P + old_v), state_dict.pop(P + old_t)], dim=0)

    stack("qkv_proj.weight", "linear1_qkv.weight", "text_linear1_qkv.weight")
    stack("qkv_proj.bias", "linear1_qkv.bias", "text_linear1_qkv.bias")
    stack("qkv_proj.q_weight", "q_norm.weight", "text_q_norm.weight")
    stack("qkv_proj.k_weight", "k_norm.weight", "text_k_norm.weight")
    stack("out_proj.weight", "attn_out.weight", "text_attn_out.weight")
    stack("out_proj.bias", "attn_out.bias", "text_attn_out.bias")
    if P + "ffn.w_up_video" not in state_dict and P + "ffn.0.weight" in state_dict:
        for new, old in (("ffn.w_up_video", "ffn.0.weight"), ("ffn.b_up_video", "ffn.0.bias"),
                         ("ffn.w_down_video", "ffn.2.weight"), ("ffn.b_down_video", "ffn.2.bias"),
                         ("ffn.w_up_text", "text_ffn.0.weight"), ("ffn.b_up_text", "text_ffn.0.bias"),
                         ("ffn.w_down_text", "text_ffn.2.weight"), ("ffn.b_down_text", "text_ffn.2.bias")):
            state_dict[P + new] = state_dict.pop(P + old)

    direct = P + "text_modulation"
    lin_b, lin_w, empty = P + "text_modulation.linear.bias", P + "text_modulation.linear.weight", P + "text_empty_embedding"
    if text_modulation_timestep_dependent:
        if lin_b not in state_dict and direct in state_dict:
            conv = state_dict.pop(direct)
            state_dict[lin_b] = conv
            state_dict[lin_w] = torch.zeros(text_linear_weight_shape, device=conv.device, dtype=conv.dtype)
        state_dict.pop(empty, None)
    else:
        if direct not in state_dict and lin_b in state_dict:
            conv = state_dict[lin_b]
            if lin_w in state_dict and empty in state_dict:
                w = state_dict[lin_w]
                e = F.silu(state_dict[empty].to(device=w.device, dtype=w.dtype))
                conv = torch.matmul(w, e) + conv.to(device=w.device, dtype=w.dtype)
            state_dict[direct] = conv
        for k in (lin_b, lin_w, empty):
            state_dict.pop(k, None)
