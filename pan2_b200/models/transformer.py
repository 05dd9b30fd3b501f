"""PAN 2 video MMDiT: patch embed, caption path, timestep encoder, joint blocks, output head.

Parameter names, shapes and initialisers are those of the reference
(pan/models/transformers/pan_transformer.py:34-1019), so state dicts and DCP checkpoints are
interchangeable (the reference's key map is in scripts/convert_checkpoint.py:55-105).  Two forwards:

* packed training (``forward(..., packed_seq_params=..., target=...)``) returns the flow-matching
  loss numerator/denominator pair over the packed batch (the caller averages across ranks);
* dense inference (``forward(latents[B,C,T,H,W], t[B], text[B,L,C], text_mask)``) returns the
  velocity ``[B, C_out, T, H, W]``.

The joint block's packed forward (``JointAttentionBlock.forward_packed``) runs on the fused ops of
:mod:`pan2_b200.ops`: LN-modulate, grouped QKV with RMS+RoPE+permute, varlen attention, grouped
out-projection, gate+residual with ``ln_stats``, grouped GELU FFN.
"""
from __future__ import annotations

import logging
import math
from typing import Any, Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F
from einops import rearrange

from .layers import RMSNorm, AdaLNProjection, rms_norm
from .embeddings import TimestepEncoder, VideoPatchEmbed
from .rope import apply_rope, rope_tables_for_grid
from .output_head import OutputHead
from .caption_encoder import CaptionEncoder
from .packed import PackedSequenceParams
from ..ops import packed as P
from ..ops.gemm import linear, grouped_linear, grouped_ffn
from ..ops.qkv import qkv_project
from ..ops.attention import varlen_attention, dense_attention
from ..parallel.ulysses import ulysses_attention
from ..parallel.cp_fused import fused_cp_enabled, fused_qkv_ulysses_attention

log = logging.getLogger(__name__)


# ---------------------------------------------------------------------------------------------
# parameter holders (same names / layout as the reference)
# ---------------------------------------------------------------------------------------------

def linear_default_init(weight: torch.Tensor, bias: Optional[torch.Tensor], fan_in: int) -> None:
    """torch's default ``nn.Linear`` initialisation for a (slice of a) stacked weight: uniform with
    bound ``1/sqrt(fan_in)`` (the Kaiming-uniform rule with a = sqrt(5)) for both weight and bias."""
    nn.init.kaiming_uniform_(weight, a=math.sqrt(5))
    if bias is not None:
        limit = fan_in ** -0.5
        with torch.no_grad():
            bias.uniform_(-limit, limit)


class GroupedQKVProj(nn.Module):
    """Video+text QKV stacked ``[2*3H, H]`` (each modality block is ``[Q|K|V]``), bias ``[2*3H]``,
    head-dim RMS affines ``q_weight``/``k_weight`` ``[2*D]`` (pan_transformer.py:34-127)."""

    def __init__(self, hidden_size: int, num_heads: int, qk_norm: bool = True, qk_norm_type: str = "rms",
                 eps: float = 1e-6):
        super().__init__()
        if not qk_norm or qk_norm_type != "rms":
            raise ValueError("GroupedQKVProj requires qk_norm=True with rms norm")
        self.hidden_size, self.num_heads = hidden_size, num_heads
        self.head_dim = hidden_size // num_heads
        self.eps = eps
        self.weight = nn.Parameter(torch.empty(2 * hidden_size * 3, hidden_size))
        self.bias = nn.Parameter(torch.empty(2 * hidden_size * 3))
        self.q_weight = nn.Parameter(torch.ones(2 * self.head_dim))
        self.k_weight = nn.Parameter(torch.ones(2 * self.head_dim))
        self.weight._muon_chunks_dim_0 = num_heads * 2 * 3
        self.reset_parameters()

    def reset_parameters(self):
        linear_default_init(self.weight, self.bias, self.hidden_size)
        with torch.no_grad():
            for w in (self.q_weight, self.k_weight):
                w.fill_(1.0)

    def project(self, x: torch.Tensor, modality: str):
        """Dense path: one modality's ``q, k, v`` ``[..., H, D]`` with RMS q/k norm (no RoPE)."""
        h3, d = 3 * self.hidden_size, self.head_dim
        g = {"video": 0, "text": 1}[modality]
        w, b = self.weight[g * h3:(g + 1) * h3], self.bias[g * h3:(g + 1) * h3]
        qw, kw = self.q_weight[g * d:(g + 1) * d], self.k_weight[g * d:(g + 1) * d]
        q, k, v = rearrange(linear(x, w, b), "... (K H D) -> K ... H D", K=3, H=self.num_heads).unbind(0)
        q = rms_norm(q, qw.to(q.dtype), self.eps).to(v.dtype)
        k = rms_norm(k, kw.to(k.dtype), self.eps).to(v.dtype)
        return q, k, v


class GroupedOutProj(nn.Module):
    """Video+text attention output projection ``[2H, H]`` + bias ``[2H]`` (pan_transformer.py:130-169)."""

    def __init__(self, hidden_size: int):
        super().__init__()
        self.hidden_size = hidden_size
        self.weight = nn.Parameter(torch.empty(2 * hidden_size, hidden_size))
        self.bias = nn.Parameter(torch.empty(2 * hidden_size))
        self.weight._muon_chunks_dim_0 = 2
        self.reset_parameters()

    def reset_parameters(self):
        linear_default_init(self.weight, self.bias, self.hidden_size)

    def project(self, x: torch.Tensor, modality: str) -> torch.Tensor:
        h = self.hidden_size
        g = {"video": 0, "text": 1}[modality]
        return linear(x, self.weight[g * h:(g + 1) * h], self.bias[g * h:(g + 1) * h])


class GroupedFFN(nn.Module):
    """Per-modality GELU-tanh MLPs (video ``mlp_ratio``, text ``context_mlp_ratio``)."""

    def __init__(self, hidden_size: int, video_mlp_hidden_dim: int, text_mlp_hidden_dim: int,
                 mlp_act_type: str = "gelu_tanh"):
        super().__init__()
        if mlp_act_type != "gelu_tanh":
            raise ValueError("GroupedFFN only supports the gelu_tanh MLP")
        if video_mlp_hidden_dim < text_mlp_hidden_dim:
            raise ValueError("GroupedFFN requires video_mlp_hidden_dim >= text_mlp_hidden_dim")
        self.hidden_size = hidden_size
        self.w_up_video = nn.Parameter(torch.empty(video_mlp_hidden_dim, hidden_size))
        self.b_up_video = nn.Parameter(torch.empty(video_mlp_hidden_dim))
        self.w_down_video = nn.Parameter(torch.empty(hidden_size, video_mlp_hidden_dim))
        self.b_down_video = nn.Parameter(torch.empty(hidden_size))
        self.w_up_text = nn.Parameter(torch.empty(text_mlp_hidden_dim, hidden_size))
        self.b_up_text = nn.Parameter(torch.empty(text_mlp_hidden_dim))
        self.w_down_text = nn.Parameter(torch.empty(hidden_size, text_mlp_hidden_dim))
        self.b_down_text = nn.Parameter(torch.empty(hidden_size))
        self.reset_parameters()

    def reset_parameters(self):
        p = self.params_grouped()  # (weight, bias) pairs in creation order
        for w, b in zip(p[0::2], p[1::2]):
            linear_default_init(w, b, w.shape[1])

    def params_grouped(self):
        return [self.w_up_video, self.b_up_video, self.w_down_video, self.b_down_video,
                self.w_up_text, self.b_up_text, self.w_down_text, self.b_down_text]

    def project(self, x: torch.Tensor, modality: str) -> torch.Tensor:
        if modality == "video":
            h = F.gelu(linear(x, self.w_up_video, self.b_up_video), approximate="tanh")
            return linear(h, self.w_down_video, self.b_down_video)
        h = F.gelu(linear(x, self.w_up_text, self.b_up_text), approximate="tanh")
        return linear(h, self.w_down_text, self.b_down_text)


class JointAttentionBlock(nn.Module):
    """Joint video+text attention block with per-modality projections (pan_transformer.py:250-619)."""

    def __init__(self, hidden_size: int, num_heads: int, *, attention_backend: Optional[str] = None,
                 normalize_qk: bool = True, qk_norm_kind: str = "rms", ffn_activation: str = "gelu_tanh",
                 mlp_ratio: float = 8.0, context_mlp_ratio: float = 4.0, zero_init_modulation: bool = True,
                 text_modulation_timestep_dependent: bool = False):
        super().__init__()
        self.attention_backend = attention_backend
        self.hidden_size, self.num_heads = hidden_size, num_heads
        self.mlp_hidden_dim = int(hidden_size * mlp_ratio)
        self.text_mlp_hidden_dim = int(hidden_size * context_mlp_ratio)
        # creation order fixes the initializer RNG stream
        self.qkv_proj = GroupedQKVProj(hidden_size, num_heads, qk_norm=normalize_qk, qk_norm_type=qk_norm_kind)
        self.out_proj = GroupedOutProj(hidden_size)
        self.pre_norm = nn.LayerNorm(hidden_size, elementwise_affine=False, eps=1e-6)
        self.modulation = AdaLNProjection(hidden_size, 6, "silu", zero_init=zero_init_modulation)
        self.norm2 = nn.LayerNorm(hidden_size, elementwise_affine=False, eps=1e-6)
        self.ffn = GroupedFFN(hidden_size, self.mlp_hidden_dim, self.text_mlp_hidden_dim, mlp_act_type=ffn_activation)
        self.text_modulation_timestep_dependent = text_modulation_timestep_dependent
        if text_modulation_timestep_dependent:
            self.text_modulation = AdaLNProjection(hidden_size, 6, "silu", zero_init=zero_init_modulation)
        else:
            self.text_modulation = nn.Parameter(torch.empty(hidden_size * 6))
            if zero_init_modulation:
                nn.init.zeros_(self.text_modulation)
            else:
                nn.init.uniform_(self.text_modulation, -hidden_size ** -0.5, hidden_size ** -0.5)

    # -- legacy checkpoint keys (pan_transformer.py:319-409) --------------------------------
    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys,
                              unexpected_keys, error_msgs):
        from ..checkpoint.keys import convert_legacy_block_keys
        convert_legacy_block_keys(state_dict, prefix, self.text_modulation_timestep_dependent,
                                  None if not self.text_modulation_timestep_dependent
                                  else self.text_modulation.linear.weight.shape)
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys,
                                      unexpected_keys, error_msgs)

    def modulation_rows(self, vec: torch.Tensor, video_mod: Optional[torch.Tensor] = None) -> torch.Tensor:
        """``[k+1, 6H]``: one row per video sample then the shared text row.  ``video_mod`` supplies
        the video rows when they were computed elsewhere (the peer-memory AdaLN projection)."""
        if video_mod is None:
            a = self.modulation.act(vec)
            video_mod = linear(a, self.modulation.linear.weight, self.modulation.linear.bias)
        text_mod = self.text_modulation.unsqueeze(0).to(video_mod.dtype)
        return torch.cat([video_mod, text_mod], dim=0)

    def forward_packed(self, x: torch.Tensor, ln_stats: torch.Tensor, vec: torch.Tensor,
                       meta: PackedSequenceParams, attn_fn=None,
                       video_mod: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Packed training forward over the concat layout; returns ``(x, ln_stats)``."""
        if self.text_modulation_timestep_dependent:
            raise ValueError("packed JointAttentionBlock assumes timestep-independent text modulation")
        bounds = meta.concat_bounds
        bt = getattr(meta, "_bounds_dev", None)
        mods = self.modulation_rows(vec, video_mod).to(x.dtype)
        shift1, scale1, gate1, shift2, scale2, gate2 = mods.chunk(6, dim=-1)
        x_mod = P.ln_modulate(x, ln_stats, shift1, scale1, bounds, bt)
        mm_bounds = [0, meta.n_video, meta.n_active]
        qkv_w = self.qkv_proj.weight.view(2, 3 * self.hidden_size, self.hidden_size)
        qkv_b = self.qkv_proj.bias.view(2, 3 * self.hidden_size)
        if attn_fn is None and meta.cp_group is not None and fused_cp_enabled(meta.cp_group, x.device):
            # Ulysses all-to-alls folded into qkv_post / attention (peer memory, one node)
            o_concat = fused_qkv_ulysses_attention(x_mod, qkv_w, qkv_b, self.qkv_proj.q_weight,
                                                   self.qkv_proj.k_weight, meta, mm_bounds, self.num_heads,
                                                   self.qkv_proj.eps)
        else:
            q, k, v = qkv_project(x_mod, qkv_w, qkv_b, self.qkv_proj.q_weight, self.qkv_proj.k_weight,
                                  meta.freqs_cos, meta.freqs_sin, meta.indices_interleave_to_concat, mm_bounds,
                                  self.num_heads, self.qkv_proj.eps)
            if attn_fn is None and meta.cp_group is not None:
                o = ulysses_attention(q, k, v, meta)
            elif attn_fn is None:
                o = varlen_attention(q, k, v, meta.joint_cu_seqlens, meta.joint_lens, meta.joint_segment_limit)
            else:
                o = attn_fn(q, k, v, meta)
            o_concat = P.permute_rows(o.reshape(o.shape[0], -1), meta.indices_interleave_to_concat,
                                      meta.indices_concat_to_interleave)
        h = self.hidden_size
        attn_out = grouped_linear(o_concat, self.out_proj.weight.view(2, h, h), self.out_proj.bias.view(2, h),
                                  mm_bounds)
        x, ln_stats = P.gate_residual(attn_out, gate1, x, bounds, bt)
        x_ffn = P.ln_modulate(x, ln_stats, shift2, scale2, bounds, bt)
        ffn_out = grouped_ffn(x_ffn, mm_bounds, self.ffn.params_grouped())
        x, ln_stats = P.gate_residual(ffn_out, gate2, x, bounds, bt)
        return x, ln_stats

    def forward_dense(self, x: torch.Tensor, vec: torch.Tensor, txt_len: int, freqs_cis,
                      text_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Unpacked inference forward over ``[B, N_video + N_text, H]``."""
        vm = linear(self.modulation.act(vec), self.modulation.linear.weight, self.modulation.linear.bias)
        v_shift1, v_scale1, v_gate1, v_shift2, v_scale2, v_gate2 = vm.chunk(6, dim=-1)
        if self.text_modulation_timestep_dependent:
            tm = self.text_modulation(vec)
        else:
            tm = self.text_modulation.unsqueeze(0).expand(vec.shape[0], -1)
        tm = tm.to(x.dtype)
        t_shift1, t_scale1, t_gate1, t_shift2, t_scale2, t_gate2 = tm.chunk(6, dim=-1)
        img, txt = x[:, :-txt_len], x[:, -txt_len:]

        def ln_mod(t, shift, scale):
            n = F.layer_norm(t.float(), (t.shape[-1],), eps=1e-6)
            return (n * (1 + scale.unsqueeze(1).float()) + shift.unsqueeze(1).float()).to(t.dtype)

        img_q, img_k, img_v = self.qkv_proj.project(ln_mod(img, v_shift1, v_scale1), "video")
        txt_q, txt_k, txt_v = self.qkv_proj.project(ln_mod(txt, t_shift1, t_scale1), "text")
        n_vid = img_q.shape[1]
        img_q, img_k = apply_rope(img_q, img_k, (freqs_cis[0][:n_vid], freqs_cis[1][:n_vid]))
        if freqs_cis[0].shape[0] > n_vid:
            txt_q, txt_k = apply_rope(txt_q, txt_k, (freqs_cis[0][n_vid:], freqs_cis[1][n_vid:]))
        q = torch.cat([img_q, txt_q], 1)
        k = torch.cat([img_k, txt_k], 1)
        v = torch.cat([img_v, txt_v], 1)
        mask = None
        if text_mask is not None:
            mask = F.pad(text_mask.bool(), (n_vid, 0), value=True)
        attn = dense_attention(q, k, v, mask).flatten(2)
        img_a, txt_a = attn[:, :n_vid], attn[:, n_vid:]
        img = img + self.out_proj.project(img_a, "video") * v_gate1.unsqueeze(1).to(img.dtype)
        txt = txt + self.out_proj.project(txt_a, "text") * t_gate1.unsqueeze(1).to(txt.dtype)
        img = img + self.ffn.project(ln_mod(img, v_shift2, v_scale2), "video") * v_gate2.unsqueeze(1).to(img.dtype)
        txt = txt + self.ffn.project(ln_mod(txt, t_shift2, t_scale2), "text") * t_gate2.unsqueeze(1).to(txt.dtype)
        return torch.cat([img, txt], dim=1)


class TextTypeEmbedding(nn.Module):
    """Learned vector added to every caption token, stored as row 0 of a ``(3, width)`` weight."""

    def __init__(self, width: int):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(3, width))

    @property
    def vector(self) -> torch.Tensor:
        return self.weight[0]


# legacy architecture key names -> constructor arguments (pan_transformer.py:671-720)
# Architecture keys of configs written before the reference renamed them.  Each rule is one of
#   ("rename", new_name)          the value moves to the constructor argument new_name
#   ("only", value)               the key had one legal value; it is checked and dropped
#   ("ffn_ratio", target or None) legacy FFN width ratios: video / text default to mlp_width_ratio (4)
_LEGACY_RULES: Dict[str, tuple] = {
    "heads_num": ("rename", "num_attention_heads"),
    "mm_single_blocks_depth": ("rename", "num_layers"),
    "mlp_act_type": ("rename", "ffn_activation"),
    "text_states_dim": ("rename", "text_embed_dim"),
    "rope_dim_list": ("rename", "rope_axes_dim"),
    "rope_t_interp": ("rename", "rope_temporal_scale"),
    "use_cond_type_embedding": ("rename", "use_text_type_embedding"),
    "qk_norm": ("rename", "normalize_qk"),
    "qk_norm_type": ("rename", "qk_norm_kind"),
    "attn_mode": ("rename", "attention_backend"),
    "use_attention_mask": ("rename", "mask_text_padding"),
    "mm_double_blocks_depth": ("only", 0),
    "single_stream_block_type": ("only", "mm_joint_attn"),
    "mlp_width_ratio": ("ffn_ratio", None),
    "video_mlp_width_ratio": ("ffn_ratio", "mlp_ratio"),
    "text_mlp_width_ratio": ("ffn_ratio", "context_mlp_ratio"),
}


def translate_architecture_config(config) -> dict:
    """Constructor arguments from an architecture config that may use the legacy key names (current
    names pass through unchanged)."""
    given = dict(config)
    out = {k: v for k, v in given.items() if k not in _LEGACY_RULES}
    ratios = {}
    for key in (k for k in given if k in _LEGACY_RULES):
        kind, arg = _LEGACY_RULES[key]
        value = given[key]
        if kind == "only":
            if value != arg:
                raise ValueError(f"legacy architecture key {key}={value!r}: only {arg!r} is supported")
        elif kind == "rename":
            if arg in given:
                raise ValueError(f"architecture config gives both the legacy {key!r} and its current name {arg!r}")
            out[arg] = value
        else:
            ratios[key] = value
    if ratios:
        base = ratios.get("mlp_width_ratio", 4.0)
        for key in ("video_mlp_width_ratio", "text_mlp_width_ratio"):
            target = _LEGACY_RULES[key][1]
            if target in given:
                raise ValueError(f"architecture config gives both legacy FFN ratios and {target!r}")
            out[target] = base if ratios.get(key) is None else ratios[key]
    renamed = sorted(k for k in given if k in _LEGACY_RULES)
    if renamed:
        log.warning(f"architecture config: legacy keys {renamed} mapped to the current names")
    return out


ARCH_DEFAULTS: Dict[str, Any] = dict(
    patch_size=(1, 2, 2), in_channels=97, out_channels=48, hidden_size=4096, num_attention_heads=32,
    num_layers=44, mlp_ratio=8.0, context_mlp_ratio=4.0, ffn_activation="gelu_tanh", attention_backend="flash",
    mask_text_padding=True, normalize_qk=True, qk_norm_kind="rms", rope_axes_dim=(16, 56, 56), rope_theta=256,
    rope_temporal_scale=16 / 24, text_embed_dim=4096, use_text_type_embedding=True, zero_init_modulation=True,
    text_modulation_timestep_dependent=False,
)


class PanVideoDiffusionTransformer(nn.Module):
    """PAN 2 video diffusion transformer (defaults: the released 29B model)."""

    def __init__(self, patch_size=(1, 2, 2), in_channels=97, out_channels=48, hidden_size=4096,
                 num_attention_heads=32, num_layers=44, mlp_ratio=8.0, context_mlp_ratio=4.0,
                 ffn_activation="gelu_tanh", attention_backend="flash", mask_text_padding=True, normalize_qk=True,
                 qk_norm_kind="rms", rope_axes_dim=(16, 56, 56), rope_theta=256, rope_temporal_scale=16 / 24,
                 text_embed_dim=4096, use_text_type_embedding=True, zero_init_modulation=True,
                 text_modulation_timestep_dependent=False, caption_encoder_layers: int = 4):
        super().__init__()
        head_dim, leftover = divmod(hidden_size, num_attention_heads)
        if leftover:
            raise ValueError(f"{num_attention_heads} attention heads do not split a hidden size of {hidden_size} evenly")
        if len(rope_axes_dim) != 3 or sum(rope_axes_dim) != head_dim:
            raise ValueError(f"rope_axes_dim {rope_axes_dim} needs three entries summing to the head dim {head_dim}")
        self.config = dict(patch_size=list(patch_size), in_channels=in_channels, out_channels=out_channels,
                           hidden_size=hidden_size, num_attention_heads=num_attention_heads, num_layers=num_layers,
                           mlp_ratio=mlp_ratio, context_mlp_ratio=context_mlp_ratio, ffn_activation=ffn_activation,
                           attention_backend=attention_backend, mask_text_padding=mask_text_padding,
                           normalize_qk=normalize_qk, qk_norm_kind=qk_norm_kind, rope_axes_dim=list(rope_axes_dim),
                           rope_theta=rope_theta, rope_temporal_scale=rope_temporal_scale,
                           text_embed_dim=text_embed_dim, use_text_type_embedding=use_text_type_embedding,
                           zero_init_modulation=zero_init_modulation,
                           text_modulation_timestep_dependent=text_modulation_timestep_dependent)
        self.patch_size = list(patch_size)
        self.in_channels = in_channels
        self.out_channels = out_channels if out_channels is not None else in_channels
        self.hidden_size, self.num_attention_heads = hidden_size, num_attention_heads
        self.head_dim = head_dim
        self.rope_axes_dim, self.rope_theta, self.rope_temporal_scale = list(rope_axes_dim), rope_theta, rope_temporal_scale
        self.attention_backend, self.mask_text_padding = attention_backend, mask_text_padding
        self.text_embed_dim = text_embed_dim
        self.text_modulation_timestep_dependent = text_modulation_timestep_dependent
        # construction order = parameter / initializer order
        self.patch_embed = VideoPatchEmbed(self.patch_size, in_channels, hidden_size)
        self.cap_embedder = nn.Sequential(RMSNorm(text_embed_dim, eps=1e-5), nn.Linear(text_embed_dim, hidden_size))
        self.caption_encoder = CaptionEncoder(hidden_size, num_attention_heads, num_layers=caption_encoder_layers)
        self.timestep_encoder = TimestepEncoder(hidden_size, "silu")
        opts = dict(attention_backend=attention_backend, normalize_qk=normalize_qk, qk_norm_kind=qk_norm_kind,
                    ffn_activation=ffn_activation, mlp_ratio=mlp_ratio, context_mlp_ratio=context_mlp_ratio,
                    zero_init_modulation=zero_init_modulation,
                    text_modulation_timestep_dependent=text_modulation_timestep_dependent)
        self.blocks = nn.ModuleList([JointAttentionBlock(hidden_size, num_attention_heads, **opts)
                                     for _ in range(num_layers)])
        self.output_head = OutputHead(hidden_size, self.patch_size, self.out_channels, "silu",
                                      zero_init_modulation=zero_init_modulation)
        self.text_type_embedding = TextTypeEmbedding(hidden_size) if use_text_type_embedding else None

    @classmethod
    def from_config(cls, config: Optional[dict] = None, **kwargs):
        arch = translate_architecture_config({k: v for k, v in dict(config or {}).items() if not k.startswith("_")})
        arch.update(kwargs)
        return cls(**arch)

    # ------------------------------------------------------------------ rope
    def rope_settings(self):
        axes_dim = tuple(self.rope_axes_dim)
        return axes_dim, self.rope_theta, (float(self.rope_temporal_scale),) + (1.0,) * (len(axes_dim) - 1)

    def rope_tables(self, grid):
        axes_dim, theta, scale = self.rope_settings()
        return rope_tables_for_grid(axes_dim, tuple(grid), theta=theta, position_scale=scale)

    # ------------------------------------------------------------------ packed (training)
    def embed_packed(self, hidden_states, timestep, text_states, meta: PackedSequenceParams):
        """Everything before the joint blocks: returns ``(x, ln_stats, vec)``."""
        vec = self.timestep_encoder(timestep)
        vec = vec.to(hidden_states.dtype) if hidden_states.is_floating_point() else vec
        txt = linear(rms_norm(text_states, self.cap_embedder[0].weight.to(text_states.dtype), self.cap_embedder[0].eps),
                     self.cap_embedder[1].weight, self.cap_embedder[1].bias)
        cap_lens = meta.cp_caption_lens if meta.cp_caption_lens is not None else meta.caption_lens
        txt = self.caption_encoder(txt, cu_seqlens=meta.caption_cu_seqlens, lens=cap_lens,
                                   max_seqlen=meta.caption_segment_limit)
        if meta.cp_text_index is not None:
            txt = txt.index_select(0, meta.cp_text_index)
        vid = self.patch_embed_packed(hidden_states)
        ttv = None if self.text_type_embedding is None else self.text_type_embedding.vector
        x, ln_stats = P.simple_concat(vid, txt.to(vid.dtype), meta.joint_packed_length, ttv)
        return x, ln_stats, vec

    def patch_embed_packed(self, hidden_states):
        patches = hidden_states.reshape(hidden_states.shape[0], -1).t()
        w = self.patch_embed.proj.weight.flatten(1)
        return linear(patches.contiguous(), w, self.patch_embed.proj.bias)

    def head_and_loss(self, x, ln_stats, vec, target, meta: PackedSequenceParams):
        """Output head over the video rows + the MSE numerator/denominator ``[2]``."""
        pred = self.output_head.forward_packed(x, vec, ln_stats, [0] + _cumsum(meta.video_lens), meta.n_video)
        return P.concat_mse_sums(pred, target, meta.n_video)

    def predict_packed(self, hidden_states, timestep, text_states, meta: PackedSequenceParams,
                       skip_layers: Sequence[int] = ()) -> torch.Tensor:
        """Inference over a packed batch: velocity rows ``[n_video, prod(patch) * C_out]`` for the video
        tokens (concat order).  ``skip_layers`` drops joint blocks (the STG weak prediction)."""
        x, ln_stats, vec = self.embed_packed(hidden_states, timestep, text_states, meta)
        order = [i for i in range(len(self.blocks)) if i not in skip_layers]
        streamer = getattr(self, "block_streamer", None)  # set when the blocks live in host memory
        blocks = streamer.run(self.blocks, order) if streamer is not None else ((i, self.blocks[i]) for i in order)
        for _, block in blocks:
            x, ln_stats = block.forward_packed(x, ln_stats, vec, meta)
        return self.output_head.forward_packed(x, vec, ln_stats, [0] + _cumsum(meta.video_lens), meta.n_video)

    def forward(self, hidden_states: torch.Tensor, timestep: torch.Tensor, text_states: torch.Tensor,
                text_mask: Optional[torch.Tensor] = None, freqs_cos=None, freqs_sin=None,
                packed_seq_params: Optional[PackedSequenceParams] = None, target: Optional[torch.Tensor] = None,
                stg_skip_layers: Optional[Sequence[int]] = None, **unused):
        if packed_seq_params is not None:
            if stg_skip_layers is not None:
                raise ValueError("STG supports only the unpacked forward, not packed training")
            if text_mask is not None:
                raise ValueError("Packed mode requires text_mask=None")
            meta = packed_seq_params
            x, ln_stats, vec = self.embed_packed(hidden_states, timestep, text_states, meta)
            for block in self.blocks:
                x, ln_stats = block.forward_packed(x, ln_stats, vec, meta)
            sums = self.head_and_loss(x, ln_stats, vec, target, meta)
            return sums[0] / sums[1]
        return self.forward_dense(hidden_states, timestep, text_states, text_mask, freqs_cos, freqs_sin,
                                  stg_skip_layers)

    # ------------------------------------------------------------------ dense (inference)
    def validate_stg_layers(self, stg_skip_layers):
        """Block indices that the skip-guidance (weak) forward leaves out, checked; () when off."""
        if stg_skip_layers is None:
            return ()
        layers = stg_skip_layers
        n = len(self.blocks)
        problems = []
        if not isinstance(layers, (list, tuple)) or len(layers) == 0:
            problems.append("give a non-empty list of block indices")
        else:
            if not all(type(i) is int for i in layers):
                problems.append("indices must be plain ints")
            elif len(set(layers)) < len(layers):
                problems.append("an index repeats")
            elif min(layers) < 0 or max(layers) >= n:
                problems.append(f"indices must lie in 0..{n - 1}")
        if not problems and (self.training or torch.is_grad_enabled()):
            problems.append("skip guidance is an inference feature: call eval() and run under no_grad")
        if problems:
            raise ValueError(f"stg_skip_layers={stg_skip_layers!r}: " + "; ".join(problems))
        return tuple(layers)

    def encode_text(self, text_states, text_mask):
        mask = text_mask if self.mask_text_padding else None
        t = linear(rms_norm(text_states, self.cap_embedder[0].weight.to(text_states.dtype), self.cap_embedder[0].eps),
                   self.cap_embedder[1].weight, self.cap_embedder[1].bias)
        t = self.caption_encoder(t, mask=mask)
        if self.text_type_embedding is not None:
            t = t + self.text_type_embedding.vector.to(t.dtype)
        return t

    def forward_dense(self, latents, timestep, text_states, text_mask=None, freqs_cos=None, freqs_sin=None,
                      stg_skip_layers=None, block_hook=None):
        """Velocity ``[B, C_out, T, H, W]`` for dense latents ``[B, C_in, T, H, W]``."""
        skip = self.validate_stg_layers(stg_skip_layers) if stg_skip_layers is not None else ()
        grid = tuple(s // p for s, p in zip(latents.shape[2:], self.patch_size))
        rope = self.rope_tables(grid) if freqs_cos is None else (freqs_cos, freqs_sin)
        dtype = latents.dtype
        pt, ph, pw = self.patch_size
        patches = rearrange(latents, "b c (t pt) (h ph) (w pw) -> b (t h w) (c pt ph pw)", pt=pt, ph=ph, pw=pw)
        video = linear(patches, self.patch_embed.proj.weight.flatten(1), self.patch_embed.proj.bias).to(dtype)
        temb = self.timestep_encoder(timestep).to(dtype)
        text = self.encode_text(text_states.to(dtype), text_mask).to(dtype)
        hidden, n_video = torch.cat((video, text), dim=1), video.shape[1]
        rope = (rope[0].to(latents.device), rope[1].to(latents.device))
        for index, block in enumerate(self.blocks):
            if index in skip:
                continue
            hidden = block.forward_dense(hidden, temb, text.shape[1], rope, text_mask)
            if block_hook is not None:
                block_hook(index)
        out = self.output_head(hidden[:, :n_video], temb)
        return self.unpatchify(out, *grid), None

    def unpatchify(self, tokens, t, h, w):
        if tokens.shape[1] != t * h * w:
            raise ValueError(f"expected {t * h * w} tokens for grid {(t, h, w)}, got {tokens.shape[1]}")
        pt, ph, pw = self.patch_size
        return rearrange(tokens, "n (t h w) (c pt ph pw) -> n c (t pt) (h ph) (w pw)",
                         t=t, h=h, w=w, c=self.out_channels, pt=pt, ph=ph, pw=pw)


def _cumsum(xs):
    out, s = [], 0
    for x in xs:
        s += int(x)
        out.append(s)
    return out
