"""Packed varlen forward of the Qwen3.5 caption encoder.

The captions of a batch run as ONE token sequence ``[T]`` with boundaries ``cu_seqlens``: every
projection and MLP GEMM sees exactly the real tokens (no padding rows), and each caption behaves as
if it had been encoded alone:

* positions restart at 0 in every caption (text-only multimodal RoPE: the three position axes are
  equal, so the interleaved sections reduce to one rotary table over the caption position);
* full-attention layers attend causally within their caption only;
* the GatedDeltaNet (linear-attention) layers reset both their causal depthwise convolution and
  their recurrent state at every caption start.

The reference gets the same behaviour from its pinned transformers / flash-attention stack by
passing ``position_ids``, ``cu_seq_lens_*`` and a per-token ``seq_idx`` into the Hugging Face model
(``dataset/packed_dataloader.py:225-244``, ``dataset/packing_dataset.py:227-232,390-420``,
``pan/models/text_encoders/__init__.py:143-200``).  The transformers release in this environment
runs Qwen3.5's linear-attention layers without sequence boundaries, so this module drives the
loaded model's own weights and sub-modules (embedding, norms, projections, MLP) and supplies the
two sequence-aware parts itself:

Gated delta rule (Yang, Kautz, Hatamizadeh, "Gated Delta Networks", 2024).  Per head, with
l2-normalised ``q, k`` (``q`` also scaled by ``d_k^-1/2``), ``beta = sigmoid(b)`` and log-decay
``g <= 0``, the state ``S`` (``d_k x d_v``) evolves token by token as
``S <- exp(g) S + k (beta (v - exp(g) S^T k))^T`` and the output is ``o = S^T q``.  Over a chunk of
``C`` tokens with cumulative log-decay ``G_i`` and entry state ``S0`` this unrolls to

    (I + A) U = beta v - (beta exp(G) k) S0,   A_ij = beta_i exp(G_i - G_j) k_i.k_j  (j < i)
    o_i      = exp(G_i) q_i S0 + sum_{j<=i} exp(G_i - G_j) (q_i.k_j) U_j
    S_exit   = exp(G_C) S0 + sum_j exp(G_C - G_j) k_j U_j^T

so one unit-lower-triangular solve per chunk (independent of ``S0``: ``U = W_v - W_k S0``) moves all
the intra-chunk work off the sequential path; only the chunk-to-chunk state hand-off is a loop.
Chunks never straddle two captions: every caption starts a new chunk, its last chunk is padded
with inert tokens (``k = v = 0, beta = 0, g = 0``), and the hand-off loop runs over the chunk
ordinal with all captions batched, starting each caption from a zero state.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Sequence

import torch
import torch.nn.functional as F

CHUNK = 64


@dataclass
class _Layout:
    """Token <-> chunk-grid maps of one packed batch."""
    pos: torch.Tensor            # [T] position of each token inside its caption
    lengths: List[int]
    grid_src: torch.Tensor       # [NC * C] token index feeding each grid slot (0 for pads)
    grid_valid: torch.Tensor     # [NC * C] bool
    by_ordinal: List[torch.Tensor]   # chunk ids holding the j-th chunk of some caption
    seg_of_ordinal: List[torch.Tensor]  # ... and the caption each of them belongs to
    n_chunks: int


def _layout(lengths: Sequence[int], chunk: int, device) -> _Layout:
    lengths = [int(n) for n in lengths]
    pos = torch.cat([torch.arange(n, dtype=torch.long) for n in lengths]) if lengths else torch.zeros(0, dtype=torch.long)
    src, valid, ordinals, segs = [], [], [], []
    start, cid = 0, 0
    for s, n in enumerate(lengths):
        nc = -(-n // chunk)
        for j in range(nc):
            a = start + j * chunk
            b = min(start + n, a + chunk)
            idx = torch.arange(a, a + chunk)
            src.append(torch.where(idx < b, idx, torch.zeros_like(idx)))
            valid.append(idx < b)
            while len(ordinals) <= j:
                ordinals.append([])
                segs.append([])
            ordinals[j].append(cid)
            segs[j].append(s)
            cid += 1
        start += n
    to = dict(device=device)
    return _Layout(
        pos=pos.to(**to), lengths=lengths,
        grid_src=(torch.cat(src) if src else torch.zeros(0, dtype=torch.long)).to(**to),
        grid_valid=(torch.cat(valid) if valid else torch.zeros(0, dtype=torch.bool)).to(**to),
        by_ordinal=[torch.tensor(o, dtype=torch.long, device=device) for o in ordinals],
        seg_of_ordinal=[torch.tensor(o, dtype=torch.long, device=device) for o in segs],
        n_chunks=cid)


def gated_delta_rule_packed(q, k, v, beta, g, lay: _Layout, chunk: int = CHUNK) -> torch.Tensor:
    """``q, k [T, H, dk]``, ``v [T, H, dv]``, ``beta, g [T, H]`` (any float dtype; computed in fp32)
    -> ``o [T, H, dv]`` fp32, the recurrence restarted at every caption of ``lay``."""
    T, H, dk = q.shape
    dv = v.shape[-1]
    NC, C = lay.n_chunks, chunk
    q = q.float() * torch.rsqrt((q.float() ** 2).sum(-1, keepdim=True) + 1e-6) * dk ** -0.5
    k = k.float() * torch.rsqrt((k.float() ** 2).sum(-1, keepdim=True) + 1e-6)
    m = lay.grid_valid.view(-1, 1)

    def grid(x):  # [T, H, ...] -> [NC, H, C, ...], pads zero
        flat = x.reshape(T, -1)[lay.grid_src] * m
        return flat.view(NC, C, H, -1).transpose(1, 2)

    qg, kg, vg = grid(q), grid(k), grid(v.float())
    bg, gg = grid(beta.float())[..., 0], grid(g.float())[..., 0]         # [NC, H, C]
    G = gg.cumsum(-1)
    ii = torch.arange(C, device=q.device)
    lower = ii.view(-1, 1) > ii.view(1, -1)
    lower_eq = ii.view(-1, 1) >= ii.view(1, -1)
    diff = G.unsqueeze(-1) - G.unsqueeze(-2)                              # G_i - G_j
    dec = torch.exp(diff.masked_fill(~lower_eq, float("-inf")))          # 0 above the diagonal
    A = (bg.unsqueeze(-1) * (kg @ kg.transpose(-1, -2)) * dec).masked_fill(~lower, 0.0)
    rhs = torch.cat([bg.unsqueeze(-1) * vg, (bg * torch.exp(G)).unsqueeze(-1) * kg], -1)
    eye = torch.eye(C, device=q.device, dtype=A.dtype)
    W = torch.linalg.solve_triangular(A + eye, rhs, upper=False, unitriangular=True)
    Wv, Wk = W[..., :dv], W[..., dv:]
    P = (qg @ kg.transpose(-1, -2)) * dec                                 # j <= i kept
    q_in = qg * torch.exp(G).unsqueeze(-1)
    k_out = kg * torch.exp(G[..., -1:] - G).unsqueeze(-1)
    keep = torch.exp(G[..., -1])                                          # [NC, H]
    out = torch.empty(NC, H, C, dv, device=q.device, dtype=torch.float32)
    state = torch.zeros(len(lay.lengths), H, dk, dv, device=q.device, dtype=torch.float32)
    for cids, sids in zip(lay.by_ordinal, lay.seg_of_ordinal):
        S0 = state[sids]
        U = Wv[cids] - Wk[cids] @ S0
        out[cids] = q_in[cids] @ S0 + P[cids] @ U
        state[sids] = keep[cids][..., None, None] * S0 + k_out[cids].transpose(-1, -2) @ U
    flat = out.transpose(1, 2).reshape(NC * C, H * dv)[lay.grid_valid]
    return flat.view(T, H, dv)


def causal_conv_packed(x: torch.Tensor, weight: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    """Depthwise causal convolution over ``x [T, D]`` with taps ``weight [D, 1, K]`` (last tap on the
    current token) that reads no token of an earlier caption; fp32 sum, rounded to ``x``'s dtype."""
    K = weight.shape[-1]
    w = weight.view(weight.shape[0], K).float()
    acc = x.float() * w[:, K - 1]
    for back in range(1, K):
        prev = torch.zeros_like(acc)
        prev[back:] = x[:-back].float()
        prev.masked_fill_((pos < back).view(-1, 1), 0.0)
        acc = acc + prev * w[:, K - 1 - back]
    return acc.to(x.dtype)


def _rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """RoPE on the leading ``cos.shape[-1]`` features of every head (halves paired: i with i + r/2)."""
    r = cos.shape[-1]
    head, tail = x[..., :r], x[..., r:]
    h1, h2 = head[..., : r // 2], head[..., r // 2:]
    turned = torch.cat([h2.neg(), h1], -1)
    return torch.cat([head * cos + turned * sin, tail], -1)


class PackedQwenForward:
    """Runs a loaded Qwen3.5 text model (``transformers`` ``Qwen3_5TextModel``-like: ``embed_tokens``,
    ``layers`` with ``layer_type``, ``rotary_emb``, ``norm``) over packed captions."""

    def __init__(self, lm, chunk: int = CHUNK):
        self.lm = lm
        self.chunk = chunk

    @staticmethod
    def supports(lm) -> bool:
        layers = getattr(lm, "layers", None)
        return (layers is not None and len(layers) > 0 and hasattr(lm, "embed_tokens")
                and hasattr(lm, "rotary_emb") and all(hasattr(l, "layer_type") for l in layers))

    # ---- mixers
    def _full_attention(self, att, x, cos, sin, lengths):
        T = x.shape[0]
        hd = att.head_dim
        qg = att.q_proj(x).view(T, -1, 2 * hd)
        H = qg.shape[1]
        q, gate = qg[..., :hd], qg[..., hd:].reshape(T, H * hd)
        q = _rotate(att.q_norm(q), cos, sin)
        k = _rotate(att.k_norm(att.k_proj(x).view(T, -1, hd)), cos, sin)
        v = att.v_proj(x).view(T, -1, hd)
        out = torch.empty(T, H, hd, device=x.device, dtype=x.dtype)
        a = 0
        for n in lengths:
            b = a + n
            o = F.scaled_dot_product_attention(q[a:b].transpose(0, 1)[None], k[a:b].transpose(0, 1)[None],
                                               v[a:b].transpose(0, 1)[None], is_causal=True,
                                               scale=att.scaling, enable_gqa=True)
            out[a:b] = o[0].transpose(0, 1)
            a = b
        return att.o_proj(out.reshape(T, H * hd) * torch.sigmoid(gate))

    def _linear_attention(self, la, x, lay: _Layout):
        T = x.shape[0]
        mixed = F.silu(causal_conv_packed(la.in_proj_qkv(x), la.conv1d.weight, lay.pos))
        q, k, v = torch.split(mixed, [la.key_dim, la.key_dim, la.value_dim], dim=-1)
        q = q.reshape(T, -1, la.head_k_dim)
        k = k.reshape(T, -1, la.head_k_dim)
        v = v.reshape(T, -1, la.head_v_dim)
        z = la.in_proj_z(x).reshape(T, -1, la.head_v_dim)
        beta = torch.sigmoid(la.in_proj_b(x))
        g = -la.A_log.float().exp() * F.softplus(la.in_proj_a(x).float() + la.dt_bias)
        rep = la.num_v_heads // la.num_k_heads
        if rep > 1:
            q = q.repeat_interleave(rep, dim=1)
            k = k.repeat_interleave(rep, dim=1)
        o = gated_delta_rule_packed(q, k, v, beta, g, lay, self.chunk).to(x.dtype)
        # gated RMS norm over each head's value features: norm first, then the SiLU gate
        of = o.float()
        eps = float(getattr(la.norm, "variance_epsilon", getattr(la.norm, "eps", la.layer_norm_epsilon)))
        of = of * torch.rsqrt(of.pow(2).mean(-1, keepdim=True) + eps)
        o = la.norm.weight * of.to(x.dtype)
        o = (o * F.silu(z.float())).to(x.dtype)
        return la.out_proj(o.reshape(T, -1))

    @torch.no_grad()
    def __call__(self, input_ids: torch.Tensor, lengths: Sequence[int]) -> torch.Tensor:
        """``input_ids [T]`` (the captions back to back), ``lengths`` their token counts ->
        ``[T, hidden]`` last hidden states."""
        lm = self.lm
        dev = lm.embed_tokens.weight.device
        ids = input_ids.to(dev)
        lay = _layout(lengths, self.chunk, dev)
        x = lm.embed_tokens(ids)
        rot = lm.rotary_emb
        freqs = lay.pos.float().unsqueeze(-1) * rot.inv_freq.float().to(dev).unsqueeze(0)
        emb = torch.cat([freqs, freqs], -1)
        scale = float(getattr(rot, "attention_scaling", 1.0))
        cos = (emb.cos() * scale).to(x.dtype).unsqueeze(1)
        sin = (emb.sin() * scale).to(x.dtype).unsqueeze(1)
        n_layers = int(getattr(lm.config, "num_hidden_layers", len(lm.layers)))
        for layer in lm.layers[:n_layers]:
            h = layer.input_layernorm(x)
            if layer.layer_type == "linear_attention":
                h = self._linear_attention(layer.linear_attn, h, lay)
            else:
                h = self._full_attention(layer.self_attn, h, cos, sin, lay.lengths)
            x = x + h
            x = x + layer.mlp(layer.post_attention_layernorm(x))
        return lm.norm(x)
