"""Ulysses context parallelism with the all-to-alls folded into the kernels around attention.

The reference trades tokens for heads with NCCL all-to-alls plus index_select permutations on
both sides of attention (pan/utils/ulysses.py:51-106, 4 collectives per block forward and 4 in
backward).  On one node the cp ranks' memories are mapped into each other over NVLink, so here the
kernels that produce or consume the exchanged tensors address the other ranks directly:

forward
  1. the QKV GEMM (local), then ``qkv_post`` (RMS q/k norm + RoPE) writes every (token, head) row
     straight into the head owner's head-sharded q/k/v buffer, at the token's global row
     ``t * cp + rank`` (the strided shard makes that a pure index computation, no permutation);
  2. device barrier; attention over the full sequence for this rank's ``H / cp`` heads, whose
     epilogue stores each output row both locally (kept for the backward) and into the token
     owner's token-sharded buffer;
  3. device barrier; the output rows are gathered into concat order for the out-projection.
backward
  1. dO (token-sharded) goes into this rank's exchange buffer; device barrier;
  2. the attention backward's prologue pulls every dO row of its heads from the token owners while
     forming Delta, its dK / dV epilogue and the dQ conversion write their rows to the token owners;
  3. device barrier; ``qkv_post`` backward and the QKV weight / input gradients run locally.

Every buffer that a peer writes is only rewritten after a barrier that all readers of its previous
contents have passed (the four barriers of a block order each producer after the previous
consumers).  Tensors that the backward needs from the forward (q/k/v in the exchange buffers) are
valid until the next block's forward runs, which is exactly the activation-checkpointing order
(recompute block l, then its backward); a backward that would read overwritten buffers raises.

No TMA ever reads another rank's memory: peer addresses appear only in plain vector loads and
stores of ``csrc/qkv_ops.cu`` and ``csrc/attention_sm100.cu``.
"""
from __future__ import annotations

import math
import os
from typing import Dict, Sequence, Tuple

import torch
import torch.distributed as dist

from ..ops._ext import ext
from ..ops.attention import work_items
from .symm import PeerMemory, peer_memory_available

REGIONS = ("q", "k", "v", "o", "do", "dq", "dk", "dv")
_ROW_QUANTUM = 2048


def fused_cp_enabled(group, device) -> bool:
    """The fused path runs for CUDA cp groups inside one node (``PAN_CP_FUSED=0`` turns it off)."""
    if os.environ.get("PAN_CP_FUSED", "1") == "0":
        return False
    return peer_memory_available(group, device)


class CPWorkspace:
    """Exchange buffers of one cp group in peer-mapped memory, one region per exchanged tensor.

    Head-sharded regions (q, k, v) hold ``[S, H/cp, D]`` and token-sharded ones (o, do, dq, dk, dv)
    ``[rows, H, D]``, where ``rows = ceil(S / cp)``; both are ``rows * H * D`` elements.
    """

    def __init__(self, group, device, rows: int, heads: int, head_dim: int):
        self.group = group
        self.cp = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.heads, self.head_dim = heads, head_dim
        self.hl = heads // self.cp
        self.rows = (rows + _ROW_QUANTUM - 1) // _ROW_QUANTUM * _ROW_QUANTUM
        self.region_elems = self.rows * heads * head_dim
        self.pm = PeerMemory(len(REGIONS) * self.region_elems * 2, group, device)
        self.tables: Dict[str, torch.Tensor] = {}
        self.offsets: Dict[str, int] = {}
        for i, name in enumerate(REGIONS):
            off = i * self.region_elems * 2
            self.offsets[name] = off
            self.tables[name] = self.pm.peer_ptrs(off).contiguous()
        self.generation = 0

    def head_view(self, name: str, S: int) -> torch.Tensor:
        return self.pm.view(self.offsets[name], S * self.hl * self.head_dim, torch.bfloat16).view(
            S, self.hl, self.head_dim)

    def token_view(self, name: str, rows: int) -> torch.Tensor:
        return self.pm.view(self.offsets[name], rows * self.heads * self.head_dim, torch.bfloat16).view(
            rows, self.heads, self.head_dim)

    def barrier(self, channel: int) -> None:
        self.pm.barrier(channel)


_WORKSPACES: Dict[Tuple, CPWorkspace] = {}


def workspace(group, device, S: int, heads: int, head_dim: int) -> CPWorkspace:
    """The cp group's workspace, (re)allocated collectively when ``S`` outgrows it (every cp rank
    sees the same ``S``, so all of them take the same decision)."""
    cp = dist.get_world_size(group)
    rows = (S + cp - 1) // cp
    key = (id(group), str(device), heads, head_dim)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.rows < rows:
        if ws is not None:
            del _WORKSPACES[key]
            torch.cuda.synchronize(device)
        ws = CPWorkspace(group, device, rows, heads, head_dim)
        _WORKSPACES[key] = ws
    return ws


class _FusedQKVAttention(torch.autograd.Function):
    """``o_concat = out-projection input`` from the normalised block input, through the grouped QKV
    GEMM, the scattering ``qkv_post``, full-sequence attention over this rank's heads and the
    gathering epilogue."""

    @staticmethod
    def forward(ctx, x, w, b, qw, kw, cos, sin, itc, cti, bounds, heads, eps, joint_lens, S, ws):
        from ..ops.gemm import grouped_mm_nt
        E = ext()
        L = x.shape[0]
        D = w.shape[-1] // heads
        wc = w.to(torch.bfloat16).contiguous()
        bc = b.to(torch.bfloat16).contiguous()
        raw = torch.empty(L, wc.shape[1], dtype=torch.bfloat16, device=x.device)
        grouped_mm_nt(x, wc, bounds, raw, bias=bc)
        qwf, kwf = qw.float().contiguous(), kw.float().contiguous()
        E.qkv_post_fwd_scatter(raw, qwf, kwf, cos, sin, itc, bounds[1], bounds[2], heads, eps,
                               ws.tables["q"], ws.tables["k"], ws.tables["v"], ws.cp, ws.rank)
        ws.barrier(0)
        q, k, v = (ws.head_view(n, S) for n in ("q", "k", "v"))
        n_valid = int(sum(joint_lens))
        scale = 1.0 / math.sqrt(D)
        o_head, lse = E.attn_fwd_cp(q, k, v, work_items(joint_lens, 256, x.device), n_valid, scale,
                                    ws.tables["o"], ws.cp, ws.rank * ws.hl, heads)
        ws.barrier(1)
        o_tok = ws.token_view("o", L).view(L, heads * D)
        o_concat = o_tok.index_select(0, itc.long())
        ws.generation += 1
        ctx.gen = ws.generation
        ctx.save_for_backward(x, wc, raw, qw, kw, cos, sin, itc, cti, o_head, lse)
        ctx.ws, ctx.S, ctx.heads, ctx.eps, ctx.scale = ws, S, heads, eps, scale
        ctx.bounds, ctx.joint_lens, ctx.n_valid = list(bounds), list(joint_lens), n_valid
        ctx.dtypes = (w.dtype, b.dtype, qw.dtype, kw.dtype)
        return o_concat

    @staticmethod
    def backward(ctx, d_oc):
        from ..ops.gemm import mm_nn, mm_tn
        from ..ops.packed import segment_sum
        ws = ctx.ws
        if ws.generation != ctx.gen:
            raise RuntimeError("fused context-parallel attention: the exchange buffers were reused by a later "
                               "forward before this backward; run every block under activation checkpointing "
                               "or set PAN_CP_FUSED=0")
        x, wc, raw, qw, kw, cos, sin, itc, cti, o_head, lse = ctx.saved_tensors
        E = ext()
        L = x.shape[0]
        heads = ctx.heads
        D = o_head.shape[-1]
        do_tok = ws.token_view("do", L).view(L, heads * D)
        torch.index_select(d_oc.contiguous(), 0, cti.long(), out=do_tok)
        ws.barrier(2)
        q, k, v = (ws.head_view(n, ctx.S) for n in ("q", "k", "v"))
        E.attn_bwd_cp(q, k, v, o_head, lse, work_items(ctx.joint_lens, 128, x.device), ctx.n_valid, ctx.scale,
                      ws.tables["do"], ws.tables["dq"], ws.tables["dk"], ws.tables["dv"], ws.cp,
                      ws.rank * ws.hl, heads)
        ws.barrier(3)
        dq, dk, dv = (ws.token_view(n, L) for n in ("dq", "dk", "dv"))
        bounds = ctx.bounds
        draw, dqw, dkw = E.qkv_post_bwd(dq, dk, dv, raw, qw.float().contiguous(), kw.float().contiguous(), cos,
                                        sin, itc, bounds[1], bounds[2], heads, ctx.eps)
        gx = torch.zeros_like(x)
        gw = torch.zeros(wc.shape, dtype=torch.float32, device=x.device)
        for g in range(len(bounds) - 1):
            r0, r1 = bounds[g], bounds[g + 1]
            if r1 <= r0:
                continue
            mm_nn(draw[r0:r1], wc[g], out=gx[r0:r1])
            mm_tn(draw[r0:r1], x[r0:r1], out=gw[g])
        gb = segment_sum(draw, bounds)
        wdt, bdt, qdt, kdt = ctx.dtypes
        return (gx, gw.to(wdt), gb.to(bdt), dqw.to(qdt), dkw.to(kdt)) + (None,) * 10


def fused_qkv_ulysses_attention(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, q_weight: torch.Tensor,
                                k_weight: torch.Tensor, meta, bounds: Sequence[int], heads: int,
                                eps: float = 1e-6) -> torch.Tensor:
    """QKV projection + Ulysses attention of a cp-sharded packed block input ``x`` (``[L, hidden]``,
    concat layout, this rank's strided token shard); returns the attention output in concat layout
    ``[L, hidden]``, ready for the out-projection."""
    group = meta.cp_group
    cp = dist.get_world_size(group)
    if heads % cp:
        raise ValueError(f"{heads} heads are not divisible by cp={cp}")
    L, hidden = x.shape
    D = hidden // heads
    S = int(meta.cp_joint_total)
    rows = (S - dist.get_rank(group) + cp - 1) // cp
    if rows != L:
        raise ValueError(f"local token count {L} != cp shard size {rows} (S={S}, cp={cp})")
    ws = workspace(group, x.device, S, heads, D)
    cos = meta.freqs_cos.reshape(meta.freqs_cos.shape[0], -1).float().contiguous()
    sin = meta.freqs_sin.reshape(meta.freqs_sin.shape[0], -1).float().contiguous()
    itc = meta.indices_interleave_to_concat.to(torch.int32).contiguous()
    cti = meta.indices_concat_to_interleave.to(torch.int32).contiguous()
    return _FusedQKVAttention.apply(x.to(torch.bfloat16).contiguous(), weight, bias, q_weight, k_weight, cos, sin,
                                    itc, cti, list(bounds), heads, eps, [int(n) for n in meta.joint_lens], S, ws)
