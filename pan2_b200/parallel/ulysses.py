"""Ulysses context parallelism for the packed attention over NCCL (the baseline transport; on one
node the exchanges run inside the kernels instead, :mod:`pan2_b200.parallel.cp_fused`).

Layout (the reference's, pan/utils/ulysses.py:1-182, so checkpoints, loaders and CP batches agree):
in a cp group of ``cp`` ranks the joint token ``i`` lives on cp-rank ``i % cp``; outside attention a
rank holds its token shard with every head, and attention runs on the FULL sequence for the rank's
``H / cp`` heads.

Exchange design (this module's own): every rank pads its shard to ``rows = ceil(S / cp)`` rows, so
the all-to-all has equal splits.  Received chunk ``r`` holds tokens ``r, r + cp, r + 2cp, ...``, so
the stack of chunks ``[cp, rows, ...]`` read column-major -- a transpose to ``[rows, cp, ...]`` --
is the sequence in its true order, with the padding rows falling past ``S``.  No permutation table
or row gather is needed in either direction.  Each direction's backward is the other direction.
"""
from __future__ import annotations

import functools
from typing import Sequence, Tuple

import torch
import torch.distributed as dist

from .collectives import all_to_all_list


@functools.lru_cache(maxsize=256)
def shard_sizes(total: int, cp: int) -> Tuple[int, ...]:
    """Tokens held by each cp-rank: rank ``r`` holds ``r, r + cp, ...`` of ``total``."""
    base, extra = divmod(total, cp)
    return tuple(base + (1 if r < extra else 0) for r in range(cp))


def _exchange(send: torch.Tensor, cp: int, group) -> torch.Tensor:
    """Equal-split all-to-all of ``send`` = ``[cp, ...]`` (chunk ``j`` goes to rank ``j``); the
    result's chunk ``j`` came from rank ``j``."""
    recv = torch.empty_like(send)
    if send.is_cuda and "nccl" in dist.get_backend(group):
        dist.all_to_all_single(recv, send, group=group)
    else:
        all_to_all_list(list(recv.unbind(0)), list(send.unbind(0)), group=group)
    return recv


def gather_heads(x: torch.Tensor, total: int, group) -> torch.Tensor:
    """``[shard, H, D]`` (this rank's tokens, all heads) -> ``[total, H / cp, D]`` (all tokens,
    this rank's heads)."""
    cp = dist.get_world_size(group)
    n, H, D = x.shape
    rows = -(-total // cp)
    hb = H // cp
    send = x.new_zeros(cp, rows, hb, D)                       # [dest head block, my rows, ...]
    send[:, :n] = x.view(n, cp, hb, D).transpose(0, 1)
    recv = _exchange(send, cp, group)                         # [source rank, its rows, my heads]
    return recv.transpose(0, 1).reshape(rows * cp, hb, D)[:total]


def scatter_heads(y: torch.Tensor, shard: int, group) -> torch.Tensor:
    """``[total, H / cp, D]`` (all tokens, this rank's heads) -> ``[shard, H, D]`` (this rank's
    tokens, all heads)."""
    cp = dist.get_world_size(group)
    total, hb, D = y.shape
    rows = -(-total // cp)
    full = y.new_zeros(rows * cp, hb, D)
    full[:total] = y
    send = full.view(rows, cp, hb, D).transpose(0, 1).contiguous()  # [dest rank, its rows, my heads]
    recv = _exchange(send, cp, group)                                # [source head block, my rows, ...]
    return recv[:, :shard].transpose(0, 1).reshape(shard, cp * hb, D)


class SeqAllToAll(torch.autograd.Function):
    """Tokens -> heads (``to_heads``) or back, for several tensors; the backward runs the other way."""

    @staticmethod
    def forward(ctx, sizes: Sequence[int], group, to_heads: bool, *tensors):
        ctx.sizes, ctx.group, ctx.to_heads = tuple(sizes), group, to_heads
        total = sum(sizes)
        if to_heads:
            return tuple(gather_heads(t.contiguous(), total, group) for t in tensors)
        mine = sizes[dist.get_rank(group)]
        return tuple(scatter_heads(t.contiguous(), mine, group) for t in tensors)

    @staticmethod
    def backward(ctx, *grads):
        back = SeqAllToAll.apply(ctx.sizes, ctx.group, not ctx.to_heads, *grads)
        return (None, None, None) + tuple(back)


def ulysses_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, meta) -> torch.Tensor:
    """Packed attention over a cp-sharded joint sequence.  ``q, k, v``: ``[shard, H, D]``, this
    rank's strided tokens; ``meta.joint_lens`` / ``joint_cu_seqlens`` describe the FULL sequence.
    Returns ``[shard, H, D]``."""
    from ..ops.attention import varlen_attention
    group = meta.cp_group
    cp = dist.get_world_size(group)
    heads = q.shape[1]
    if heads % cp:
        raise ValueError(f"Ulysses splits heads across the cp group: {heads} heads over cp={cp} does not divide")
    total = int(meta.cp_joint_total)
    sizes = shard_sizes(total, cp)
    mine = sizes[dist.get_rank(group)]
    if q.shape[0] != mine:
        raise ValueError(f"this rank holds {q.shape[0]} tokens but its strided share of {total} over cp={cp} is "
                         f"{mine}: split batches with pan2_b200.data.cp_batch")
    qf, kf, vf = SeqAllToAll.apply(sizes, group, True, q, k, v)
    o = varlen_attention(qf, kf, vf, meta.joint_cu_seqlens, meta.joint_lens, meta.joint_segment_limit)
    (out,) = SeqAllToAll.apply(sizes, group, False, o.view(total, heads // cp, -1))
    return out
