"""Ulysses context parallelism for the packed attention (reference: pan/utils/ulysses.py:1-182).

Layout: within a cp group of size ``cp`` the joint (interleave-order) token ``i`` lives on cp-rank
``i % cp``, so shard sizes differ by at most one and any sequence length works.  Outside attention a
rank holds its token shard with all ``H`` heads; the attention trades tokens for heads: after the
forward all-to-all a rank holds the FULL sequence for heads ``[r*H/cp, (r+1)*H/cp)``, attends with the
full-sequence segment lengths, and the reverse all-to-all restores its token shard.

An all-to-all concatenates the received chunks in source-rank order ("grouped": rank 0's tokens
``[0::cp]``, then rank 1's ``[1::cp]`` ...), a permutation of the real order; one row permutation per
direction (cached per length/cp/device) converts it.  Each direction's backward is the other
direction, so the q/k/v trio rides three back-to-back collectives waited on once.

Transport: NCCL ``all_to_all_single`` over NVLink (gloo point-to-point on CPU test ranks).
"""
from __future__ import annotations

import functools
from typing import Sequence, Tuple

import torch
import torch.distributed as dist

from .collectives import all_to_all_list


@functools.lru_cache(maxsize=256)
def shard_sizes(total: int, cp: int) -> Tuple[int, ...]:
    """Rows of shard ``r`` = tokens ``[r::cp]``."""
    return tuple((total - r + cp - 1) // cp for r in range(cp))


_PERM_CACHE: dict = {}


def grouped_perms(total: int, cp: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
    """``(to_full, to_grouped)`` with ``full = grouped[to_full]`` and ``grouped = full[to_grouped]``."""
    key = (total, cp, str(device))
    hit = _PERM_CACHE.get(key)
    if hit is None:
        sizes = shard_sizes(total, cp)
        to_grouped = torch.cat([torch.arange(sizes[r]) * cp + r for r in range(cp)])
        to_full = torch.argsort(to_grouped)
        hit = (to_full.to(device), to_grouped.to(device))
        if len(_PERM_CACHE) > 64:
            _PERM_CACHE.clear()
        _PERM_CACHE[key] = hit
    return hit


def _a2a(recv: torch.Tensor, send: torch.Tensor, out_splits: Sequence[int], in_splits: Sequence[int], group):
    be = dist.get_backend(group)
    if "nccl" in be and send.is_cuda:
        return dist.all_to_all_single(recv, send, output_split_sizes=list(out_splits),
                                      input_split_sizes=list(in_splits), group=group, async_op=True)
    all_to_all_list(list(recv.split(list(out_splits))), list(send.split(list(in_splits))), group=group)
    return None


def _tokens_to_heads(x: torch.Tensor, sizes: Sequence[int], group):
    """``[s_local, H, D]`` (my tokens, all heads) -> ``[S, H/cp, D]`` (all tokens, my heads)."""
    cp = len(sizes)
    s_local, H, D = x.shape
    hl = H // cp
    S = sum(sizes)
    send = x.reshape(s_local, cp, hl, D).transpose(0, 1).contiguous().view(-1)
    recv = send.new_empty(S * hl * D)
    work = _a2a(recv, send, [s * hl * D for s in sizes], [s_local * hl * D] * cp, group)
    to_full, _ = grouped_perms(S, cp, x.device)
    return work, send, lambda: recv.view(S, hl, D).index_select(0, to_full)


def _heads_to_tokens(y: torch.Tensor, sizes: Sequence[int], group):
    """``[S, H/cp, D]`` (all tokens, my heads) -> ``[s_local, H, D]`` (my tokens, all heads)."""
    cp = len(sizes)
    S, hl, D = y.shape
    s_local = sizes[dist.get_rank(group)]
    _, to_grouped = grouped_perms(S, cp, y.device)
    send = y.index_select(0, to_grouped).contiguous().view(-1)
    recv = send.new_empty(cp * s_local * hl * D)
    work = _a2a(recv, send, [s_local * hl * D] * cp, [s * hl * D for s in sizes], group)
    return work, send, lambda: recv.view(cp, s_local, hl, D).transpose(0, 1).reshape(s_local, cp * hl, D).contiguous()


class SeqAllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, sizes, group, to_heads, *tensors):
        ctx.sizes, ctx.group, ctx.to_heads = sizes, group, to_heads
        fn = _tokens_to_heads if to_heads else _heads_to_tokens
        pending = [fn(t.contiguous(), sizes, group) for t in tensors]
        outs = []
        for work, _send, finish in pending:
            if work is not None:
                work.wait()
            outs.append(finish())
        return tuple(outs)

    @staticmethod
    def backward(ctx, *grads):
        back = SeqAllToAll.apply(ctx.sizes, ctx.group, not ctx.to_heads, *[g.contiguous() for g in grads])
        return (None, None, None) + tuple(back)


def ulysses_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, meta) -> torch.Tensor:
    """Packed attention over a cp-sharded joint sequence.  ``q, k, v``: ``[s_local, H, D]`` (this
    rank's strided token shard); ``meta.joint_lens`` / ``joint_cu_seqlens`` are the FULL sequence's
    segments.  Returns ``[s_local, H, D]``."""
    from ..ops.attention import varlen_attention
    group = meta.cp_group
    cp = dist.get_world_size(group)
    H = q.shape[1]
    if H % cp:
        raise ValueError(f"{H} heads are not divisible by cp={cp}")
    S = int(meta.cp_joint_total)
    sizes = shard_sizes(S, cp)
    me = dist.get_rank(group)
    if q.shape[0] != sizes[me]:
        raise ValueError(f"local token count {q.shape[0]} != cp shard size {sizes[me]} (S={S}, cp={cp}); "
                         "the batch was not split by pan2_b200.data.cp_batch")
    qf, kf, vf = SeqAllToAll.apply(sizes, group, True, q, k, v)
    o = varlen_attention(qf, kf, vf, meta.joint_cu_seqlens, meta.joint_lens, meta.joint_segment_limit)
    (out,) = SeqAllToAll.apply(sizes, group, False, o.view(S, H // cp, -1))
    return out
