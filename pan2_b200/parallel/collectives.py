"""Collective helpers that work on both NCCL (GPU) and gloo (CPU test ranks)."""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist


def _backend(group) -> str:
    try:
        return dist.get_backend(group)
    except Exception:  # pragma: no cover
        return "unknown"


def all_to_all_list(out: List[torch.Tensor], inp: List[torch.Tensor], group: Optional[dist.ProcessGroup] = None):
    """``out[j] <- rank j's inp[me]`` for every rank ``j`` (tensor sizes may differ per pair).

    NCCL runs a grouped all-to-all; gloo (which has no all-to-all) uses matched point-to-point sends."""
    be = _backend(group)
    if "nccl" in be and inp[0].is_cuda:
        dist.all_to_all(out, inp, group=group)
        return
    world = dist.get_world_size(group)
    me = dist.get_rank(group)
    reqs = []
    for j in range(world):
        gj = dist.get_global_rank(group, j) if group is not None else j
        if j == me:
            if out[j].numel():
                out[j].copy_(inp[j])
            continue
        if inp[j].numel():
            reqs.append(dist.isend(inp[j].contiguous(), gj, group=group))
        if out[j].numel():
            reqs.append(dist.irecv(out[j], gj, group=group))
    for r in reqs:
        r.wait()
