"""Process groups and device meshes (reference: pan/commons/parallel_layout.py:27-89).

``init_parallel_layout(cp, hybrid_shard)`` creates the default process group (``cpu:gloo,cuda:nccl``
when CUDA is present, gloo otherwise), a ``(dp, cp)`` mesh and an FSDP mesh
``(dp_replicate, fsdp_shard)``.  With ``hybrid_shard`` the shard axis is the ranks of one node and
the replicate axis spans nodes; otherwise everything shards.  A world of one is created from a
``HashStore`` when the process was not launched by torchrun, so single-process tools work
unchanged.  ``current_parallel_layout()`` returns the active layout (a trivial one before init).
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


@dataclass
class ParallelLayout:
    world_size: int = 1
    rank: int = 0
    cp_size: int = 1
    dp_size: int = 1
    cp_rank: int = 0
    dp_rank: int = 0
    shard_size: int = 1
    shard_rank: int = 0
    replicate_size: int = 1
    replicate_rank: int = 0
    cp_group: Optional[dist.ProcessGroup] = None
    dp_group: Optional[dist.ProcessGroup] = None
    shard_group: Optional[dist.ProcessGroup] = None
    replicate_group: Optional[dist.ProcessGroup] = None
    cpu_group: Optional[dist.ProcessGroup] = None
    cp_cpu_group: Optional[dist.ProcessGroup] = None   # gloo twin of cp_group (host metadata)

    @property
    def cp_enabled(self) -> bool:
        return self.cp_size > 1


_LAYOUT = ParallelLayout()


def current_parallel_layout() -> ParallelLayout:
    return _LAYOUT


def _local_world() -> int:
    v = os.environ.get("LOCAL_WORLD_SIZE")
    if v is not None:
        return int(v)
    return max(1, torch.cuda.device_count()) if torch.cuda.is_available() else 1


def init_process_group(timeout_s: float = 600.0, backend: Optional[str] = None) -> None:
    """Default process group; a single-process world comes from a HashStore."""
    if dist.is_initialized():
        return
    timeout = datetime.timedelta(seconds=timeout_s)
    if backend is None:
        backend = "cpu:gloo,cuda:nccl" if torch.cuda.is_available() else "gloo"
    if "RANK" in os.environ and "WORLD_SIZE" in os.environ:
        if torch.cuda.is_available():
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        dist.init_process_group(backend=backend, timeout=timeout)
    else:
        store = dist.HashStore()
        dist.init_process_group(backend=backend, store=store, rank=0, world_size=1, timeout=timeout)


def init_parallel_layout(cp: int = 1, hybrid_shard: bool = False, timeout_s: float = 600.0,
                         backend: Optional[str] = None) -> ParallelLayout:
    """Create the process group (if needed) and the dp/cp and shard/replicate groups."""
    global _LAYOUT
    init_process_group(timeout_s, backend)
    world, rank = dist.get_world_size(), dist.get_rank()
    if world % cp:
        raise ValueError(f"{world} ranks cannot be split into context-parallel groups of {cp}")
    dp = world // cp
    # (dp, cp) mesh, cp fastest: ranks [d*cp, (d+1)*cp) form one cp group
    cp_groups = [list(range(d * cp, (d + 1) * cp)) for d in range(dp)]
    dp_groups = [list(range(c, world, cp)) for c in range(cp)]
    shard = min(world, _local_world()) if hybrid_shard else world
    if world % shard:
        shard = world
    rep = world // shard
    shard_groups = [list(range(r * shard, (r + 1) * shard)) for r in range(rep)]
    rep_groups = [list(range(s, world, shard)) for s in range(shard)]

    def pick(groups):
        mine = None
        for g in groups:
            pg = dist.new_group(g) if len(groups) > 1 or len(g) != world else dist.group.WORLD
            if rank in g:
                mine = pg
        return mine

    layout = ParallelLayout(world_size=world, rank=rank, cp_size=cp, dp_size=dp, cp_rank=rank % cp,
                            dp_rank=rank // cp, shard_size=shard, shard_rank=rank % shard, replicate_size=rep,
                            replicate_rank=rank // shard)
    layout.cp_group = pick(cp_groups)
    layout.dp_group = pick(dp_groups)
    layout.shard_group = pick(shard_groups)
    layout.replicate_group = pick(rep_groups)
    try:
        layout.cpu_group = dist.new_group(list(range(world)), backend="gloo") if world > 1 else None
    except Exception:  # pragma: no cover
        layout.cpu_group = None
    if cp > 1:
        for g in cp_groups:
            pg = dist.new_group(g, backend="gloo")
            if rank in g:
                layout.cp_cpu_group = pg
    _LAYOUT = layout
    return layout


def reset_parallel_layout(destroy: bool = False) -> None:
    """Forget the layout; with ``destroy`` also tear down the default process group (and with it
    every subgroup), e.g. when a process that trained in-process exits cleanly."""
    global _LAYOUT
    _LAYOUT = ParallelLayout()
    if destroy and dist.is_initialized():
        dist.destroy_process_group()
