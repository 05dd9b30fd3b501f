"""Peer memory of one node: symmetric buffers, device barriers and the fused gather / reduce plans.

Every rank of the shard group allocates the same-sized buffer through PyTorch's symmetric memory
(CUDA virtual-memory allocations mapped into all peers over NVLink); :class:`PeerMemory` holds the
peer base addresses and signal pads as device arrays, so the kernels of ``csrc/comm_ops.cu`` address
any rank's memory directly:

* :meth:`PeerMemory.barrier` -- a device-side barrier on one of 8 signal channels (monotonic epochs,
  bounded 4 s wait that records an error code instead of hanging);
* :class:`GatherPlan` -- the FSDP all-gather of one unit fused with the unpack: rank ``r`` pulls row
  range ``r`` of every parameter from peer ``r``'s ``hi`` shard into the natural full layout;
* :class:`ReducePlan` -- the gradient reduce-scatter of one unit fused with the bf16 -> fp32 cast and
  scale: each rank sums its row range of every parameter across all peers' bf16 gradients;
* :class:`PeerProjection` -- the all-gather fused into the consuming projection for a skinny
  activation (the AdaLN modulation: k <= 8 conditioning rows against a 6H x H weight): the weight
  is read once, row by row from the rank that owns it, and never materialised locally.

Plans are lists of contiguous element runs computed once per unit on the host (the row-sharded
layout makes every parameter's rank slice one run in both layouts).
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from ..ops._ext import ext

N_CHANNELS = 8


def peer_memory_available(group, device) -> bool:
    """Symmetric memory works for CUDA NCCL groups whose ranks share one node."""
    if group is None or not dist.is_initialized() or torch.device(device).type != "cuda":
        return False
    import importlib
    try:
        importlib.import_module("torch.distributed._symmetric_memory")
    except ImportError:
        return False
    if "nccl" not in dist.get_backend(group):
        return False
    import os
    local = int(os.environ.get("LOCAL_WORLD_SIZE", "0") or 0)
    return local >= dist.get_world_size(group) > 1


class PeerMemory:
    def __init__(self, nbytes: int, group, device):
        import torch.distributed._symmetric_memory as symm_mem
        self.device = torch.device(device)
        nbytes = (int(nbytes) + 255) // 256 * 256
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=self.device)
        self.handle = symm_mem.rendezvous(self.buf, group)
        self.rank, self.world = self.handle.rank, self.handle.world_size
        self.peers = torch.tensor(list(self.handle.buffer_ptrs), dtype=torch.int64, device=self.device)
        self.pads = torch.tensor(list(self.handle.signal_pad_ptrs), dtype=torch.int64, device=self.device)
        self.epoch = [0] * N_CHANNELS
        self.nbytes = nbytes
        # start from clean signal slots on every rank
        self.handle.get_signal_pad(self.rank).zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)

    def view(self, offset_bytes: int, numel: int, dtype) -> torch.Tensor:
        es = torch.empty(0, dtype=dtype).element_size()
        assert offset_bytes % 16 == 0 and offset_bytes + numel * es <= self.nbytes
        return self.buf[offset_bytes:offset_bytes + numel * es].view(dtype)

    def peer_ptrs(self, offset_bytes: int) -> torch.Tensor:
        """Device array of every rank's address of byte ``offset_bytes`` of this buffer."""
        return self.peers + offset_bytes

    def barrier(self, channel: int = 0, timeout_ms: int = 4000) -> None:
        """Device-side barrier of all ranks on the current stream (every rank must call it).  A rank
        that waits longer than ``timeout_ms`` records error code 100 + peer and continues."""
        self.epoch[channel] += 1
        ext().symm_barrier(self.pads, self.rank, self.world, self.epoch[channel] & 0x7FFFFFFF, channel, timeout_ms)


def _pack(segs: List[Tuple[int, int, int]], peers: Optional[List[int]], device):
    """Device tensors of a run list: (segs [n,3], prefix [n], total work units, seg_peer [n])."""
    prefix, total = [], 0
    for src, dst, n in segs:
        prefix.append(total)
        aligned = (src | dst | n) % 8 == 0
        total += n // 8 if aligned else n
    t = torch.tensor(segs if segs else [(0, 0, 0)], dtype=torch.int64).reshape(-1, 3).to(device)
    p = torch.tensor(prefix if prefix else [0], dtype=torch.int64).to(device)
    sp = torch.tensor(peers if peers else [0] * max(1, len(segs)), dtype=torch.int32).to(device)
    return t, p, total, sp


class GatherPlan:
    """Unit all-gather: ``full[natural]`` <- every peer's ``hi`` shard rows (peer memory reads).
    Slots in ``skip`` are left out (their region of ``full`` stays unwritten)."""

    def __init__(self, unit, world: int, hi_offset_elems: int, device, skip=()):
        segs, peers = [], []
        skip = {id(s) for s in skip}
        for s in unit.slots:
            if id(s) in skip:
                continue
            for r in range(world):
                a = min(s.rows, r * s.shard_rows)
                b = min(s.rows, a + s.shard_rows)
                if b > a:
                    segs.append((hi_offset_elems + s.shard_off, s.full_off + a * s.cols, (b - a) * s.cols))
                    peers.append(r)
        self.segs, self.prefix, self.total, self.seg_peer = _pack(segs, peers, device)

    def run(self, pm: PeerMemory, full: torch.Tensor) -> None:
        ext().peer_gather(pm.peers, self.segs, self.seg_peer, self.prefix, self.total, full)


class ReducePlan:
    """Unit reduce-scatter: ``shard[fp32]`` <- scale * sum over peers of their natural-layout bf16
    gradient rows owned by this rank."""

    def __init__(self, unit, rank: int, world: int, device):
        segs = []
        for s in unit.slots:
            a = min(s.rows, rank * s.shard_rows)
            b = min(s.rows, a + s.shard_rows)
            if b > a:
                segs.append((s.full_off + a * s.cols, s.shard_off, (b - a) * s.cols))
        self.segs, self.prefix, self.total, _ = _pack(segs, None, device)
        self.world = world

    def run(self, peer_grad_ptrs: torch.Tensor, out: torch.Tensor, scale: float = 1.0) -> None:
        ext().peer_reduce(peer_grad_ptrs, self.world, self.segs, self.prefix, self.total, scale, out)


class PeerProjection:
    """``y [k, N] = a [k, K] @ W^T + b`` for a weight slot ``W`` of a sharded unit, reading every row
    of ``W`` from its owner's ``hi`` shard (peer memory) inside the projection kernel."""

    def __init__(self, slot, hi_offset_elems: int):
        self.slot = slot
        self.w_off = hi_offset_elems + slot.shard_off
        if self.w_off % 8 or slot.cols % 8:
            raise ValueError("peer projection needs 16-byte aligned weight rows")

    def run(self, pm: PeerMemory, a: torch.Tensor, bias: Optional[torch.Tensor], out: torch.Tensor) -> None:
        ext().peer_gemv(pm.peers, self.w_off, self.slot.shard_rows, a, bias, out)
