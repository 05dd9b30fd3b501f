"""Flat sharded parameter units: the B200 replacement for FSDP2 ``fully_shard`` (train.py:788-815).

Every joint block (and one root unit holding everything else) owns one flat buffer.  Within a unit,
each parameter is split row-wise (dim 0) across the shard group exactly like FSDP2's per-parameter
``Shard(0)``: rank ``r`` owns rows ``[r*R/N, (r+1)*R/N)`` of every parameter (rows padded to a
multiple of N).  That keeps Muon's chunk structure local (QKV's 192 row chunks split evenly) and
makes every rank's shard one contiguous buffer, so

* the parameter all-gather is one ``all_gather_into_tensor`` of bf16 ``hi`` shards per unit, followed
  by an unpack into the natural per-parameter layout the model reads;
* the gradient reduce-scatter packs the unit's bf16 gradients rank-major, casts to fp32 and runs one
  ``reduce_scatter_tensor`` (the reference reduces in fp32: ``MixedPrecisionPolicy(reduce=fp32)``).

Master weights are exact fp32 values kept as two 16-bit halves (``hi``: the bf16 compute weight,
``lo``: the low bits).  With one rank the natural and shard layouts coincide and ``hi`` *is* the
model's weight storage.  When the planner decides the GPU cannot hold everything (29B on 1-2 GPUs),
``lo`` and the optimizer state live in pinned host memory and the optimizer streams them per unit.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn

from ..optim.muon import use_muon_for


@dataclass
class ParamSlot:
    name: str                 # name relative to the model root
    module: nn.Module
    attr: str
    shape: Tuple[int, ...]
    rows: int
    cols: int
    rows_pad: int
    full_off: int             # offset in the natural (gathered) layout
    shard_off: int            # offset in the per-rank shard layout
    kind: str                 # "muon" | "adamw"
    chunks: Optional[Tuple[int, int]] = None

    @property
    def numel(self) -> int:
        return self.rows * self.cols

    @property
    def shard_rows(self) -> int:
        return self.rows_pad // self._world

    _world: int = 1


@dataclass
class Unit:
    index: int
    name: str
    module: nn.Module
    slots: List[ParamSlot]
    numel_full: int
    numel_shard: int
    world: int
    hi: Optional[torch.Tensor] = None          # bf16 [numel_shard] (GPU)
    lo: Optional[torch.Tensor] = None          # int16 [numel_shard] (GPU or pinned host)
    full_hi: Optional[torch.Tensor] = None     # bf16 [numel_full] gathered weights (alias of hi when world==1)
    full_grad: Optional[torch.Tensor] = None   # bf16 [numel_full] unsharded gradients
    grad_shard: Optional[torch.Tensor] = None  # fp32 [numel_shard] (world > 1)
    state: Dict[str, torch.Tensor] = field(default_factory=dict)  # optimizer state (flat shard layout)
    gather_event: Optional[torch.cuda.Event] = None
    grad_slot: int = 0                          # peer mode: gradient ring slot of the current backward
    adaln_rows: Optional[torch.Tensor] = None   # peer AdaLN: the forward's modulation rows [k, 6H]
    partial_gather: bool = False                # full_hi lacks the AdaLN weight (forward-only gather)

    def slot_full(self, buf: torch.Tensor, s: ParamSlot) -> torch.Tensor:
        return buf[s.full_off:s.full_off + s.numel].view(s.shape)

    def slot_shard(self, buf: torch.Tensor, s: ParamSlot) -> torch.Tensor:
        n = s.shard_rows * s.cols
        return buf[s.shard_off:s.shard_off + n].view(s.shard_rows, s.cols)


def _align(n: int, a: int) -> int:
    return (n + a - 1) // a * a


def pack_rows(pk: torch.Tensor, s: "ParamSlot", full: torch.Tensor, world: int) -> None:
    """Scatter a full ``[rows, cols]`` parameter into the rank-major packed buffer ``pk``
    (``[world, numel_shard]``): rank ``r`` gets rows ``[r*shard_rows, (r+1)*shard_rows)`` (zero padding)."""
    n = s.shard_rows * s.cols
    dst = pk[:, s.shard_off:s.shard_off + n].view(world, s.shard_rows, s.cols)
    src = full.view(s.rows, s.cols)
    if s.rows == s.rows_pad:
        dst.copy_(src.view(world, s.shard_rows, s.cols))
        return
    for r in range(world):
        a = r * s.shard_rows
        k = max(0, min(s.shard_rows, s.rows - a))
        if k:
            dst[r, :k].copy_(src[a:a + k])
        if k < s.shard_rows:
            dst[r, k:].zero_()


def unpack_rows(pk: torch.Tensor, s: "ParamSlot", full: torch.Tensor, world: int) -> None:
    """Inverse of :func:`pack_rows`: gather the rank-major shards of one parameter into ``full``."""
    n = s.shard_rows * s.cols
    src = pk[:, s.shard_off:s.shard_off + n].view(world, s.shard_rows, s.cols)
    dst = full.view(s.rows, s.cols)
    if s.rows == s.rows_pad:
        dst.view(world, s.shard_rows, s.cols).copy_(src)
        return
    for r in range(world):
        a = r * s.shard_rows
        k = max(0, min(s.shard_rows, s.rows - a))
        if k:
            dst[a:a + k].copy_(src[r, :k])


def build_unit(index: int, name: str, module: nn.Module, world: int, prefix: str = "") -> Unit:
    """Lay out the parameters of ``module`` (names prefixed with ``prefix``)."""
    from ..optim.muon import muon_chunks
    chunk_map = muon_chunks(module)
    slots = []
    full_off = shard_off = 0
    for pname, p in module.named_parameters():
        mod_name, _, attr = pname.rpartition(".")
        owner = module.get_submodule(mod_name) if mod_name else module
        shape = tuple(p.shape)
        rows = shape[0] if len(shape) >= 1 else 1
        cols = int(math.prod(shape[1:])) if len(shape) >= 2 else 1
        rows_pad = _align(rows, world)
        full_name = prefix + pname
        slot = ParamSlot(name=full_name, module=owner, attr=attr, shape=shape, rows=rows, cols=cols,
                         rows_pad=rows_pad, full_off=full_off, shard_off=shard_off,
                         kind="muon" if use_muon_for(full_name, shape) else "adamw",
                         chunks=chunk_map.get(pname))
        slot._world = world
        slots.append(slot)
        # 16-byte aligned offsets (8 bf16 elements) keep every view TMA-addressable
        full_off += _align(rows * cols, 8)
        shard_off += _align(slot.shard_rows * cols, 8)
    return Unit(index=index, name=name, module=module, slots=slots, numel_full=full_off,
                numel_shard=shard_off, world=world)


class ShardedModel:
    """Owns the units of a model and moves weights / gradients between layouts.

    ``units[0..n_blocks-1]`` are the joint blocks; ``units[-1]`` is the root (everything else).
    """

    def __init__(self, units: List[Unit], group: Optional[dist.ProcessGroup], device: torch.device,
                 offload: bool, replicate_group: Optional[dist.ProcessGroup] = None):
        self.units = units
        self.group = group
        # called before the weights are read outside a step (the engine waits for deferred updates)
        self.before_read = None
        # HSDP: shards are replicated across this group (one member per node); gradients are
        # all-reduced over it after the reduce-scatter
        self.replicate_group = (replicate_group if replicate_group is not None and dist.is_initialized()
                                and dist.get_world_size(replicate_group) > 1 else None)
        self.world = units[0].world if units else 1
        self.rank = dist.get_rank(group) if (group is not None and self.world > 1) else 0
        self.device = device
        self.offload = offload
        self.comm_stream = torch.cuda.Stream(device) if device.type == "cuda" else None
        # peer-memory collectives (enable_peer_memory): hi shards and a ring of gradient buffers live
        # in symmetric memory, gathers / reductions are single kernels reading peers over NVLink
        self.peer = False
        self.n_reduce = 0           # gradient reductions issued so far (identical on every rank)
        self._ring_next = 0         # block gradients attached so far
        self._slot_last: Dict[int, int] = {}   # slot -> index of the reduction that last read it
        self._latest: Optional[Tuple[int, torch.cuda.Event]] = None  # last reduction barrier passed
        self._begin_event: Optional[torch.cuda.Event] = None
        # peer AdaLN (enable_peer_memory(peer_adaln=True)): per block unit, the modulation weight is
        # left out of the forward's gather and read from the peers by the projection kernel itself
        self.adaln: Dict[int, tuple] = {}   # unit index -> (PeerProjection, bias slot)
        self.adaln_on = False               # this step's forward uses it (set by the engine)
        self.adaln_input: Optional[torch.Tensor] = None  # act(vec) [k, H] bf16, once known

    # ---------------------------------------------------------------- parameter views
    def bind_weights(self, u: Unit, full: Optional[torch.Tensor]) -> None:
        """Point every module parameter of ``u`` at its view of ``full`` (or an empty placeholder)."""
        for s in u.slots:
            p = getattr(s.module, s.attr)
            if full is None:
                p.data = torch.empty(0, dtype=torch.bfloat16, device=self.device)
            else:
                p.data = u.slot_full(full, s)

    # ---------------------------------------------------------------- peer memory
    GRAD_SLOTS = 4  # slot 0: the root unit's gradient (alive for the whole backward); 1..3: block ring

    def enable_peer_memory(self, peer_adaln: bool = False) -> bool:
        """Move ``hi`` shards into symmetric memory and set up the fused gather / reduce plans.
        Returns False (NCCL collectives stay in use) when peer memory is unavailable.  With
        ``peer_adaln`` every block's AdaLN modulation weight is also set up for the fused
        projection (:meth:`adaln_projection`)."""
        from .symm import GatherPlan, PeerMemory, PeerProjection, ReducePlan, peer_memory_available
        if self.world == 1 or self.replicate_group is not None or not peer_memory_available(self.group, self.device):
            return False
        offs, total = [], 0
        for u in self.units:
            offs.append(total)
            total += _align(u.numel_shard, 128)
        self.hi_mem = PeerMemory(total * 2, self.group, self.device)
        for u, off in zip(self.units, offs):
            view = self.hi_mem.view(off * 2, u.numel_shard, torch.bfloat16)
            view.copy_(u.hi)
            u.hi = view
        self.slot_elems = _align(max(u.numel_full for u in self.units), 128)
        self.grad_mem = PeerMemory(self.GRAD_SLOTS * self.slot_elems * 2, self.group, self.device)
        self.gather_plans = [GatherPlan(u, self.world, off, self.device) for u, off in zip(self.units, offs)]
        self.gather_plans_fwd = list(self.gather_plans)
        if peer_adaln:
            for u, off in zip(self.units, offs):
                lin = getattr(getattr(u.module, "modulation", None), "linear", None)
                w = next((x for x in u.slots if lin is not None and x.module is lin and x.attr == "weight"), None)
                b = next((x for x in u.slots if lin is not None and x.module is lin and x.attr == "bias"), None)
                if w is None or len(w.shape) != 2:
                    continue
                self.adaln[u.index] = (PeerProjection(w, off), b)
                self.gather_plans_fwd[u.index] = GatherPlan(u, self.world, off, self.device, skip=[w])
        self.reduce_plans = [ReducePlan(u, self.rank, self.world, self.device) for u in self.units]
        self.slot_ptrs = [self.grad_mem.peer_ptrs(j * self.slot_elems * 2) for j in range(self.GRAD_SLOTS)]
        torch.cuda.synchronize(self.device)
        self.peer = True
        return True

    def begin_gathers(self) -> None:
        """Peer mode: every rank's optimizer step (which writes ``hi``) precedes this step's gathers."""
        if not self.peer:
            return
        self.comm_stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.comm_stream):
            self.hi_mem.barrier(0)
            # also: every rank finished last step's reductions (they precede this barrier in each
            # rank's communication stream), so the root's gradient slot may be rewritten
            self._begin_event = torch.cuda.Event()
            self._begin_event.record(self.comm_stream)

    def end_gathers(self) -> None:
        """Peer mode: no rank still reads this rank's ``hi`` when the optimizer overwrites it."""
        if not self.peer:
            return
        self.comm_stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.comm_stream):
            self.hi_mem.barrier(1)
        torch.cuda.current_stream(self.device).wait_stream(self.comm_stream)

    def comm_error(self) -> int:
        from ..ops._ext import ext
        return ext().error_flag(False)

    # ---------------------------------------------------------------- all-gather
    def gather(self, u: Unit, stream: Optional[torch.cuda.Stream] = None, forward: bool = False) -> None:
        """Make ``u.full_hi`` hold the unit's full bf16 weights and bind the module to it.  With
        ``forward`` and the peer AdaLN path on, the modulation weight is not gathered; its rows of
        this step's modulation are computed from the peers instead (``take_adaln_rows``)."""
        if self.world == 1:
            u.full_hi = u.hi
            self.bind_weights(u, u.full_hi)
            return
        if u.full_hi is None:
            self.prefetch(u, forward=forward)
        elif u.partial_gather and not forward:
            raise RuntimeError(f"unit {u.index}: forward-only gather reused outside the forward")
        if u.partial_gather and u.adaln_rows is None:
            self._adaln_projection(u)
        if u.gather_event is not None:
            torch.cuda.current_stream(self.device).wait_event(u.gather_event)
            u.gather_event = None
        self.bind_weights(u, u.full_hi)

    def _fused_adaln(self, u: Unit, forward: bool) -> bool:
        return forward and self.peer and self.adaln_on and u.index in self.adaln

    def _adaln_projection(self, u: Unit) -> None:
        """Issue the peer AdaLN projection of ``u`` on the communication stream (after the unit's
        gather, which brings the bias) and move the unit's gather event behind it."""
        if self.adaln_input is None:
            raise RuntimeError("peer AdaLN: the conditioning rows are not set")
        proj, bias_slot = self.adaln[u.index]
        a = self.adaln_input
        out = torch.empty(a.shape[0], proj.slot.rows, dtype=torch.bfloat16, device=self.device)
        self.comm_stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.comm_stream):
            if u.gather_event is not None:
                self.comm_stream.wait_event(u.gather_event)
            bias = u.slot_full(u.full_hi, bias_slot) if bias_slot is not None else None
            proj.run(self.hi_mem, a, bias, out)
            ev = torch.cuda.Event()
            ev.record(self.comm_stream)
        out.record_stream(self.comm_stream)
        a.record_stream(self.comm_stream)
        u.gather_event = ev
        u.adaln_rows = out

    def take_adaln_rows(self, u: Unit) -> Optional[torch.Tensor]:
        rows, u.adaln_rows = u.adaln_rows, None
        return rows

    def prefetch(self, u: Unit, forward: bool = False) -> None:
        """Start the all-gather of ``u`` on the communication stream (no-op if in flight/done)."""
        if self.world == 1 or u.full_hi is not None:
            return
        if self.peer:
            fused = self._fused_adaln(u, forward)
            full = torch.empty(u.numel_full, dtype=torch.bfloat16, device=self.device)
            self.comm_stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.comm_stream):
                (self.gather_plans_fwd if fused else self.gather_plans)[u.index].run(self.hi_mem, full)
                ev = torch.cuda.Event()
                ev.record(self.comm_stream)
            full.record_stream(self.comm_stream)
            u.gather_event = ev
            u.full_hi = full
            u.partial_gather = fused
            if fused and self.adaln_input is not None:
                self._adaln_projection(u)
            return
        packed = torch.empty(self.world * u.numel_shard, dtype=torch.bfloat16, device=self.device)
        full = torch.empty(u.numel_full, dtype=torch.bfloat16, device=self.device)

        def run():
            dist.all_gather_into_tensor(packed, u.hi, group=self.group)
            pk = packed.view(self.world, u.numel_shard)
            for s in u.slots:
                unpack_rows(pk, s, u.slot_full(full, s), self.world)

        if self.comm_stream is None:
            run()
        else:
            self.comm_stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.comm_stream):
                run()
                ev = torch.cuda.Event()
                ev.record(self.comm_stream)
            packed.record_stream(self.comm_stream)
            full.record_stream(self.comm_stream)
            u.gather_event = ev
        u.full_hi = full

    def release(self, u: Unit) -> None:
        """Drop the gathered weights of ``u`` (world > 1); the module keeps an empty placeholder."""
        if self.world == 1:
            return
        u.full_hi = None
        u.adaln_rows = None
        u.partial_gather = False
        self.bind_weights(u, None)

    # ---------------------------------------------------------------- gradients
    def attach_grads(self, u: Unit, zero: bool = True) -> None:
        """Give every parameter of ``u`` a ``.grad`` view of the unit's flat bf16 gradient (zeroed
        unless ``zero`` is False: gradient accumulation with one rank)."""
        if self.peer:
            cur = torch.cuda.current_stream(self.device)
            if u.index == len(self.units) - 1:
                slot = 0
                if self._begin_event is not None:
                    cur.wait_event(self._begin_event)
            else:
                slot = 1 + self._ring_next % (self.GRAD_SLOTS - 1)
                self._ring_next += 1
                last = self._slot_last.get(slot)
                if last is not None:
                    # every rank has finished reading this slot once any later reduction barrier passed
                    if self._latest is None or self._latest[0] <= last:
                        self.comm_stream.wait_stream(cur)
                        with torch.cuda.stream(self.comm_stream):
                            self.grad_mem.barrier(2)
                            ev = torch.cuda.Event()
                            ev.record(self.comm_stream)
                        self._latest = (self.n_reduce, ev)
                        self._slot_last = {k: v for k, v in self._slot_last.items() if v >= self.n_reduce}
                    cur.wait_event(self._latest[1])
            # always zeroed: the previous contents were already reduced into the fp32 shard
            u.full_grad = self.grad_mem.view(slot * self.slot_elems * 2, u.numel_full, torch.bfloat16)
            u.full_grad.zero_()
            u.grad_slot = slot
            for s in u.slots:
                getattr(s.module, s.attr).grad = u.slot_full(u.full_grad, s)
            return
        if u.full_grad is None:
            u.full_grad = torch.zeros(u.numel_full, dtype=torch.bfloat16, device=self.device)
        elif zero:
            u.full_grad.zero_()
        for s in u.slots:
            getattr(s.module, s.attr).grad = u.slot_full(u.full_grad, s)

    def detach_grads(self, u: Unit) -> None:
        for s in u.slots:
            getattr(s.module, s.attr).grad = None

    def reduce_grads(self, u: Unit, accumulate: bool = False) -> None:
        """world > 1: fp32 reduce-scatter of the unit's gradient into ``u.grad_shard`` (async on the
        communication stream).  world == 1: the bf16 gradient stays as is."""
        self.detach_grads(u)
        if self.world == 1:
            return
        if self.peer:
            c = self.n_reduce
            self.n_reduce += 1
            out = torch.zeros(u.numel_shard, dtype=torch.float32, device=self.device)
            self.comm_stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.comm_stream):
                self.grad_mem.barrier(2)  # every rank's gradient of this unit is complete
                ev = torch.cuda.Event()
                ev.record(self.comm_stream)
                self._latest = (c, ev)
                self.reduce_plans[u.index].run(self.slot_ptrs[u.grad_slot], out)
                self._slot_last[u.grad_slot] = c
                if u.grad_shard is None or not accumulate:
                    u.grad_shard = out
                else:
                    u.grad_shard.add_(out)
            out.record_stream(self.comm_stream)
            u.full_grad = None
            return
        g = u.full_grad
        u.full_grad = None
        packed = torch.zeros(self.world * u.numel_shard, dtype=torch.float32, device=self.device)
        out = torch.empty(u.numel_shard, dtype=torch.float32, device=self.device)

        def run():
            pk = packed.view(self.world, u.numel_shard)
            for s in u.slots:
                pack_rows(pk, s, u.slot_full(g, s), self.world)
            dist.reduce_scatter_tensor(out, packed, op=dist.ReduceOp.SUM, group=self.group)
            if self.replicate_group is not None:
                dist.all_reduce(out, op=dist.ReduceOp.SUM, group=self.replicate_group)
            if u.grad_shard is None or not accumulate:
                u.grad_shard = out
            else:
                u.grad_shard.add_(out)

        if self.comm_stream is None:
            run()
            return
        self.comm_stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.comm_stream):
            run()
        g.record_stream(self.comm_stream)
        packed.record_stream(self.comm_stream)
        out.record_stream(self.comm_stream)

    def wait_comm(self) -> None:
        if self.comm_stream is not None and self.world > 1:
            torch.cuda.current_stream(self.device).wait_stream(self.comm_stream)

    def grad_of(self, u: Unit) -> torch.Tensor:
        """Gradient in the shard layout (bf16 full buffer when world == 1, fp32 shard otherwise)."""
        return u.full_grad if self.world == 1 else u.grad_shard

    # ---------------------------------------------------------------- state dict
    def full_state_dict(self, to_cpu: bool = True) -> Dict[str, torch.Tensor]:
        """fp32 full weights of every parameter (gathers all shards; collective when world > 1)."""
        from ..optim.flat_ops import join_master
        if self.before_read is not None:
            self.before_read()
        out = {}
        for u in self.units:
            x = join_master(u.hi, u.lo)
            if self.world > 1:
                full = torch.empty(self.world * u.numel_shard, dtype=torch.float32, device=self.device)
                dist.all_gather_into_tensor(full, x, group=self.group)
                pk = full.view(self.world, u.numel_shard)
            else:
                pk = x.view(1, u.numel_shard)
            for s in u.slots:
                t = torch.empty(s.shape, dtype=torch.float32, device=x.device)
                unpack_rows(pk, s, t, self.world)
                out[s.name] = t.cpu() if to_cpu else t
        return out

    def load_full_state_dict(self, sd: Dict[str, torch.Tensor], strict: bool = False) -> List[str]:
        """Load full fp32 weights into the local shards; unmatched parameters keep their values.
        Returns the names that were missing from ``sd``."""
        from ..optim.flat_ops import join_master
        missing = []
        for u in self.units:
            x = join_master(u.hi, u.lo).clone()
            for s in u.slots:
                t = sd.get(s.name)
                if t is None:
                    missing.append(s.name)
                    continue
                t = t.reshape(s.rows, s.cols).float().cpu()
                pad = torch.zeros(s.rows_pad, s.cols)
                pad[:s.rows] = t
                mine = pad[self.rank * s.shard_rows:(self.rank + 1) * s.shard_rows]
                n = s.shard_rows * s.cols
                x[s.shard_off:s.shard_off + n] = mine.reshape(-1).to(x.device)
            set_master(u, x)
            if self.world == 1:
                self.bind_weights(u, u.hi)
        if strict and missing:
            raise KeyError(f"missing parameters: {missing[:8]}")
        return missing


def join_master_cpu(hi: torch.Tensor, lo: torch.Tensor) -> torch.Tensor:
    h = hi.cpu().view(torch.int16).to(torch.int32) & 0xFFFF
    l = lo.cpu().view(torch.int16).to(torch.int32) & 0xFFFF
    return ((h << 16) | l).view(torch.float32)


def split_master_cpu(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    b = x.float().contiguous().view(torch.int32)
    hi = ((b >> 16) & 0xFFFF).to(torch.int16).view(torch.bfloat16)
    lo = (b & 0xFFFF).to(torch.int16)
    return hi, lo


def set_master(u: Unit, x: torch.Tensor) -> None:
    """Write fp32 shard values ``x`` into ``u.hi`` / ``u.lo`` (``lo`` may live in host memory)."""
    from ..optim.flat_ops import split_master
    lo_dev = torch.empty(x.numel(), dtype=torch.int16, device=x.device)
    split_master(x, u.hi, lo_dev)
    u.lo.copy_(lo_dev)
