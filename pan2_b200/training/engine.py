"""Training engine: sharded units, block-level activation checkpointing and the fused optimizer step.

This is the B200 restatement of the reference trainer's model wrapping and step
(train.py:572-1055): FSDP2 + ``checkpoint_wrapper`` + ``torch.optim.Muon``/``AdamW`` become

* one :class:`~pan2_b200.parallel.sharded.Unit` per joint block plus a root unit, with exact fp32
  masters stored as (bf16 hi, 16-bit lo) shards;
* :class:`BlockCheckpoint`, an autograd node per block that gathers the block's weights (prefetching
  the next block on a communication stream), runs the fused forward without saving activations,
  and in backward re-gathers, recomputes, back-propagates into the block's flat bf16 gradient and
  launches the fp32 reduce-scatter while the previous block computes;
* a flat optimizer over the shards: Nesterov-momentum Muon with Gram Newton-Schulz on tcgen05
  batched GEMMs (chunked QKV / out-projection locally, other matrices gathered to an owner rank
  with all-to-all, as in patch_muon.py:174-268) and fused AdamW for everything else; learning rate
  and clip coefficient stay on the device;
* optional host offload of ``lo`` and the optimizer state (pinned memory, streamed per unit on
  copy-engine streams), chosen automatically when the GPU cannot hold a full replica's state —
  the 29B model on one or two B200s.
"""
from __future__ import annotations

import math
import os
import threading
import weakref
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import torch
import torch.distributed as dist
import torch.nn as nn

from ..models.transformer import PanVideoDiffusionTransformer, JointAttentionBlock
from ..models.packed import PackedSequenceParams
from ..ops._ext import ext
from ..optim import flat_ops as F
from ..optim.muon import adjust_lr_scale, chunk_view, gram_newton_schulz
from ..parallel.collectives import all_to_all_list
from ..parallel.sharded import ShardedModel, Unit, build_unit


def _align256(n: int) -> int:
    return (int(n) + 255) // 256 * 256


def muon_exchange_layout(remote, world: int) -> dict:
    """Byte offsets of one unit's distributed-Muon buffers (identical on every rank).

    ``remote`` lists the unit's Muon matrices that need the whole matrix on one rank, in slot order;
    matrix j belongs to owner ``j % world``.  The exchange region holds, per matrix, this rank's
    ``shard_rows x cols`` bf16 momentum rows at ``xoff[j]``; an owner's result region holds each
    of its matrices whole (``rows_pad x cols`` bf16) at ``roff[j]``.  Offsets are 256-byte aligned."""
    xoff, off = [], 0
    for s in remote:
        xoff.append(off)
        off += _align256(s.shard_rows * s.cols * 2)
    roff, per_owner = [], [0] * world
    for j, s in enumerate(remote):
        roff.append(per_owner[j % world])
        per_owner[j % world] += _align256(s.rows_pad * s.cols * 2)
    return dict(xoff=xoff, x_bytes=off, roff=roff, r_bytes=max(per_owner) if per_owner else 0, plans={})


class _Root(nn.Module):
    """Everything outside the joint blocks, as one parameter unit (names match the model)."""

    def __init__(self, model: PanVideoDiffusionTransformer):
        super().__init__()
        for name, child in model.named_children():
            if name != "blocks":
                self.add_module(name, child)


@dataclass
class OptimConfig:
    lr: float = 1e-5
    weight_decay: float = 0.05
    use_muon: bool = True
    momentum: float = 0.95
    adamw_betas: tuple = (0.95, 0.95)
    adamw_eps: float = 1e-8
    max_grad_norm: float = 1.0
    adjust_lr_fn: str = "match_rms_adamw"


class BlockCheckpoint(torch.autograd.Function):
    """Activation-checkpointed joint block driven by the engine's gather / reduce-scatter."""

    @staticmethod
    def forward(ctx, engine: "TrainEngine", idx: int, x, ln_stats, vec):
        sm = engine.sharded
        u = sm.units[idx]
        engine._wait_update(u)
        if idx > 0:
            engine._wait_update(sm.units[idx - 1])  # its gradient buffer receives this block's checkpoint
        sm.gather(u, forward=True)
        if idx + 1 < engine.n_blocks:
            sm.prefetch(sm.units[idx + 1], forward=True)
        blk = engine.model.blocks[idx]
        video_mod = sm.take_adaln_rows(u)
        with torch.no_grad():
            y, st = blk.forward_packed(x, ln_stats, vec, engine.meta, attn_fn=engine._attention_keeper(idx),
                                       video_mod=video_mod)
        sm.release(u)
        ctx.engine, ctx.idx = engine, idx
        stash = engine.stash_checkpoint(idx, x, ln_stats)
        if stash is None:
            ctx.save_for_backward(x, ln_stats, vec)
            ctx.stash = None
        else:
            ctx.save_for_backward(vec)
            ctx.stash = stash
        ctx.mark_non_differentiable(st)
        return y, st

    @staticmethod
    def backward(ctx, gy, _gst):
        engine, idx = ctx.engine, ctx.idx
        sm = engine.sharded
        u = sm.units[idx]
        if ctx.stash is None:
            x, ln_stats, vec = ctx.saved_tensors
        else:
            (vec,) = ctx.saved_tensors
            x, ln_stats = ctx.stash
            ctx.stash = None
        sm.gather(u)
        if idx > 0:
            sm.prefetch(sm.units[idx - 1])
        blk = engine.model.blocks[idx]
        x_ = x.detach().requires_grad_(True)
        vec_ = vec.detach().requires_grad_(True)
        sm.attach_grads(u, zero=not engine.accumulating)
        params = [getattr(s.module, s.attr) for s in u.slots]
        with torch.enable_grad():
            y, _ = blk.forward_packed(x_, ln_stats, vec_, engine.meta, attn_fn=engine._attention_replayer(idx))
        torch.autograd.backward([y], [gy], inputs=[x_, vec_] + params)
        sm.reduce_grads(u, accumulate=engine.accumulating)
        sm.release(u)
        return None, None, x_.grad, None, vec_.grad


class BlockKeepGraph(torch.autograd.Function):
    """Joint block without activation checkpointing: the forward keeps the block's autograd graph
    (every activation, and the gathered weights it saved), the backward runs it without
    recomputing.  Memory grows with every block, so this suits small models only."""

    @staticmethod
    def forward(ctx, engine: "TrainEngine", idx: int, x, ln_stats, vec):
        sm = engine.sharded
        u = sm.units[idx]
        engine._wait_update(u)
        sm.gather(u)
        if idx + 1 < engine.n_blocks:
            sm.prefetch(sm.units[idx + 1])
        blk = engine.model.blocks[idx]
        x_ = x.detach().requires_grad_(True)
        vec_ = vec.detach().requires_grad_(True)
        with torch.enable_grad():
            y, st = blk.forward_packed(x_, ln_stats, vec_, engine.meta)
        ctx.full = u.full_hi  # the graph holds views of these weights already; rebound in backward
        sm.release(u)
        ctx.engine, ctx.idx, ctx.graph = engine, idx, (x_, vec_, y)
        ctx.mark_non_differentiable(st)
        return y.detach(), st

    @staticmethod
    def backward(ctx, gy, _gst):
        engine, idx = ctx.engine, ctx.idx
        sm = engine.sharded
        u = sm.units[idx]
        x_, vec_, y = ctx.graph
        ctx.graph = None
        u.full_hi, full = ctx.full, ctx.full
        ctx.full = None
        sm.bind_weights(u, full)
        sm.attach_grads(u, zero=not engine.accumulating)
        params = [getattr(s.module, s.attr) for s in u.slots]
        torch.autograd.backward([y], [gy], inputs=[x_, vec_] + params)
        sm.reduce_grads(u, accumulate=engine.accumulating)
        sm.release(u)
        return None, None, x_.grad, None, vec_.grad


def _host_available_bytes() -> Optional[int]:
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) * 1024
    except OSError:
        return None
    return None


class _HostArena:
    """One page-locked host allocation that the offloaded state is carved from.

    The caching pinned-memory allocator rounds every block up to a power of two, which for the
    1-4 GB per-unit moments of the 29B model costs up to ~1.7x the state in locked host memory;
    here the state is one exact-size pageable allocation registered with the driver once, and
    every unit's tensors are 256-byte aligned views of it."""

    def __init__(self, nbytes: int):
        self.size = int(nbytes)
        self.buf = torch.empty(self.size, dtype=torch.uint8)
        self.off = 0
        self.registered = False
        ptr = self.buf.data_ptr()
        if self.size > 0 and int(torch.cuda.cudart().cudaHostRegister(ptr, self.size, 0)) == 0:
            self.registered = True
            weakref.finalize(self, _host_unregister, ptr)
        else:
            self.buf = None  # registration refused: the state falls back to pinned allocations

    def take(self, n: int, dtype) -> Optional[torch.Tensor]:
        nbytes = n * torch.empty(0, dtype=dtype).element_size()
        start = (self.off + 255) // 256 * 256
        if not self.registered or start + nbytes > self.size:
            return None
        self.off = start + nbytes
        t = self.buf[start:start + nbytes].view(dtype)
        t.zero_()
        return t


def _host_unregister(ptr: int) -> None:
    torch.cuda.cudart().cudaHostUnregister(ptr)


def _local_ranks() -> int:
    return int(os.environ.get("LOCAL_WORLD_SIZE", "1"))


def _hbm_bytes(device) -> int:
    if device.type != "cuda":
        return 1 << 62
    free, total = torch.cuda.mem_get_info(device)
    return total


class TrainEngine:
    """Owns the model, its sharded units and the optimizer state; runs one training step."""

    DEFER_ENQUEUE_TIMEOUT_S = 600.0  # host-side bound on waiting for the optimizer thread

    def __init__(self, arch: dict, device: torch.device, *, group: Optional[dist.ProcessGroup] = None,
                 seed: int = 42, optim: Optional[OptimConfig] = None, offload: str = "auto",
                 activation_bytes_estimate: int = 0, replicate_group: Optional[dist.ProcessGroup] = None,
                 offload_gpu_bytes: Optional[int] = None):
        self.device = device
        self.group = group
        self.replicate_group = replicate_group
        self.world = dist.get_world_size(group) if (group is not None and dist.is_initialized()) else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        self.optim = optim or OptimConfig()
        self.arch = dict(arch)
        self.meta: Optional[PackedSequenceParams] = None
        self.step_count = 0
        self.host_bytes_planned = 0
        self._arena: Optional[_HostArena] = None
        # skeleton on the meta device, then each unit materialised on the device with its own seed
        with torch.device("meta"):
            model = PanVideoDiffusionTransformer(**arch)
        self.n_blocks = len(model.blocks)
        units: List[Unit] = []
        blk_opts = dict(attention_backend=model.attention_backend, mlp_ratio=arch.get("mlp_ratio", 8.0),
                        context_mlp_ratio=arch.get("context_mlp_ratio", 4.0),
                        zero_init_modulation=arch.get("zero_init_modulation", True),
                        text_modulation_timestep_dependent=arch.get("text_modulation_timestep_dependent", False))
        total = sum(p.numel() for p in model.parameters())
        self.total_params = total
        self.offload = self._plan_offload(total, offload, activation_bytes_estimate)
        # GPU bytes left for offloadable state (lo halves, optimizer state) after the resident
        # weights, gradients and the activation reserve; the rest goes to pinned host memory.
        self._gpu_budget = 0
        if self.offload and device.type == "cuda":
            resident = total * 2 / self.world + (total * 2 if self.world == 1 else total * 4 / self.world)
            self._gpu_budget = int(_hbm_bytes(device) - resident - activation_bytes_estimate - 8e9)
            if offload_gpu_bytes is not None:
                self._gpu_budget = int(offload_gpu_bytes)
            from ..optim.muon import use_muon_for
            n_muon = sum(p.numel() for n, p in model.named_parameters()
                         if self.optim.use_muon and use_muon_for(n, tuple(p.shape)))
            state = (total * 2 + n_muon * 4 + (total - n_muon) * 8) / self.world
            self.host_bytes_planned = max(0, int(state - max(self._gpu_budget, 0)))
            avail = _host_available_bytes()
            if avail is not None and self.host_bytes_planned > 0.85 * avail / max(1, _local_ranks()):
                raise MemoryError(
                    f"offloaded optimizer state needs {self.host_bytes_planned / 1e9:.0f} GB of pinned host memory per "
                    f"rank but only {avail / 1e9:.0f} GB are available on this host")
        # Offloadable state (lo halves, optimizer state) takes the GPU budget in the order the next
        # step's forward needs the units, each unit whole: the root first (with deferred updates its
        # update gates the embedding that starts every forward), then the blocks in forward order;
        # the rest lives in pinned host memory and streams.  The root is built last, so its share
        # is set aside now.
        self._soff: Dict[int, int] = {}
        root_reserve = 0
        if self.offload and device.type == "cuda":
            root_reserve = min(max(self._gpu_budget, 0), self._offloadable_bytes(
                [(n, tuple(p.shape)) for n, p in model.named_parameters() if not n.startswith("blocks.")]))
            self._gpu_budget -= root_reserve
        for i in range(self.n_blocks):
            torch.manual_seed(seed * 1000003 + i)
            with torch.device(device):
                blk = JointAttentionBlock(model.hidden_size, model.num_attention_heads, **blk_opts)
            model.blocks[i] = blk
            units.append(self._materialise(i, f"blocks.{i}", blk, f"blocks.{i}."))
            self._alloc_unit_state(units[-1])
        torch.manual_seed(seed * 1000003 + self.n_blocks)
        with torch.device(device):
            small = PanVideoDiffusionTransformer(**{**arch, "num_layers": 0})
        for name, child in small.named_children():
            if name != "blocks":
                setattr(model, name, child)
        root = _Root(model)
        self._gpu_budget += root_reserve
        units.append(self._materialise(self.n_blocks, "root", root, ""))
        self._alloc_unit_state(units[-1])
        self.model = model
        self.sharded = ShardedModel(units, group, device, self.offload, replicate_group)
        self.sharded.before_read = self.flush_updates
        for u in units:
            if self.world == 1:
                self.sharded.bind_weights(u, u.hi)
            else:
                self.sharded.bind_weights(u, None)
        # gathers / gradient reductions as peer-memory kernels when the shard group is one node
        self.peer_comm = False
        if self.world > 1 and device.type == "cuda" and os.environ.get("PAN_PEER_COMM", "1") != "0":
            # PAN_PEER_ADALN=1: the forward reads each block's AdaLN weight from the peers inside the
            # modulation projection instead of gathering it (parameter all-gather fused into the op)
            self.peer_comm = self.sharded.enable_peer_memory(
                peer_adaln=os.environ.get("PAN_PEER_ADALN", "0") == "1")
        self._muon_pm = None  # peer-mapped exchange / result regions of distributed Muon
        self._muon_layouts: Dict[int, dict] = {}
        self.stash_in_grads = self.world == 1
        # activation checkpointing of the joint blocks (set_activation_checkpointing)
        self.recompute_blocks = True
        self.keep_attention = False
        self._kept_attn: Dict[int, tuple] = {}
        self.accum_steps = 1
        self.accumulating = False
        if self.world == 1:  # persistent gradient buffers (they also hold activation checkpoints)
            for u in units:
                u.full_grad = torch.zeros(u.numel_full, dtype=torch.bfloat16, device=device)
        self.lr_t = torch.full((1,), self.optim.lr, dtype=torch.float32, device=device)
        self.norm_clip = torch.zeros(2, dtype=torch.float32, device=device)
        # deferred (overlapped) optimizer updates with host-offloaded state and one rank
        self.defer_optimizer = device.type == "cuda" and os.environ.get("PAN_DEFER_OPTIMIZER", "1") == "1"
        self._upd_events: Dict[int, torch.cuda.Event] = {}
        self._upd_ready: Dict[int, threading.Event] = {}
        self._upd_thread: Optional[threading.Thread] = None
        self._upd_error: Optional[BaseException] = None
        self._lr_used = torch.zeros(1, dtype=torch.float32, device=device)
        self._clip_used = torch.ones(1, dtype=torch.float32, device=device)
        self._lr_override = None
        self._partials = torch.zeros(len(units) * 256, dtype=torch.float32, device=device)
        if self.offload and device.type == "cuda":
            self._h2d = torch.cuda.Stream(device)
            self._d2h = torch.cuda.Stream(device)
            self._opt_stream = torch.cuda.Stream(device)
        # streamed optimizer state: two persistent device slots (unit i uses slot i % 2), so the
        # per-unit staging never goes through the caching allocator; _slot_free[s] marks the end of
        # the write-back that last read slot s
        self._slots: List[torch.Tensor] = []
        self._slot_free: List[Optional[torch.cuda.Event]] = [None, None]
        if self._peer_muon() and self.sharded.units:
            self._muon_layout(self.sharded.units[0])  # allocate now, before memory placement

    # ---------------------------------------------------------------- construction
    def _plan_offload(self, total: int, offload: str, act_bytes: int) -> bool:
        if offload in (True, "on", "true", "1"):
            return True
        if offload in (False, "off", "false", "0") or self.device.type != "cuda":
            return False
        per_rank = total / self.world
        grad_bytes = 2 if self.world == 1 else 4
        need = per_rank * (2 + 2 + grad_bytes + 4) + act_bytes + (2 if self.world == 1 else 0) * 0
        return need > 0.9 * _hbm_bytes(self.device)

    def _materialise(self, idx: int, name: str, module: nn.Module, prefix: str) -> Unit:
        u = build_unit(idx, name, module, self.world, prefix)
        x = torch.zeros(u.numel_shard, dtype=torch.float32, device=self.device)
        for s in u.slots:
            p = getattr(s.module, s.attr).detach().float().reshape(s.rows, s.cols)
            if s.rows_pad != s.rows:
                p = torch.cat([p, p.new_zeros(s.rows_pad - s.rows, s.cols)], 0)
            mine = p[self.rank * s.shard_rows:(self.rank + 1) * s.shard_rows]
            n = s.shard_rows * s.cols
            x[s.shard_off:s.shard_off + n] = mine.reshape(-1)
        u.hi = torch.empty(u.numel_shard, dtype=torch.bfloat16, device=self.device)
        u.lo = self._state_tensor(u.numel_shard, torch.int16)
        lo_dev = torch.empty(u.numel_shard, dtype=torch.int16, device=self.device)
        F.split_master(x, u.hi, lo_dev)
        u.lo.copy_(lo_dev)
        # free the fp32 initial values held by the module
        for s in u.slots:
            getattr(s.module, s.attr).data = torch.empty(0, dtype=torch.bfloat16, device=self.device)
        return u

    def _state_tensor(self, n: int, dtype) -> torch.Tensor:
        """Offloadable state: on the GPU while the budget lasts, else pinned host memory."""
        nbytes = n * torch.empty(0, dtype=dtype).element_size()
        if not self.offload or nbytes <= self._gpu_budget:
            self._gpu_budget -= nbytes if self.offload else 0
            return torch.zeros(n, dtype=dtype, device=self.device)
        if self._arena is None and self.host_bytes_planned > 0:
            # exact size of the planned host state plus alignment slack
            self._arena = _HostArena(int(self.host_bytes_planned * 1.01) + (256 << 20))
        t = self._arena.take(n, dtype) if self._arena is not None else None
        return t if t is not None else torch.zeros(n, dtype=dtype, pin_memory=True)

    def _offloadable_bytes(self, params) -> int:
        """Upper bound of the lo halves and optimizer state of ``params`` (name, shape) on this rank."""
        from ..optim.muon import use_muon_for
        total = 0
        for name, shape in params:
            rows = shape[0] if shape else 1
            n = -(-rows // self.world) * (int(math.prod(shape[1:])) if len(shape) >= 2 else 1) + 8
            muon = self.optim.use_muon and use_muon_for(name, shape)
            total += n * (2 + (4 if muon else 8))
        return total + (1 << 20)

    def _alloc_unit_state(self, u: Unit) -> None:
        """Compact per-unit state: Muon momentum for Muon slots, AdamW (m, v) for the others."""
        mo = ao = 0
        for s in u.slots:
            n = s.shard_rows * s.cols
            if self._is_muon(s):
                self._soff[id(s)] = mo
                mo += n
            else:
                self._soff[id(s)] = ao
                ao += n
        u.state["mom"] = self._state_tensor(mo, torch.float32) if mo else None
        u.state["m"] = self._state_tensor(ao, torch.float32) if ao else None
        u.state["v"] = self._state_tensor(ao, torch.float32) if ao else None

    def _is_muon(self, s) -> bool:
        return self.optim.use_muon and s.kind == "muon"

    # ---------------------------------------------------------------- step
    def set_context_parallel(self, group, size: int, rank: int) -> None:
        """Record the Ulysses context-parallel group.  Batches split by
        :func:`pan2_b200.data.cp_batch.strided_split` carry the group in their metadata, and the
        joint blocks then run attention through :func:`pan2_b200.parallel.ulysses.ulysses_attention`."""
        self.cp_group, self.cp_size, self.cp_rank = group, int(size), int(rank)
        if self.cp_size > 1 and self.arch.get("num_attention_heads", 32) % self.cp_size:
            raise ValueError(f"cp_size={size} must divide the {self.arch.get('num_attention_heads')} attention heads")
        if self.cp_size > 1 and self.keep_attention:
            raise ValueError("keeping attention outputs (use_dedicated_gradient_checkpointing) is not supported "
                             "with context parallelism (cp_size > 1)")

    def set_activation_checkpointing(self, enabled: bool = True, keep_attention: bool = False) -> None:
        """``enabled``: recompute each joint block's forward before its backward (the default);
        off, every block keeps its activations.  ``keep_attention``: selective checkpointing that
        keeps each block's attention output and log-sum-exp from the forward, so the recompute skips
        the attention forward (about 0.8 GB per block at 95k tokens of the 29B model); the QKV
        projection is still recomputed (reference: train.py:817-845)."""
        self.recompute_blocks = bool(enabled)
        self.keep_attention = bool(keep_attention) and self.recompute_blocks
        if self.keep_attention and getattr(self, "cp_size", 1) > 1:
            raise ValueError("keeping attention outputs (use_dedicated_gradient_checkpointing) is not supported "
                             "with context parallelism (cp_size > 1)")

    def _attention_keeper(self, idx: int):
        """Block ``idx``'s attention for the checkpointed forward: records ``(o, lse)``."""
        if not self.keep_attention:
            return None
        from ..ops.attention import attention_forward

        def run(q, k, v, meta):
            o, lse = attention_forward(q, k, v, meta.joint_lens)
            self._kept_attn[idx] = (o, lse)
            return o
        return run

    def _attention_replayer(self, idx: int):
        """Block ``idx``'s attention for the recompute: the kept forward, the normal backward."""
        kept = self._kept_attn.pop(idx, None)
        if kept is None:
            return None
        from ..ops.attention import kept_attention
        o, lse = kept
        return lambda q, k, v, meta: kept_attention(q, k, v, o, lse, meta.joint_lens)

    def set_accumulation(self, steps: int) -> None:
        """Prepare for ``steps`` micro-batches per optimizer step.  With more than one, gradients
        persist across micro-batches, so activation checkpoints no longer live in gradient buffers."""
        self.accum_steps = max(1, int(steps))
        if self.accum_steps > 1:
            self.stash_in_grads = False

    def forward_backward(self, batch: dict, micro_step: int = 0) -> torch.Tensor:
        """Forward + backward of one packed batch; returns the (global-mean) loss as a device scalar.

        With gradient accumulation the loss is divided by the number of micro-batches and
        micro-batches after the first add into the gradients."""
        self.accumulating = micro_step > 0
        scale = 1.0 / self.accum_steps
        meta: PackedSequenceParams = batch["packed_seq_params"]
        self.meta = meta
        model = self.model
        sm = self.sharded
        root = sm.units[-1]
        self._wait_update(root)
        sm.begin_gathers()
        # peer AdaLN path: only with recomputed blocks (their backward gathers every weight) and at
        # most 8 conditioning rows (the projection kernel's limit)
        sm.adaln_on = bool(sm.adaln) and self.recompute_blocks and int(batch["timestep"].shape[0]) <= 8
        sm.adaln_input = None
        sm.gather(root)
        if self.n_blocks:
            sm.prefetch(sm.units[0], forward=True)
        sm.attach_grads(root, zero=not self.accumulating)
        x, ln_stats, vec = model.embed_packed(batch["hidden_states"], batch["timestep"], batch["text_states"], meta)
        if sm.adaln_on:
            sm.adaln_input = model.blocks[0].modulation.act(vec.detach()).to(torch.bfloat16).contiguous()
        self._kept_attn = {}
        block_fn = BlockCheckpoint if self.recompute_blocks else BlockKeepGraph
        for i in range(self.n_blocks):
            x, ln_stats = block_fn.apply(self, i, x, ln_stats, vec)
        sums = model.head_and_loss(x, ln_stats, vec, batch["target"], meta)
        glob = sums.detach().clone()
        if dist.is_initialized() and dist.get_world_size() > 1:
            # global mean over every rank's tokens (shard, replica and context-parallel ranks)
            dist.all_reduce(glob, op=dist.ReduceOp.SUM)
        loss = sums[0] * (scale / glob[1])
        loss.backward()
        sm.reduce_grads(root, accumulate=self.accumulating)
        sm.wait_comm()
        if self.world > 1:
            sm.release(root)
        return (glob[0] / glob[1]).detach()

    def stash_checkpoint(self, idx: int, x: torch.Tensor, ln_stats: torch.Tensor):
        """Keep block ``idx``'s input inside block ``idx-1``'s gradient buffer.

        With one rank every block has a persistent bf16 gradient buffer that is idle from the
        optimizer step until that block's backward.  Block ``idx``'s backward (which needs the
        checkpoint) always finishes before block ``idx-1``'s backward zeroes its buffer, so the
        checkpointed activations (44 x 0.78 GB for the 29B batch) cost no extra memory.
        """
        if self.world != 1 or idx == 0 or not self.stash_in_grads:
            return None
        buf = self.sharded.units[idx - 1].full_grad
        nx = x.numel()
        ns = ln_stats.numel() * 2  # fp32 -> bf16-sized slots
        if buf is None or nx + ns > buf.numel() or x.dtype != torch.bfloat16 or nx % 2:
            return None
        xs = buf[:nx].view(x.shape)
        xs.copy_(x)
        ss = buf[nx:nx + ns].view(torch.float32).view(ln_stats.shape)
        ss.copy_(ln_stats)
        return xs, ss

    def _cur_stream(self):
        return torch.cuda.current_stream(self.device) if self.device.type == "cuda" else None

    def grad_norm(self) -> torch.Tensor:
        """Global gradient L2 norm and clip coefficient (``self.norm_clip = [norm, clip]``)."""
        parts = self._partials.view(len(self.sharded.units), 256)
        for i, u in enumerate(self.sharded.units):
            F.sumsq_partial(self.sharded.grad_of(u), parts[i])
        if self.world > 1:
            dist.all_reduce(self._partials, op=dist.ReduceOp.SUM, group=self.group)
        F.norm_and_clip(self._partials, float(self.optim.max_grad_norm), self.norm_clip)
        return self.norm_clip

    def set_lr(self, lr: float) -> None:
        self.lr_t.fill_(lr)

    def _lr(self) -> torch.Tensor:
        return self._lr_override if self._lr_override is not None else self.lr_t

    def _wait_update(self, u: Unit) -> None:
        """Order the current stream after a deferred optimizer update of ``u`` (if one is pending).
        With the update enqueued from the optimizer thread, first wait (on the host, bounded) until
        that thread has enqueued the unit and recorded its completion event."""
        ready = self._upd_ready.pop(u.index, None)
        if ready is not None and not ready.wait(timeout=self.DEFER_ENQUEUE_TIMEOUT_S):
            raise RuntimeError(f"deferred optimizer: unit {u.index} was not enqueued within "
                               f"{self.DEFER_ENQUEUE_TIMEOUT_S} s")
        if self._upd_error is not None:
            err, self._upd_error = self._upd_error, None
            raise RuntimeError("deferred optimizer update failed on its enqueue thread") from err
        ev = self._upd_events.pop(u.index, None)
        if ev is not None:
            torch.cuda.current_stream(self.device).wait_event(ev)

    def flush_updates(self) -> None:
        """Wait for every deferred optimizer update (before reading weights or optimizer state)."""
        for u in self.sharded.units:
            self._wait_update(u)
        if self._upd_thread is not None:
            self._upd_thread.join()
            self._upd_thread = None

    def optimizer_step(self) -> None:
        self.sharded.end_gathers()
        if self._upd_thread is not None:  # a previous deferred step that no forward consumed
            self.flush_updates()
        self.step_count += 1
        units = self.sharded.units
        if not self.offload:
            clip = self.norm_clip[1:2] if self.optim.max_grad_norm > 0 else None
            for u in units:
                self._step_unit(u, u.lo, u.state, clip)
            return
        # streamed: H2D of unit i+1 overlaps compute of unit i; D2H after compute.  Tensors that
        # the placement kept on the GPU are used in place.  With one rank the whole pipeline runs
        # on side streams and overlaps the next forward, which waits per unit (root first, then the
        # blocks in forward order) right before it reads that unit's weights.  Its few thousand
        # launches and PCIe-paced copies are enqueued from a host thread of their own, so the main
        # thread goes on to enqueue the next step while this one's update streams.
        launch = torch.cuda.current_stream(self.device)
        deferred = self.defer_optimizer and self.world == 1
        if not deferred:
            clip = self.norm_clip[1:2] if self.optim.max_grad_norm > 0 else None
            self._stream_update(units, launch, self.lr_t, clip)
            return
        # private copies: the caller may change the learning rate right after this call
        self._lr_used.copy_(self.lr_t)
        self._clip_used.copy_(self.norm_clip[1:2])
        start = torch.cuda.Event()
        start.record(launch)  # everything the update reads is enqueued on `launch` before this point
        order = [units[-1]] + list(units[:-1])
        self._upd_events = {}
        self._upd_error = None
        ready = {u.index: threading.Event() for u in order}
        self._upd_ready = dict(ready)  # the forward pops from this copy; the thread signals `ready`
        clip = self._clip_used if self.optim.max_grad_norm > 0 else None

        dev_index = self.device.index if self.device.index is not None else torch.cuda.current_device()

        def run():
            try:
                torch.cuda.set_device(dev_index)
                self._opt_stream.wait_event(start)
                self._stream_update(order, self._opt_stream, self._lr_used, clip, publish=ready)
            except BaseException as e:  # surfaced by the next _wait_update
                self._upd_error = e
            finally:
                for ev in ready.values():
                    ev.set()

        self._upd_thread = threading.Thread(target=run, name="pan2-optimizer-enqueue", daemon=True)
        self._upd_thread.start()

    def _stream_update(self, units: List[Unit], cur, lr_t: torch.Tensor, clip,
                       publish: Optional[Dict[int, threading.Event]] = None) -> None:
        """The streamed update of ``units`` on stream ``cur``.  With ``publish`` (deferred mode) a
        completion event is recorded per unit and ``publish[unit]`` is set once it is."""
        self._lr_override = lr_t
        staged = {}

        def on_host(t):
            return t is not None and t.device.type == "cpu"

        def host_parts(u):
            parts = [("lo", None, u.lo)] if on_host(u.lo) else []
            return parts + [("state", k, v) for k, v in u.state.items() if on_host(v)]

        slots = self._staging_slots(max(sum(_align256(t.numel() * t.element_size()) for *_, t in host_parts(u))
                                        for u in units))

        def stage(i):
            u = units[i]
            parts = host_parts(u)
            self._h2d.wait_stream(cur)
            s = i % 2
            if parts and slots and self._slot_free[s] is not None:
                self._h2d.wait_event(self._slot_free[s])
            lo, st, views = u.lo, dict(u.state), []
            with torch.cuda.stream(self._h2d):
                off = 0
                for kind, k, t in parts:
                    nb = t.numel() * t.element_size()
                    if slots:
                        dev = slots[s][off:off + nb].view(t.dtype).view(t.shape)
                        dev.copy_(t, non_blocking=True)
                        off += _align256(nb)
                    else:  # no room for persistent slots: allocate per unit
                        dev = t.to(self.device, non_blocking=True)
                    views.append(dev)
                    if kind == "lo":
                        lo = dev
                    else:
                        st[k] = dev
                ev = torch.cuda.Event()
                ev.record(self._h2d)
            staged[i] = (lo, st, ev, parts, views)

        stage(0)
        for i, u in enumerate(units):
            if i + 1 < len(units):
                stage(i + 1)
            lo, st, ev, parts, views = staged.pop(i)
            cur.wait_event(ev)
            if not slots:
                for t in views:
                    t.record_stream(cur)
            with torch.cuda.stream(cur):
                self._step_unit(u, lo, st, clip)
            if publish is not None:
                done_u = torch.cuda.Event()
                done_u.record(cur)
                self._upd_events[u.index] = done_u
                publish[u.index].set()
            if parts:
                self._d2h.wait_stream(cur)
                with torch.cuda.stream(self._d2h):
                    for (_, _, host), dev in zip(parts, views):
                        host.copy_(dev, non_blocking=True)
                    done = torch.cuda.Event()
                    done.record(self._d2h)
                self._slot_free[i % 2] = done
                if not slots:
                    for t in views:
                        t.record_stream(self._d2h)
        self._lr_override = None
        # the host halves must be written back before the next step re-reads them
        cur.wait_stream(self._d2h)

    def _staging_slots(self, nbytes: int) -> List[torch.Tensor]:
        """The two device slots for streamed optimizer state (grown to ``nbytes`` each); empty when
        the GPU has no room, in which case units are staged through the caching allocator."""
        if nbytes <= 0:
            return []
        if self._slots and self._slots[0].numel() >= nbytes:
            return self._slots
        torch.cuda.current_stream(self.device).wait_stream(self._h2d)
        torch.cuda.current_stream(self.device).wait_stream(self._d2h)
        self._slots, self._slot_free = [], [None, None]
        try:
            self._slots = [torch.empty(nbytes, dtype=torch.uint8, device=self.device) for _ in range(2)]
        except torch.cuda.OutOfMemoryError:
            self._slots = []
        return self._slots

    def place_state(self, reserve_bytes: int) -> Dict[str, int]:
        """Move offloaded ``lo`` halves / optimizer state back to the GPU while free memory minus
        ``reserve_bytes`` allows (largest savings of PCIe traffic first: ``lo`` then momentum)."""
        if not self.offload or self.device.type != "cuda":
            return {}
        free = torch.cuda.mem_get_info(self.device)[0] - reserve_bytes
        moved = {"lo": 0, "state": 0}
        for u in self.sharded.units:
            nb = u.lo.numel() * 2
            if u.lo.device.type == "cpu" and nb < free:
                u.lo = u.lo.to(self.device)
                free -= nb
                moved["lo"] += nb
        for u in self.sharded.units:
            for k, v in list(u.state.items()):
                if v is not None and v.device.type == "cpu" and v.numel() * 4 < free:
                    u.state[k] = v.to(self.device)
                    free -= v.numel() * 4
                    moved["state"] += v.numel() * 4
        return moved

    def _step_unit(self, u: Unit, lo: torch.Tensor, st: Dict[str, torch.Tensor], clip) -> None:
        E = F
        o = self.optim
        g = self.sharded.grad_of(u)
        b1, b2 = o.adamw_betas
        muon_work = []
        lay = self._muon_layout(u) if self._peer_muon() else None
        n_remote = 0
        for s in u.slots:
            n = s.shard_rows * s.cols
            sl = slice(s.shard_off, s.shard_off + n)
            so = self._soff[id(s)]
            ss = slice(so, so + n)
            if self._is_muon(s):
                if lay is not None and not self._muon_local(s):
                    # straight into this rank's exchange region, where the matrix owner reads it
                    upd = self._muon_pm.view(lay["xoff"][n_remote], n, torch.bfloat16)
                    n_remote += 1
                else:
                    upd = torch.empty(n, dtype=torch.bfloat16, device=self.device)
                E.muon_momentum(st["mom"][ss], g[sl], clip, o.momentum, upd)
                muon_work.append((s, sl, upd))
            else:
                E.adamw_update(u.hi[sl], lo[sl], g[sl], st["m"][ss], st["v"][ss], clip, self._lr(), b1, b2,
                               o.adamw_eps, o.weight_decay, self.step_count)
        if not muon_work:
            return
        local, remote = [], []
        for item in muon_work:
            (local if self._muon_local(item[0]) else remote).append(item)
        for s, sl, upd in local:
            chunked = s.chunks is not None and s.chunks[0] == 0
            n_local = s.chunks[1] // self.world if chunked else 1
            mat = upd.view(s.shard_rows, s.cols)
            orth = (gram_newton_schulz(chunk_view(mat, n_local)).reshape(s.shard_rows, s.cols) if n_local > 1
                    else gram_newton_schulz(mat))
            shape = (s.rows // s.chunks[1], s.cols) if chunked else (s.rows, s.cols)
            E.muon_update(u.hi[sl], lo[sl], orth.reshape(-1), self._lr(), adjust_lr_scale(shape, o.adjust_lr_fn),
                          o.weight_decay)
        if remote:
            if lay is not None:
                self._muon_peer(u, lo, remote, lay)
            else:
                self._muon_all_to_all(u, lo, remote)

    def _muon_local(self, s) -> bool:
        """A Muon matrix each rank can orthogonalise alone: its row shard is a whole number of the
        independent row chunks (or there is one rank)."""
        return self.world == 1 or (s.chunks is not None and s.chunks[0] == 0 and s.chunks[1] % self.world == 0
                                   and s.rows == s.rows_pad)

    def _peer_muon(self) -> bool:
        return self.peer_comm and self.world > 1 and os.environ.get("PAN_PEER_MUON", "1") != "0"

    def _muon_layout(self, u: Unit) -> dict:
        """Byte offsets of unit ``u``'s distributed-Muon buffers, identical on every rank: the
        exchange region holds each remote matrix's momentum rows of this rank; matrix j of the unit
        belongs to owner j % world, whose result region holds the full orthogonalised matrix.
        The peer-mapped buffer is allocated at the first call for the largest unit."""
        lay = self._muon_layouts.get(u.index)
        if lay is not None:
            return lay
        from ..parallel.symm import PeerMemory
        for unit in self.sharded.units:
            remote = [s for s in unit.slots if self._is_muon(s) and not self._muon_local(s)]
            self._muon_layouts[unit.index] = muon_exchange_layout(remote, self.world)
        x_max = max(l["x_bytes"] for l in self._muon_layouts.values())
        r_max = max(l["r_bytes"] for l in self._muon_layouts.values())
        for l in self._muon_layouts.values():
            l["rbase"] = x_max
        self._muon_pm = PeerMemory(max(256, x_max + r_max), self.group, self.device)
        return self._muon_layouts[u.index]

    def _muon_peer(self, u: Unit, lo: torch.Tensor, work, lay: dict) -> None:
        """Distributed Muon over peer memory (reference: patch_muon.py:174-268, which moves the rows
        with two NCCL all-to-alls): the momentum kernel already wrote this rank's rows of every
        remote matrix into its exchange region; each owner gathers its matrices' rows from all ranks
        with peer loads straight into its result region, orthogonalises them in place, and every
        rank's update kernel reads its own rows from the owner's result region over NVLink."""
        from ..parallel.symm import _pack
        E = F
        o = self.optim
        W, me, pm = self.world, self.rank, self._muon_pm
        pm.barrier(0)  # every rank's momentum rows are in its exchange region
        for j, (s, sl, upd) in enumerate(work):
            if j % W != me:
                continue
            n = s.shard_rows * s.cols
            plan = lay["plans"].get(j)
            if plan is None:
                segs = [(lay["xoff"][j] // 2, r * n, n) for r in range(W)]
                plan = lay["plans"][j] = _pack(segs, list(range(W)), self.device)
            full = pm.view(lay["rbase"] + lay["roff"][j], s.rows_pad * s.cols, torch.bfloat16).view(s.rows_pad, s.cols)
            seg_t, prefix, total, seg_peer = plan
            ext().peer_gather(pm.peers, seg_t, seg_peer, prefix, total, full)
            real = full[:s.rows]
            if s.chunks is not None and s.chunks[0] == 0 and s.chunks[1] > 1:
                orth = gram_newton_schulz(chunk_view(real, s.chunks[1])).reshape(s.rows, s.cols)
            else:
                orth = gram_newton_schulz(real)
            real.copy_(orth)
            full[s.rows:].zero_()
        pm.barrier(1)  # every owner's orthogonalised matrices are ready
        ptrs = pm.handle.buffer_ptrs
        for j, (s, sl, upd) in enumerate(work):
            addr = ptrs[j % W] + lay["rbase"] + lay["roff"][j] + me * s.shard_rows * s.cols * 2
            shape = (s.rows // s.chunks[1], s.cols) if (s.chunks and s.chunks[0] == 0) else (s.rows, s.cols)
            ext().muon_update_peer(u.hi[sl], lo[sl], int(addr), self._lr(), adjust_lr_scale(shape, o.adjust_lr_fn),
                                   o.weight_decay)

    def _muon_all_to_all(self, u: Unit, lo: torch.Tensor, work) -> None:
        """Owner-rank orthogonalisation of row-sharded matrices (reference: patch_muon.py:174-268)."""
        E = F
        o = self.optim
        W = self.world
        for start in range(0, len(work), W):
            chunk = work[start:start + W]
            send = [chunk[j][2].view(chunk[j][0].shard_rows, chunk[j][0].cols) if j < len(chunk)
                    else torch.empty(0, dtype=torch.bfloat16, device=self.device) for j in range(W)]
            mine = chunk[self.rank] if self.rank < len(chunk) else None
            if mine is not None:
                s = mine[0]
                full = torch.empty(W * s.shard_rows, s.cols, dtype=torch.bfloat16, device=self.device)
                recv = list(full.split(s.shard_rows, 0))
            else:
                full = None
                recv = [torch.empty(0, dtype=torch.bfloat16, device=self.device) for _ in range(W)]
            all_to_all_list(recv, send, group=self.group)
            if full is not None:
                s = mine[0]
                real = full[:s.rows]
                if s.chunks is not None and s.chunks[0] == 0 and s.chunks[1] > 1:
                    orth = gram_newton_schulz(chunk_view(real, s.chunks[1])).reshape(s.rows, s.cols)
                else:
                    orth = gram_newton_schulz(real)
                full[:s.rows].copy_(orth)
                full[s.rows:].zero_()
            all_to_all_list(send, recv, group=self.group)
            for s, sl, upd in chunk:
                shape = (s.rows // s.chunks[1], s.cols) if (s.chunks and s.chunks[0] == 0) else (s.rows, s.cols)
                E.muon_update(u.hi[sl], lo[sl], upd, self._lr(), adjust_lr_scale(shape, o.adjust_lr_fn),
                              o.weight_decay)

    def zero_grad(self) -> None:
        for u in self.sharded.units:
            if self.world == 1:
                continue
            u.grad_shard = None

    def parameters_bytes(self) -> Dict[str, int]:
        us = self.sharded.units
        return dict(hi=sum(u.hi.numel() * 2 for u in us), lo=sum(u.lo.numel() * 2 for u in us))
