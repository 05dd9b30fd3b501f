"""One optimizer step through the engine, with the reference trainer's safety semantics.

``StepRunner.train_step(host_batch)`` is the public per-step call (reference: PanVideoTrainer.train_step,
train.py:949-1055): copy the step's inputs host->device, forward+backward, global grad norm and clip
coefficient on the device, a host read of loss and norm, a cross-rank vote on whether the update is
finite (every rank must agree before the optimizer runs: train.py:1000-1023), the optimizer step
(skipped, with gradients dropped, when not finite), then the learning-rate schedule.
"""
from __future__ import annotations

import math
from typing import Callable, Dict, Optional

import torch
import torch.distributed as dist

from ..data.synthetic import batch_to_device
from .engine import TrainEngine


class StepRunner:
    def __init__(self, engine: TrainEngine, lr_lambda: Optional[Callable[[int], float]] = None,
                 base_lr: Optional[float] = None, cpu_group=None):
        self.engine = engine
        self.lr_lambda = lr_lambda or (lambda step: 1.0)
        self.base_lr = engine.optim.lr if base_lr is None else base_lr
        self.cpu_group = cpu_group
        self.global_step = 0
        dev = engine.device
        pin = dev.type == "cuda"
        self.loss_host = torch.zeros(2, dtype=torch.float32, pin_memory=pin)
        self.engine.set_lr(self.base_lr * self.lr_lambda(0))
        self.skipped = 0
        self._events = None

    def phase_times(self) -> Dict[str, float]:
        """Device milliseconds of the last step's phases (call after a synchronize)."""
        ev = self._events
        if ev is None:
            return {}
        return {"forward_backward": ev[0].elapsed_time(ev[1]), "grad_norm": ev[1].elapsed_time(ev[2]),
                "optimizer": ev[3].elapsed_time(ev[4])}

    def device_step(self, batch_dev, poison: bool = False) -> Dict:
        """One optimizer step over ``batch_dev`` (a device batch, or a list of micro-batches for
        gradient accumulation).  ``poison`` makes this rank vote the update non-finite (host-side
        fault injection)."""
        eng = self.engine
        micro = batch_dev if isinstance(batch_dev, (list, tuple)) else [batch_dev]
        if eng.accum_steps != len(micro):
            eng.set_accumulation(len(micro))
        timing = eng.device.type == "cuda"
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)] if timing else None
        if timing:
            ev[0].record()
        loss = None
        for k, b in enumerate(micro):
            lk = eng.forward_backward(b, micro_step=k)
            loss = lk if loss is None else loss + lk
        loss = loss / len(micro)
        if timing:
            ev[1].record()
        norm_clip = eng.grad_norm()
        if timing:
            ev[2].record()
        self.loss_host[0].copy_(loss, non_blocking=True)
        self.loss_host[1].copy_(norm_clip[0], non_blocking=True)
        if eng.device.type == "cuda":
            torch.cuda.current_stream(eng.device).synchronize()
        loss_v, norm_v = float(self.loss_host[0]), float(self.loss_host[1])
        ok = math.isfinite(loss_v) and math.isfinite(norm_v) and not poison
        if eng.world > 1:
            flag = torch.tensor([int(ok)], dtype=torch.int32)
            if self.cpu_group is not None:
                dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.cpu_group)
            else:
                f = flag.to(eng.device)
                dist.all_reduce(f, op=dist.ReduceOp.MIN, group=eng.group)
                flag = f.cpu()
            ok = bool(flag.item())
        if timing:
            ev[3].record()
        if ok:
            eng.optimizer_step()
        else:
            self.skipped += 1
        if timing:
            ev[4].record()
        self._events = ev
        eng.zero_grad()
        self.global_step += 1
        lr = self.base_lr * self.lr_lambda(self.global_step)
        eng.set_lr(lr)
        return dict(loss=loss_v, grad_norm=norm_v, lr=lr, step_skipped=not ok)

    def train_step(self, host_batch) -> Dict:
        """Host batch (or list of micro-batches) in, pinned CPU tensors; metrics out (host floats)."""
        if isinstance(host_batch, (list, tuple)):
            dev = [batch_to_device(b, self.engine.device, non_blocking=True) for b in host_batch]
        else:
            dev = batch_to_device(host_batch, self.engine.device, non_blocking=True)
        return self.device_step(dev)

    def state_dict(self) -> Dict:
        return {"last_epoch": self.global_step}

    def load_state_dict(self, sd: Dict) -> None:
        self.global_step = int(sd["last_epoch"])
        self.engine.set_lr(self.base_lr * self.lr_lambda(self.global_step))
