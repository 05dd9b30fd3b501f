"""Learning-rate schedules (reference: train.py:415-452 and pan/optim/patch_lr_scheduler.py).

Linear warmup from ``warmup_start_ratio`` to 1 over ``warmup_steps`` (``progress = step / (warmup - 1)``),
then constant, linear or cosine decay to ``decay_floor_ratio`` over ``decay_steps`` (default
``max_steps - warmup_steps``).  The multiplier is computed on the host; the trainer writes
``base_lr * lambda(step)`` into a device scalar so the optimizer kernels never sync.
"""
from __future__ import annotations

import math
from typing import Callable, Dict, Optional

import torch

LR_SCHEDULER_TYPES = ("constant_with_warmup", "linear_decay", "cosine_decay")


def make_lr_lambda(scheduler_type: str, warmup_steps: int, decay_steps: Optional[int], max_steps: int,
                   warmup_start_ratio: float, decay_floor_ratio: float) -> Callable[[int], float]:
    if scheduler_type not in LR_SCHEDULER_TYPES:
        raise ValueError(f"learning-rate schedule {scheduler_type!r} is not one of {LR_SCHEDULER_TYPES}")
    eff_decay = decay_steps if decay_steps is not None else max(max_steps - warmup_steps, 0)

    def lr_lambda(step: int) -> float:
        if warmup_steps > 0 and step < warmup_steps:
            if warmup_steps == 1:
                return 1.0
            p = step / float(warmup_steps - 1)
            return warmup_start_ratio * (1.0 - p) + p
        if scheduler_type == "constant_with_warmup":
            return 1.0
        if eff_decay <= 1:
            return decay_floor_ratio
        d = min(max(step - warmup_steps, 0), eff_decay - 1)
        p = d / float(eff_decay - 1)
        if scheduler_type == "linear_decay":
            return (1.0 - p) + decay_floor_ratio * p
        return decay_floor_ratio + (1.0 - decay_floor_ratio) * 0.5 * (1.0 + math.cos(math.pi * p))

    return lr_lambda


def lr_lambda_from_config(tr: Dict) -> Callable[[int], float]:
    return make_lr_lambda(tr.get("lr_scheduler_type", "constant_with_warmup"), int(tr.get("warmup_steps", 500)),
                          tr.get("lr_decay_steps"), int(tr.get("max_steps", 10000)),
                          float(tr.get("lr_warmup_start_ratio", 0.0)), float(tr.get("lr_decay_floor_ratio", 0.3)))


class HostLambdaLR:
    """``LambdaLR``-like scheduler whose learning rate lives in a device scalar (no host syncs)."""

    def __init__(self, base_lr: float, lr_lambda: Callable[[int], float], lr_tensor: Optional[torch.Tensor] = None):
        self.base_lr = base_lr
        self.lr_lambda = lr_lambda
        self.last_epoch = 0
        self.lr_tensor = lr_tensor
        self._apply()

    def _apply(self):
        if self.lr_tensor is not None:
            self.lr_tensor.fill_(self.get_last_lr()[0])

    def get_last_lr(self):
        return [self.base_lr * self.lr_lambda(self.last_epoch)]

    def step(self):
        self.last_epoch += 1
        self._apply()

    def state_dict(self):
        return {"last_epoch": self.last_epoch}

    def load_state_dict(self, sd):
        self.last_epoch = int(sd["last_epoch"])
        self._apply()
