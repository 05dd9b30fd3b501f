"""Classifier-free guidance controls and spatiotemporal skip guidance (STG).

Semantics of the reference (pan/utils/inference_guidance.py:9-111):

* a :class:`GuidancePlan` makes CFG active at step ``i`` when ``i < end_step`` and (``i >= start_step``
  or a warmup scale above 1 is set) and ``i`` is outside the optional skip interval; elsewhere the
  positive prediction is used alone;
* before ``start_step`` the warmup scale replaces the guidance scale;
* CFG is ``neg + scale * (pos - neg)`` in the prediction dtype; STG then adds
  ``stg_scale * (pos - weak)`` in fp32 and casts back, where ``weak`` is the positive prediction of a
  forward that skips the given blocks (text-to-video only).  The order of these operations is part of
  the bf16 result.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from numbers import Integral, Real
from typing import Callable, Optional, Tuple

import torch

SCHEDULES = ("standard", "early_refine_2x")


def validate_sampling_extensions(num_steps: int, timestep_schedule: str = "standard") -> None:
    if timestep_schedule not in SCHEDULES:
        raise ValueError(f"unknown timestep_schedule {timestep_schedule!r}")
    if timestep_schedule == "early_refine_2x" and num_steps != 50:
        raise ValueError("early_refine_2x requires exactly 50 inference steps")


def _is_int(v) -> bool:
    return isinstance(v, Integral) and not isinstance(v, bool)


@dataclass(frozen=True)
class GuidancePlan:
    num_steps: int
    start_step: int
    end_step: int
    stg_scale: float
    skip_interval: Optional[Tuple[int, int]] = None
    warmup_scale: float = 1.0

    def active(self, i: int) -> bool:
        if not _is_int(i):
            raise ValueError("step_index must be an integer")
        if not 0 <= i < self.num_steps:
            raise ValueError("step_index is outside the scheduler's timestep sequence")
        in_window = i < self.end_step and (i >= self.start_step or self.warmup_scale > 1)
        skipped = self.skip_interval is not None and self.skip_interval[0] <= i < self.skip_interval[1]
        return in_window and not skipped

    def scale_at(self, i: int, guidance_scale: float) -> float:
        return self.warmup_scale if i < self.start_step else guidance_scale


def resolve_guidance_plan(num_steps: int, *, start_step: int = 0, end_step: Optional[int] = None,
                          stg_scale: float = 0.0, skip_interval=None, warmup_scale: float = 1.0) -> GuidancePlan:
    end_step = num_steps if end_step is None else end_step
    for name, v in (("num_steps", num_steps), ("start_step", start_step), ("end_step", end_step)):
        if not _is_int(v):
            raise ValueError(f"{name} must be an integer")
    if num_steps < 1:
        raise ValueError("num_steps must be positive")
    if not 0 <= start_step < end_step <= num_steps:
        raise ValueError("require 0 <= start_step < end_step <= the scheduler's step count")
    if skip_interval is not None:
        if not isinstance(skip_interval, (list, tuple)) or len(skip_interval) != 2 or not all(map(_is_int, skip_interval)):
            raise ValueError("skip_interval must be a pair of integer step indices")
        if not 0 <= skip_interval[0] < skip_interval[1] <= num_steps:
            raise ValueError("require 0 <= skip_interval start < end <= the scheduler's step count")
        skip_interval = (int(skip_interval[0]), int(skip_interval[1]))
    if not isinstance(stg_scale, Real) or isinstance(stg_scale, bool) or not math.isfinite(stg_scale) or stg_scale < 0:
        raise ValueError("stg_scale must be finite and nonnegative")
    if (not isinstance(warmup_scale, Real) or isinstance(warmup_scale, bool) or not math.isfinite(warmup_scale)
            or warmup_scale < 1):
        raise ValueError("warmup_scale must be finite and at least 1")
    return GuidancePlan(int(num_steps), int(start_step), int(end_step), float(stg_scale), skip_interval,
                        float(warmup_scale))


def apply_guidance(negative: torch.Tensor, positive: torch.Tensor, guidance_scale: float, *, step_index: int,
                   plan: GuidancePlan, weak_predict_fn: Optional[Callable[[], torch.Tensor]] = None) -> torch.Tensor:
    if negative.shape != positive.shape or negative.dtype != positive.dtype:
        raise ValueError("CFG predictions must have matching shape and dtype")
    if negative.device != positive.device or not positive.is_floating_point():
        raise ValueError("CFG predictions must be floating tensors on the same device")
    if (not isinstance(guidance_scale, Real) or isinstance(guidance_scale, bool) or not math.isfinite(guidance_scale)
            or guidance_scale <= 1):
        raise ValueError("this guidance path requires a finite guidance_scale > 1")
    if not plan.active(step_index):
        return positive
    guided = negative + plan.scale_at(step_index, guidance_scale) * (positive - negative)
    if plan.stg_scale:
        if weak_predict_fn is None:
            raise ValueError("STG requires a weak positive prediction")
        weak = weak_predict_fn()
        if weak.shape != positive.shape or weak.dtype != positive.dtype or weak.device != positive.device:
            raise ValueError("STG prediction must match the positive shape, dtype and device")
        guided = (guided.float() + plan.stg_scale * (positive.float() - weak.float())).to(guided.dtype)
    return guided
