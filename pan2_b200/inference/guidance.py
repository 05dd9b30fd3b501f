"""Guidance schedule for sampling: classifier-free guidance (CFG) windows and spatiotemporal skip
guidance (STG).

Behaviour matches the reference's guidance controls (pan/utils/inference_guidance.py:9-111):

* steps are zero-based and windows end-exclusive; CFG runs at step ``i`` when ``i < end_step``, and
  either ``i >= start_step`` or a warmup scale above 1 was given, and ``i`` is outside the optional
  skip interval; at every other step the positive prediction is used alone;
* steps before ``start_step`` use the warmup scale in place of the guidance scale;
* the mix is ``neg + scale * (pos - neg)`` in the prediction dtype, then STG adds
  ``stg_scale * (pos - weak)`` in fp32 and casts back (``weak`` comes from a forward that skips
  some blocks).  That order of operations is part of the bf16 result, so it is kept.

Here the plan is resolved once into a per-step table (:attr:`GuidancePlan.scales`: 0 for a
positive-only step, otherwise the scale of that step), which the sampler indexes.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from numbers import Integral, Real
from typing import Callable, Optional, Tuple

import torch

SCHEDULES = ("standard", "early_refine_2x")


def _whole(v) -> bool:
    return isinstance(v, Integral) and not isinstance(v, bool)


def _real(v) -> bool:
    return isinstance(v, Real) and not isinstance(v, bool) and math.isfinite(v)


def _check(ok: bool, message: str) -> None:
    if not ok:
        raise ValueError(message)


def validate_sampling_extensions(num_steps: int, timestep_schedule: str = "standard") -> None:
    """The timestep schedule is known and, for ``early_refine_2x``, runs its fixed 50 steps."""
    _check(timestep_schedule in SCHEDULES, f"timestep_schedule {timestep_schedule!r} is not one of {SCHEDULES}")
    _check(timestep_schedule != "early_refine_2x" or num_steps == 50,
           "the early_refine_2x schedule is defined for 50 sampling steps only")


@dataclass(frozen=True)
class GuidancePlan:
    num_steps: int
    start_step: int
    end_step: int
    stg_scale: float
    skip_interval: Optional[Tuple[int, int]] = None
    warmup_scale: float = 1.0
    # per step: None = positive only, "warmup" = warmup scale, "main" = the caller's guidance scale
    modes: Tuple[Optional[str], ...] = field(default=(), compare=False)

    def _mode(self, i: int) -> Optional[str]:
        _check(_whole(i), f"guidance step index {i!r} is not an integer")
        _check(0 <= i < self.num_steps, f"guidance step index {i} is not within the {self.num_steps} sampling steps")
        return self.modes[i]

    def active(self, i: int) -> bool:
        """Whether step ``i`` mixes the negative prediction in."""
        return self._mode(i) is not None

    def scale_at(self, i: int, guidance_scale: float) -> float:
        return self.warmup_scale if i < self.start_step else guidance_scale


def resolve_guidance_plan(num_steps: int, *, start_step: int = 0, end_step: Optional[int] = None,
                          stg_scale: float = 0.0, skip_interval=None, warmup_scale: float = 1.0) -> GuidancePlan:
    """Check the window against the sampler's step count and tabulate the mode of every step."""
    stop = num_steps if end_step is None else end_step
    for label, v in (("num_steps", num_steps), ("start_step", start_step), ("end_step", stop)):
        _check(_whole(v), f"{label} ({v!r}) is not an integer")
    _check(num_steps >= 1, "there must be at least one sampling step")
    _check(0 <= start_step < stop <= num_steps,
           f"CFG window [{start_step}, {stop}) does not fit in {num_steps} sampling steps")
    skip = None
    if skip_interval is not None:
        _check(isinstance(skip_interval, (list, tuple)) and len(skip_interval) == 2
               and all(_whole(v) for v in skip_interval), "skip_interval takes two integer step indices")
        a, b = int(skip_interval[0]), int(skip_interval[1])
        _check(0 <= a < b <= num_steps, f"skip interval [{a}, {b}) does not fit in {num_steps} sampling steps")
        skip = (a, b)
    _check(_real(stg_scale) and stg_scale >= 0, f"stg_scale ({stg_scale!r}) must be a finite number >= 0")
    _check(_real(warmup_scale) and warmup_scale >= 1, f"warmup_scale ({warmup_scale!r}) must be a finite number >= 1")
    modes = []
    for i in range(num_steps):
        if i >= stop or (skip is not None and skip[0] <= i < skip[1]):
            modes.append(None)
        elif i >= start_step:
            modes.append("main")
        else:
            modes.append("warmup" if warmup_scale > 1 else None)
    return GuidancePlan(int(num_steps), int(start_step), int(stop), float(stg_scale), skip, float(warmup_scale),
                        tuple(modes))


def apply_guidance(negative: torch.Tensor, positive: torch.Tensor, guidance_scale: float, *, step_index: int,
                   plan: GuidancePlan, weak_predict_fn: Optional[Callable[[], torch.Tensor]] = None) -> torch.Tensor:
    """The prediction used at ``step_index``; ``weak_predict_fn`` runs only when STG applies."""
    mode = plan._mode(step_index)
    _check(negative.shape == positive.shape and negative.dtype == positive.dtype,
           "negative and positive predictions differ in shape or dtype")
    _check(negative.device == positive.device and positive.is_floating_point(),
           "negative and positive predictions must be floating-point tensors on one device")
    _check(_real(guidance_scale) and guidance_scale > 1, f"guidance_scale ({guidance_scale!r}) must be finite and > 1")
    if mode is None:
        return positive
    scale = plan.warmup_scale if mode == "warmup" else guidance_scale
    out = negative + scale * (positive - negative)
    if not plan.stg_scale:
        return out
    _check(weak_predict_fn is not None, "stg_scale > 0 needs the skip-block (weak) prediction")
    weak = weak_predict_fn()
    _check(weak.shape == positive.shape and weak.dtype == positive.dtype and weak.device == positive.device,
           "the skip-block prediction differs from the positive one in shape, dtype or device")
    return (out.float() + plan.stg_scale * (positive.float() - weak.float())).to(out.dtype)
