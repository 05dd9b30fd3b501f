"""Deterministic Euler sampler for velocity prediction, and the ``early_refine_2x`` schedule.

Semantics of the reference's FlowEulerScheduler (pan/schedulers/scheduling_flow_match_discrete.py:27-83):
noise levels run from 1 to 0 on ``steps + 1`` evenly spaced points warped by the static shift
``s*sigma / (1 + (s-1)*sigma)``; the model is queried at the first ``steps`` levels scaled to
``num_train_timesteps``; one step adds ``velocity * (sigma_next - sigma)`` in fp32.  The sigma grid
stays on the host, so the step coefficient is a Python float and no device value is read back.  A
timestep listed twice resolves to its later position.

``early_refine_2x`` (pan/schedulers/timestep_schedule.py:5-28) drops grid indices 15 and 25 of a
50-step shifted grid and inserts the midpoints of its first two intervals: still 50 evaluations,
finer steps at high noise.
"""
from __future__ import annotations

from typing import Optional

import torch


def shifted_sigmas(steps: int, shift: float) -> torch.Tensor:
    g = torch.linspace(1, 0, steps + 1)
    if shift == 1.0:
        return g
    return shift * g / (1 + (shift - 1) * g)


class FlowEulerScheduler:
    def __init__(self, num_train_timesteps: int = 1000, shift: float = 1.0):
        self.num_train_timesteps = int(num_train_timesteps)
        self.shift = float(shift)
        self.num_inference_steps: Optional[int] = None
        self._index: Optional[int] = None
        self._set(torch.linspace(1, 0, self.num_train_timesteps + 1), None)

    def _set(self, sigmas: torch.Tensor, device) -> None:
        self.sigmas = sigmas.float()
        self.timesteps = (self.sigmas[:-1] * self.num_train_timesteps).to(device=device, dtype=torch.float32)
        self._host_t = self.timesteps.cpu()

    @property
    def step_index(self) -> Optional[int]:
        return self._index

    def set_timesteps(self, steps: int, device=None) -> None:
        self.num_inference_steps = int(steps)
        self._index = None
        self._set(shifted_sigmas(self.num_inference_steps, self.shift), device)

    def index_of(self, timestep) -> int:
        v = float(timestep) if not torch.is_tensor(timestep) else float(timestep.detach().cpu())
        hits = (self._host_t == v).nonzero().view(-1).tolist()
        if not hits:
            raise ValueError(f"no step of the current schedule has timestep {timestep} (was set_timesteps() called?)")
        return hits[1] if len(hits) > 1 else hits[0]

    def coefficient(self, timestep) -> float:
        """``sigma_next - sigma`` of the interval that starts at ``timestep`` (advances the index)."""
        if isinstance(timestep, int) or (torch.is_tensor(timestep) and not timestep.is_floating_point()):
            raise ValueError("step() expects a value taken from scheduler.timesteps, not a loop index")
        if self._index is None:
            self._index = self.index_of(timestep)
        a, b = float(self.sigmas[self._index]), float(self.sigmas[self._index + 1])
        self._index += 1
        return b - a

    def step(self, velocity: torch.Tensor, timestep, sample: torch.Tensor) -> torch.Tensor:
        """Euler step to the next level; the result is fp32."""
        return sample.float() + velocity.float() * self.coefficient(timestep)


def apply_timestep_schedule(sched: FlowEulerScheduler, name: str) -> torch.Tensor:
    if name == "standard":
        return sched.timesteps
    if name != "early_refine_2x":
        raise ValueError(f"unknown timestep schedule {name!r}")
    s = sched.sigmas
    ok = (s.ndim == 1 and s.numel() == 51 and sched.timesteps.numel() == 50 and bool(torch.isfinite(s).all())
          and bool((s[:-1] > s[1:]).all()) and abs(float(s[0]) - 1.0) < 1e-6 and abs(float(s[-1])) < 1e-6)
    if not ok:
        raise ValueError("the early_refine_2x grid is defined only for 50 sigmas falling from 1 to 0")
    keep = torch.ones(51, dtype=torch.bool)
    keep[15] = False
    keep[25] = False
    mids = (s[:2] + s[1:3]) / 2
    refined = torch.cat([s[keep], mids]).sort(descending=True).values
    if not bool((refined[:-1] > refined[1:]).all()):
        raise ValueError("refined sigma grid must be strictly decreasing")
    sched._set(refined, sched.timesteps.device)
    sched._index = None
    return sched.timesteps
