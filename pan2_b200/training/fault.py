"""Failure detection and handling on the host: heartbeat watchdog, anomaly detector, fault injection.

* :class:`Heartbeat` -- a daemon thread that, when the training loop has not reported progress for
  ``threshold_s``, prints the rank, the last stage and step, dumps every thread's traceback and ends the
  process (reference: train.py:1431-1459).  ``on_stuck`` is replaceable so tests observe it without
  exiting.
* :class:`AnomalyDetector` -- EMA (decay 0.99) of finite losses and gradient norms; a step is anomalous
  on a non-finite loss or norm, a norm above 1e6, or (after ``warmup_steps``) a loss above 20x its EMA
  or a norm above 6x its EMA (when above 1e-3).  Every rank's verdict is combined with a MAX all-reduce
  on the CPU group so all ranks recover together (train.py:1650-1729).
* :class:`FaultInjector` -- host-side faults for tests and drills, parsed from a spec such as
  ``"nan_loss@5,stall@7:2.5,raise@9,exit@11/1"``: a NaN loss reported at step 5 (the update is voted
  non-finite and skipped), a 2.5 s stall at step 7, an exception at step 9, ``os._exit`` of rank 1 at
  step 11 (between steps, nothing in flight).  Each event fires once.  Nothing is injected on the GPU.
"""
from __future__ import annotations

import faulthandler
import math
import os
import sys
import threading
import time
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Tuple

import torch
import torch.distributed as dist


class Heartbeat:
    def __init__(self, rank: int, threshold_s: float = 50000.0, poll_s: float = 5.0,
                 on_stuck: Optional[Callable[[str], None]] = None):
        self.rank = rank
        self.threshold_s = threshold_s
        self.poll_s = poll_s
        self.stage = "init"
        self.step = 0
        self.last = time.monotonic()
        self._stop = threading.Event()
        self.on_stuck = on_stuck or self._exit
        self.fired = False
        self._thread: Optional[threading.Thread] = None

    def beat(self, stage: Optional[str] = None, step: Optional[int] = None) -> None:
        if stage is not None:
            self.stage = stage
        if step is not None:
            self.step = step
        self.last = time.monotonic()

    def start(self) -> "Heartbeat":
        self._thread = threading.Thread(target=self._loop, name="heartbeat", daemon=True)
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2 * self.poll_s)

    def _loop(self):
        while not self._stop.wait(self.poll_s):
            stuck = time.monotonic() - self.last
            if stuck > self.threshold_s and not self.fired:
                self.fired = True
                self.on_stuck(f"[heartbeat] rank={self.rank} stuck for {stuck:.1f}s at stage='{self.stage}' "
                              f"step={self.step}")

    @staticmethod
    def _exit(msg: str) -> None:
        print(msg + "; dumping all-thread tracebacks then exiting", file=sys.stderr, flush=True)
        try:
            faulthandler.dump_traceback(file=sys.stderr, all_threads=True)
        except Exception:
            pass
        sys.stderr.flush()
        os._exit(1)


@dataclass
class AnomalyDetector:
    warmup_steps: int = 100
    decay: float = 0.99
    loss_spike: float = 20.0
    grad_spike: float = 6.0
    grad_spike_min: float = 1e-3
    grad_hard_limit: float = 1e6
    group: Optional[object] = None
    ema_loss: Optional[float] = None
    ema_grad: Optional[float] = None
    last_reasons: List[str] = field(default_factory=list)

    def reset(self) -> None:
        self.ema_loss = None
        self.ema_grad = None

    def _ema(self, cur, v):
        return v if cur is None else self.decay * cur + (1 - self.decay) * v

    def local_verdict(self, step: int, loss: float, grad_norm: float) -> Tuple[bool, List[str]]:
        spikes_on = step >= max(0, int(self.warmup_steps))
        if math.isfinite(loss):
            self.ema_loss = self._ema(self.ema_loss, loss)
        if math.isfinite(grad_norm):
            self.ema_grad = self._ema(self.ema_grad, grad_norm)
        reasons = []
        if not math.isfinite(loss):
            reasons.append(f"non-finite loss={loss}")
        elif spikes_on and self.ema_loss and self.ema_loss > 0 and loss > self.loss_spike * self.ema_loss:
            reasons.append(f"loss spike: {loss:.6f} > {self.loss_spike:.1f} * ema_loss({self.ema_loss:.6f})")
        if not math.isfinite(grad_norm):
            reasons.append(f"non-finite grad_norm={grad_norm}")
        elif grad_norm > self.grad_hard_limit:
            reasons.append(f"grad norm overflow: {grad_norm:.6f} > {self.grad_hard_limit:.1f}")
        elif (spikes_on and grad_norm > self.grad_spike_min and self.ema_grad and self.ema_grad > 0
              and grad_norm > self.grad_spike * self.ema_grad):
            reasons.append(f"grad norm spike: {grad_norm:.6f} > {self.grad_spike:.1f} * ema_grad({self.ema_grad:.6f})")
        return bool(reasons), reasons

    def __call__(self, step: int, loss: float, grad_norm: float) -> bool:
        bad, self.last_reasons = self.local_verdict(step, loss, grad_norm)
        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            t = torch.tensor([int(bad)], dtype=torch.int32)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
            return bool(t.item())
        return bad


class InjectedFault(RuntimeError):
    pass


class FaultInjector:
    KINDS = ("nan_loss", "inf_grad", "stall", "raise", "exit")

    def __init__(self, spec: Optional[str] = None, rank: Optional[int] = None):
        self.events: Dict[int, List[Tuple[str, float, Optional[int]]]] = {}
        for part in (spec or "").split(","):
            part = part.strip()
            if not part:
                continue
            kind, _, rest = part.partition("@")
            if kind not in self.KINDS or not rest:
                raise ValueError(f"bad fault spec {part!r}; expected kind@step[:arg][/rank] with kind in {self.KINDS}")
            only_rank = None
            if "/" in rest:
                rest, r = rest.split("/", 1)
                only_rank = int(r)
            step_s, _, arg = rest.partition(":")
            self.events.setdefault(int(step_s), []).append((kind, float(arg) if arg else 0.0, only_rank))
        self.rank = rank
        self.fired = set()

    def _active(self, step: int, consume: bool = False):
        """Events due at ``step`` on this rank.  Each event fires once: a rolled-back run that
        reaches the step again does not meet the same fault (a transient fault, as in production)."""
        for i, (kind, arg, r) in enumerate(self.events.get(step, [])):
            if (step, i) in self.fired or not (r is None or r == self.rank):
                continue
            if consume:
                self.fired.add((step, i))
            yield kind, arg

    def before_step(self, step: int) -> None:
        for kind, arg in list(self._active(step)):
            if kind in ("stall", "raise", "exit"):
                self.fired.update((step, i) for i, e in enumerate(self.events.get(step, [])) if e[0] == kind)
            if kind == "stall":
                time.sleep(arg)
            elif kind == "raise":
                raise InjectedFault(f"injected exception at step {step}")
            elif kind == "exit":
                sys.stderr.flush()
                os._exit(int(arg) if arg else 17)

    def after_step(self, step: int, metrics: Dict) -> Dict:
        for kind, _ in list(self._active(step, consume=True)):
            if kind == "nan_loss":
                metrics = dict(metrics, loss=float("nan"))
            elif kind == "inf_grad":
                metrics = dict(metrics, grad_norm=float("inf"))
        return metrics

    def poisons_update(self, step: int) -> bool:
        """True when this step's update must be treated as non-finite (before the optimizer runs)."""
        return any(k in ("nan_loss", "inf_grad") for k, _ in self._active(step))
