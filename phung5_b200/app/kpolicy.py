"""Policies for K, the number of coder candidates per prompt, and the batch-boundary guards.

Reference: adaptive K from the CPU quota (pipeline_service/modules/metrics/adaptive_k.py:87-365), per-photo
token budget K (modules/metrics/budget_k.py:33-177), the batch time guard (pgh_timeguard.py), the CPU
render-backlog brake (pgh_kcpu.py) and deadline salvage (pgh_salvage.py). The formulas below are this
framework's own:

- `cpu_k`: candidates cost host CPU for checking (interpreter) and, without a GPU, rendering, so K is capped
  at quota / cpu_per_candidate (a floor of k_min; None quota = unlimited = base K).
- `TimeGuard`: after each batch, K_next = K * clamp(target_wall / observed_wall) with a dead band, bounded to
  [k_min, k_max]; the target is the batch budget minus a safety margin.
- `BudgetK`: give every prompt about the same coder tokens instead of the same number of drafts. Candidate
  cost c (bytes of code) is only known after drafts come back, so a prompt first launches K_lo drafts,
  estimates c from them (shrunk toward the reference mean of earlier prompts) and tops up to
  K_i = clamp(lam * c^-p, K_lo, K_hi), with lam solved by bisection so that the reference prompts'
  mean K_i * c_i equals K * mean c_i.
- `RenderBrake`: holds new coder launches while the render backlog exceeds `max_backlog` per render slot.
"""
from __future__ import annotations

import asyncio
import math
from dataclasses import dataclass, field
from typing import List, Optional


def cpu_k(base_k: int, quota: Optional[float], cpu_per_candidate: float = 0.25, k_min: int = 2) -> int:
    if quota is None or quota <= 0:
        return base_k
    return max(k_min, min(base_k, int(quota / cpu_per_candidate)))


@dataclass
class TimeGuard:
    budget_s: float
    margin_s: float = 120.0
    k_min: int = 2
    k_max: int = 256
    dead_band: float = 0.05
    max_step: float = 2.0
    history: List[tuple] = field(default_factory=list)

    def next_k(self, k: int, wall_s: Optional[float]) -> int:
        if wall_s is None or wall_s <= 0:
            return k
        target = max(1.0, self.budget_s - self.margin_s)
        r = target / wall_s
        self.history.append((k, wall_s, r))
        if abs(r - 1.0) <= self.dead_band:
            return k
        r = min(self.max_step, max(1.0 / self.max_step, r))
        return max(self.k_min, min(self.k_max, int(round(k * r))))


@dataclass
class BudgetK:
    p: float = 1.0
    lo: float = 0.5
    hi: float = 1.5
    n0: int = 8
    shrink: float = 4.0
    floor: int = 8
    min_ref: int = 8
    ref: List[float] = field(default_factory=list)        # mean draft bytes of earlier prompts
    pending: List[float] = field(default_factory=list)

    def active(self, k: int) -> bool:
        return len(self.ref) >= self.min_ref and k > self.floor

    def initial(self, k: int) -> int:
        """Drafts to launch before the cost estimate."""
        return max(self.floor, int(round(self.lo * k))) if self.active(k) else k

    def _lam(self, k: int) -> float:
        ref = self.ref
        mean_c = sum(ref) / len(ref)
        k_lo, k_hi = self.initial(k), max(self.initial(k), int(round(self.hi * k)))
        target = k * mean_c

        def spend(lam):
            return sum(min(k_hi, max(k_lo, lam * c ** -self.p)) * c for c in ref) / len(ref)
        a, b = 1e-9, 1e-9
        while spend(b) < target and b < 1e30:
            b *= 4
        for _ in range(80):
            m = math.sqrt(a * b)
            if spend(m) < target:
                a = m
            else:
                b = m
        return b

    def decide(self, k: int, draft_bytes: List[float]) -> int:
        """Total drafts for a prompt from its first drafts' code sizes."""
        if not self.active(k):
            return k
        mean_ref = sum(self.ref) / len(self.ref)
        c_hat = (sum(draft_bytes) + self.shrink * mean_ref) / (len(draft_bytes) + self.shrink)
        k_lo, k_hi = self.initial(k), max(self.initial(k), int(round(self.hi * k)))
        return int(min(k_hi, max(k_lo, round(self._lam(k) * c_hat ** -self.p))))

    def observe(self, mean_bytes: float) -> None:
        if mean_bytes > 0:
            self.pending.append(mean_bytes)

    def batch_end(self) -> None:
        self.ref.extend(self.pending)
        self.pending.clear()


class RenderBrake:
    def __init__(self, slots: int, max_backlog: float = 4.0):
        self.slots, self.max_backlog = max(1, slots), max_backlog
        self.backlog = 0
        self._cond = asyncio.Condition()
        self.held_s = 0.0

    async def enter_render(self):
        async with self._cond:
            self.backlog += 1

    async def leave_render(self):
        async with self._cond:
            self.backlog -= 1
            self._cond.notify_all()

    async def before_coder(self, timeout: float = 60.0):
        """Wait (bounded) while renders are backed up."""
        loop = asyncio.get_running_loop()
        t0 = loop.time()
        async with self._cond:
            try:
                await asyncio.wait_for(self._cond.wait_for(lambda: self.backlog <= self.max_backlog * self.slots), timeout)
            except asyncio.TimeoutError:
                pass
        self.held_s += loop.time() - t0
