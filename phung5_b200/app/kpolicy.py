"""Policies for K, the number of coder candidates per prompt, and the batch-boundary guards.

Reference: adaptive K from the CPU quota (pipeline_service/modules/metrics/adaptive_k.py:87-365), per-photo
token budget K (modules/metrics/budget_k.py:33-177), the round-budget time guard (pgh_timeguard.py), the CPU
render-backlog brake (pgh_kcpu.py) and deadline salvage (pgh_salvage.py). The formulas below are this
framework's own:

- `start_k` (once, at start-up): "fixed" keeps the configured K; "cpu" caps it at the host's share of
  candidate checking, cores / cpu_per_candidate (cores = min(cgroup quota, allowed CPUs, CPU count), read
  once by `detect_cores`); "off" = configured K, no detection.
- `RoundGuard` (batch boundaries): batches are grouped into rounds of `round_batches` with a wall budget of
  `round_s`. Before batch b > 0 of a round the guard fits wall = overhead + unit * K to the round's finished
  batches (unit = mean of (wall - overhead) / K), gives each remaining batch an equal share of what is left of
  the budget minus `margin_s`, and if the current K's predicted wall exceeds that share, cuts K to the largest
  step (a fraction of the round's start K) whose prediction fits (else `k_floor`). It never raises K within a
  round; a round ends after `round_batches` batches or an idle gap longer than `idle_reset_s`. A cut keeps
  positions 0..K'-1 of every bracket (seeds task.seed + k), so a cut batch's pool is a prefix of the uncut one.
  "shadow" computes and logs the cut without applying it; `replay` reruns the decisions from recorded walls.
- `BudgetK` (per prompt): give every prompt about the same coder tokens instead of the same number of drafts.
  Candidate cost c (bytes of code) is only known after drafts come back, so a prompt first launches K_lo
  drafts, estimates c from them (shrunk toward the reference mean of earlier prompts) and tops up to
  K_i = clamp(lam * c^-p, K_lo, K_hi), with lam solved by bisection so that the reference prompts'
  mean K_i * c_i equals K * mean c_i.
- `RenderBrake`: holds new coder launches while the render backlog exceeds `max_backlog` per render slot.
"""
from __future__ import annotations

import asyncio
import logging
import math
import os
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence, Tuple

log = logging.getLogger("phx.kpolicy")


def cpu_k(base_k: int, quota: Optional[float], cpu_per_candidate: float = 0.25, k_min: int = 2) -> int:
    if quota is None or quota <= 0 or math.isinf(quota):
        return base_k
    return max(k_min, min(base_k, int(quota / cpu_per_candidate)))


def detect_cores(cgroup_root: str = "/sys/fs/cgroup", affinity: Optional[Callable[[], int]] = None,
                 cpu_count: Optional[Callable[[], Optional[int]]] = None) -> Tuple[Optional[float], str]:
    """(cores, source): the smallest of the cgroup CPU quota, the CPUs this process may run on and the CPU
    count; (None, "unknown") when none of them can be read."""
    from ..utils.affinity import read_quota

    def _aff():
        return len(os.sched_getaffinity(0))
    vals = []
    q = read_quota(cgroup_root)
    if q is not None and not math.isinf(q) and q > 0:
        vals.append((q, "quota"))
    for fn, name in ((affinity or _aff, "affinity"), (cpu_count or os.cpu_count, "cpu_count")):
        try:
            v = fn()
        except (AttributeError, OSError):
            v = None
        if v:
            vals.append((float(v), name))
    if not vals:
        return None, "unknown"
    return min(vals)


def start_k(mode: str, k_cfg: int, cores: Optional[float], cpu_per_candidate: float = 0.25, k_min: int = 2
            ) -> Tuple[int, str]:
    """K for the run and where it came from."""
    if mode == "cpu":
        if cores is None:
            return k_cfg, "cpu:unknown-cores"
        return cpu_k(k_cfg, cores, cpu_per_candidate, k_min), f"cpu:{cores:g}"
    return k_cfg, mode


def guard_cut(k: int, k_start: int, walls: Sequence[Tuple[int, float]], batch_index: int, round_batches: int,
              round_s: float, margin_s: float, overhead_s: float, steps: Sequence[float], k_floor: int
              ) -> Tuple[int, dict]:
    """The round guard's decision before batch `batch_index` (> 0) of a round, from the round's finished
    batches `walls` [(K, wall seconds)]. Pure: (K for the batch, record of the inputs)."""
    spent = sum(w for _, w in walls)
    left = max(1, round_batches - batch_index)
    allowed = (round_s - margin_s - spent) / left
    units = [max(w - overhead_s, 0.0) / max(kk, 1) for kk, w in walls]
    unit = sum(units) / len(units) if units else 0.0

    def pred(kk):
        return overhead_s + unit * kk
    rec = {"spent": round(spent, 1), "allowed": round(allowed, 1), "unit": round(unit, 3),
           "pred": round(pred(k), 1), "k": k}
    if not walls or pred(k) <= allowed:
        return k, rec
    new = k_floor
    for f in sorted(steps, reverse=True):
        kk = max(k_floor, int(math.floor(f * k_start)))
        if kk < k and pred(kk) <= allowed:
            new = kk
            break
    rec["cut_to"] = new
    return min(k, new), rec


@dataclass
class RoundGuard:
    mode: str = "off"                    # live | shadow | off
    round_batches: int = 4
    round_s: float = 7200.0
    margin_s: float = 250.0
    overhead_s: float = 90.0
    steps: Sequence[float] = (0.85, 0.7, 0.55, 0.4, 0.25)
    k_floor: int = 2
    idle_reset_s: float = 900.0
    clock: Callable[[], float] = field(default=None, repr=False)
    walls: List[Tuple[int, float]] = field(default_factory=list)     # this round's finished batches
    k: Optional[int] = None              # the K the guard currently allows (None before the first batch)
    k_start: Optional[int] = None
    last_end: Optional[float] = None
    log: List[dict] = field(default_factory=list)

    def _now(self) -> float:
        import time
        return (self.clock or time.monotonic)()

    def before_batch(self, k_start: int) -> int:
        """K for the next batch (k_start when off, in shadow mode, or at the start of a round)."""
        if self.mode == "off":
            return k_start
        now = self._now()
        if (self.k_start != k_start or len(self.walls) >= self.round_batches or
                (self.last_end is not None and now - self.last_end > self.idle_reset_s)):
            self.walls, self.k, self.k_start = [], k_start, k_start
        if not self.walls:
            self.log.append({"batch": 0, "k": k_start})
            return k_start
        k, rec = guard_cut(self.k, self.k_start, self.walls, len(self.walls), self.round_batches, self.round_s,
                           self.margin_s, self.overhead_s, self.steps, self.k_floor)
        rec["batch"] = len(self.walls)
        rec["mode"] = self.mode
        self.log.append(rec)
        if "cut_to" in rec:
            log.info("[round guard] %s batch %d: predicted %.0f s > allowed %.0f s -> K %d -> %d", self.mode,
                     rec["batch"], rec["pred"], rec["allowed"], self.k, k)
        if self.mode == "live":
            self.k = k
            return k
        return self.k

    def after_batch(self, k: int, wall_s: float) -> None:
        if self.mode == "off":
            return
        self.walls.append((k, wall_s))
        self.last_end = self._now()


def replay(walls: Sequence[float], k_start: int, **params) -> List[int]:
    """K of every batch of a recorded run (walls in order, assumed back to back) under a live guard whose
    batches took those walls scaled to the K the guard chose (wall proportional to K past the overhead)."""
    g = RoundGuard(mode="live", **params)
    t = [0.0]
    g.clock = lambda: t[0]
    out = []
    for w in walls:
        k = g.before_batch(k_start)
        w_k = g.overhead_s + max(w - g.overhead_s, 0.0) * k / k_start
        out.append(k)
        t[0] += w_k
        g.after_batch(k, w_k)
    return out


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
