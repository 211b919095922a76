"""Burst controller: in the judge-only tail of a batch, lend the coder GPUs to extra judge replicas.

Reference: `BurstController` (pipeline_service/llm/burst.py:43-225, setup :227-258) with the proxy's
`to_judge` / `to_coder` swaps (docker/opt/sgl/lb_proxy.py:171-240). A per-batch ledger records which prompts
have started coding and which coder calls are open; once every prompt has been seen and no call is open,
coding is over for the batch while judging continues. After a quiet period with no batch event, the coder
engines behind the proxy are parked (drained, weights released with /sleep) and sleeping judge
replicas on the same GPUs are woken and added to the judge's `LoadBalancedClient`. Any coder call
(a retry, a refinement, the next batch) first swaps back: judge replicas leave the client, drain and sleep,
the coder engines are unparked.

Swaps are serialised by a lock and undone on partial failure (a judge replica that failed to wake is
put back to sleep and the coders are unparked). State is "coder", "judge" or "broken" (an undo failed:
no further swaps; coder calls proceed against whatever answers).
"""
from __future__ import annotations

import asyncio
import logging
import time
from typing import Dict, FrozenSet, Iterable, List, Optional, Set

import httpx

log = logging.getLogger("phung5_b200.app")


class _Ledger:
    """Coding progress of the running batch: which prompts have started coding (or finished), and which coder
    calls are open. Coding is over once every prompt of the batch has been seen and no call is open."""

    def __init__(self, size: int, stems: Optional[Iterable[str]]):
        self.size = size
        self.stems: Optional[FrozenSet[str]] = frozenset(stems) if stems is not None else None
        self.seen: Set[str] = set()
        self.open_calls: Dict[int, str] = {}

    def see(self, stem: str) -> None:
        if self.stems is None or stem in self.stems:
            self.seen.add(stem)

    def coding_over(self) -> bool:
        return not self.open_calls and len(self.seen) >= self.size


class BurstController:
    def __init__(self, judge_lb, judge_idxs: List[int], proxy_url: str, coder_upstreams: List[str],
                 http: Optional[httpx.AsyncClient] = None, delay_s: float = 2.0, drain_s: float = 60.0):
        self.lb = judge_lb
        self.idxs = list(judge_idxs)
        self.proxy = proxy_url.rstrip("/")
        self.coders = list(coder_upstreams)
        self.http = http or httpx.AsyncClient(timeout=httpx.Timeout(600.0, connect=10.0))
        self.delay_s, self.drain_s = delay_s, drain_s
        self.state = "coder"
        self.parked: List[str] = []             # the coder upstreams the last swap parked
        self.lock = asyncio.Lock()
        self.ledger: Optional[_Ledger] = None
        self.events: List[dict] = []
        self._activity = 0                      # bumped by every batch event; the quiet-period watcher reads it
        self._next_call = 0
        self._watcher: Optional[asyncio.Task] = None
        self._background: Set[asyncio.Task] = set()
        self.t0 = time.time()

    def _ev(self, what: str, **kw):
        self.events.append({"t": round(time.time() - self.t0, 2), "what": what, **kw})
        log.info("[burst] %s %s", what, kw or "")

    def _run_later(self, coro) -> asyncio.Task:
        task = asyncio.get_running_loop().create_task(coro)
        self._background.add(task)                  # keep a reference until it finishes
        task.add_done_callback(self._background.discard)
        return task

    # ---------------------------------------------------------------------------------------- batch events
    # The pipeline reports batch and coder-call events; when coding is over the controller waits for a quiet
    # period of delay_s with no new event and only then lends the coder GPUs to the judge.

    def batch_start(self, n: int, stems=None) -> None:
        self.ledger = _Ledger(n, stems)
        self.t0 = time.time()
        self._ev("batch_start", n=n)
        self._activity_changed()

    def batch_end(self) -> None:
        self.ledger = None
        self._ev("batch_end", state=self.state)
        self._activity_changed()
        if self.state == "judge":
            self._run_later(self.ensure_coder("batch end"))

    def coder_begin(self, stem: str) -> int:
        """Register one coder call; returns its id for coder_end."""
        self._next_call += 1
        if self.ledger is not None:
            self.ledger.open_calls[self._next_call] = stem
            self.ledger.see(stem)
        self._activity_changed()
        return self._next_call

    def coder_end(self, call_id: int) -> None:
        # calls opened before the current batch started are not in its ledger and change nothing
        if self.ledger is not None and self.ledger.open_calls.pop(call_id, None) is not None:
            self._activity_changed()

    def task_done(self, stem: str) -> None:
        if self.ledger is not None:
            self.ledger.see(stem)
            self._activity_changed()

    def _judge_tail(self) -> bool:
        return self.state == "coder" and self.ledger is not None and self.ledger.coding_over()

    def _activity_changed(self) -> None:
        self._activity += 1
        if self._judge_tail() and (self._watcher is None or self._watcher.done()):
            self._watcher = self._run_later(self._swap_after_quiet_period())
            self._ev("armed", delay=self.delay_s)

    async def _swap_after_quiet_period(self) -> None:
        while True:
            before = self._activity
            await asyncio.sleep(self.delay_s)
            if not self._judge_tail():
                return
            if self._activity == before:
                break
        await self.to_judge()

    # ------------------------------------------------------------------------------------------------ swaps

    async def _post(self, url: str, body: Optional[dict] = None):
        r = await self.http.post(url, json=body or {})
        if r.status_code >= 400:
            raise RuntimeError(f"{url} -> {r.status_code} {r.text[:120]}")
        return r

    async def _coder_upstreams(self) -> List[str]:
        """The configured coder upstreams, else every upstream the proxy has active now."""
        if self.coders:
            return self.coders
        r = await self.http.get(self.proxy + "/park_state")
        if r.status_code >= 400:
            raise RuntimeError(f"{self.proxy}/park_state -> {r.status_code}")
        return list(r.json().get("active", []))

    async def to_judge(self) -> bool:
        async with self.lock:
            if self.state != "coder":
                return False
            woken: List[int] = []
            try:
                self.parked = await self._coder_upstreams()
                await self._post(self.proxy + "/park", {"upstreams": self.parked})
                for i in self.idxs:
                    await self._post(self.lb.urls[i] + "/wake_up")
                    woken.append(i)
                self.lb.set_active(self.idxs, True)
                self.state = "judge"
                self._ev("to_judge", replicas=len(self.idxs))
                return True
            except Exception as e:  # noqa: BLE001 - undo what was done
                self._ev("to_judge_failed", error=str(e)[:160])
                try:
                    for i in woken:
                        await self._post(self.lb.urls[i] + "/sleep")
                    await self._post(self.proxy + "/unpark", {"upstreams": self.parked})
                except Exception as e2:  # noqa: BLE001
                    self.state = "broken"
                    self._ev("broken", error=str(e2)[:160])
                return False

    async def _drain_judges(self):
        t0 = time.monotonic()
        while any(self.lb.inflight[i] for i in self.idxs):
            if time.monotonic() - t0 > self.drain_s:
                raise TimeoutError("judge replicas did not drain")
            await asyncio.sleep(0.05)

    async def ensure_coder(self, why: str = "") -> bool:
        """Call before any coder request; returns once the coder engines take requests again."""
        if self.state != "judge":
            return self.state == "coder"
        async with self.lock:
            if self.state != "judge":
                return self.state == "coder"
            try:
                self.lb.set_active(self.idxs, False)
                await self._drain_judges()
                for i in self.idxs:
                    await self._post(self.lb.urls[i] + "/sleep")
                await self._post(self.proxy + "/unpark", {"upstreams": self.parked})
                self.state = "coder"
                self._ev("to_coder", why=why)
                return True
            except Exception as e:  # noqa: BLE001
                self.state = "broken"
                self._ev("broken", error=str(e)[:160])
                return False


class BurstCoderBackend:
    """Coder backend wrapper: swaps back to coder mode before each call and reports begin/end."""

    def __init__(self, inner, ctrl: BurstController):
        self.inner, self.ctrl = inner, ctrl

    async def chat(self, body: dict) -> dict:
        from ..serve.router import affinity_key
        await self.ctrl.ensure_coder("coder call")
        call = self.ctrl.coder_begin(str(affinity_key.get() or body.get("metadata", {}).get("stem", "?")))
        try:
            return await self.inner.chat(body)
        finally:
            self.ctrl.coder_end(call)
