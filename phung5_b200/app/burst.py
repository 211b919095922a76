"""Burst controller: in the judge-only tail of a batch, lend the coder GPUs to extra judge replicas.

Reference: `BurstController` (pipeline_service/llm/burst.py:43-225, setup :227-258) with the proxy's
`to_judge` / `to_coder` swaps (docker/opt/sgl/lb_proxy.py:171-240). Once every prompt of the batch has
launched its coders and no coder call is in flight, coding is over for the batch while judging continues;
the coder engines behind the proxy are parked (drained, weights released with /sleep) and sleeping judge
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
from typing import List, Optional, Set

import httpx

log = logging.getLogger("phung5_b200.app")


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
        self.lock = asyncio.Lock()
        self.gen = 0
        self.n: Optional[int] = None
        self.stems: Optional[Set[str]] = None
        self.pending = 0
        self.launched: Set[str] = set()
        self.done: Set[str] = set()
        self.events: List[dict] = []
        self._timer: Optional[asyncio.TimerHandle] = None
        self._tasks: Set[asyncio.Task] = set()
        self.t0 = time.time()

    def _ev(self, what: str, **kw):
        self.events.append({"t": round(time.time() - self.t0, 2), "gen": self.gen, "what": what, **kw})
        log.info("[burst] %s %s", what, kw or "")

    def _spawn(self, coro):
        t = asyncio.get_running_loop().create_task(coro)
        self._tasks.add(t)
        t.add_done_callback(self._tasks.discard)
        return t

    # ---------------------------------------------------------------------------------------- batch events

    def batch_start(self, n: int, stems=None) -> None:
        self.gen += 1
        self.n, self.stems = n, (set(stems) if stems is not None else None)
        self.pending, self.launched, self.done = 0, set(), set()
        self.t0 = time.time()
        self._cancel()
        self._ev("batch_start", n=n)

    def batch_end(self) -> None:
        self.n = None
        self._cancel()
        self._ev("batch_end", state=self.state)
        if self.state == "judge":
            self._spawn(self.ensure_coder("batch end"))

    def coder_begin(self, stem: str, k: int = 1) -> int:
        self.pending += k
        self.launched.add(stem)
        self._cancel()
        return self.gen

    def coder_end(self, gen: int) -> None:
        if gen != self.gen:
            return
        self.pending -= 1
        self._maybe_arm()

    def task_done(self, stem: str) -> None:
        self.done.add(stem)
        self._maybe_arm()

    def _maybe_arm(self) -> None:
        seen = self.launched | self.done
        if self.stems is not None:
            seen &= self.stems
        if self.n is not None and self.pending <= 0 and len(seen) >= self.n and self.state == "coder" \
                and self._timer is None:
            loop = asyncio.get_running_loop()
            gen = self.gen
            self._timer = loop.call_later(self.delay_s, lambda: self._spawn(self._fire(gen)))
            self._ev("armed", delay=self.delay_s)

    def _cancel(self):
        if self._timer is not None:
            self._timer.cancel()
            self._timer = None

    async def _fire(self, gen: int):
        self._timer = None
        if gen != self.gen or self.n is None or self.pending > 0:
            return
        await self.to_judge()

    # ------------------------------------------------------------------------------------------------ swaps

    async def _post(self, url: str, body: Optional[dict] = None):
        r = await self.http.post(url, json=body or {})
        if r.status_code >= 400:
            raise RuntimeError(f"{url} -> {r.status_code} {r.text[:120]}")
        return r

    async def to_judge(self) -> bool:
        async with self.lock:
            if self.state != "coder":
                return False
            woken: List[int] = []
            try:
                await self._post(self.proxy + "/park", {"upstreams": self.coders})
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
                    await self._post(self.proxy + "/unpark", {"upstreams": self.coders})
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
                await self._post(self.proxy + "/unpark", {"upstreams": self.coders})
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
        await self.ctrl.ensure_coder("coder call")
        gen = self.ctrl.coder_begin(body.get("metadata", {}).get("stem", f"anon{self.ctrl.pending}"))
        try:
            return await self.inner.chat(body)
        finally:
            self.ctrl.coder_end(gen)
