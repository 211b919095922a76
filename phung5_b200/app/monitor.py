"""Engine health monitoring and the warm-up watcher.

Reference: `OrchestratorChecker` (pipeline_service/modules/monitoring/orchestrator.py:19-53), `_watch_models`
(:67-129) and the per-engine prober (modules/monitoring/module.py:13-72): each local engine is probed for
health and for serving the expected model; the watcher moves the service to READY once every engine runs
and the coder probe / warm-up finished, and handles an engine going down.

Here a prober polls `GET /health` and `GET /v1/models` of every enabled client concurrently (bounded by a
request timeout), mapping the result to STARTING (not answering yet, within the start grace), RUNNING,
or DOWN (failed after grace, or answering with the wrong model). The watcher drives `MinerState`:
WARMING_UP -> READY when all RUNNING and `on_ready` (probe, warm-up) completed, or -> REPLACE when `on_ready`
reports an unhealthy coder (probe below its min_tps floor) and replacements remain; a DOWN engine during
READY/COMPLETE -> REPLACE when replacements remain, else the service keeps serving what it can.
"""
from __future__ import annotations

import asyncio
import logging
import time
from typing import Awaitable, Callable, Dict, Optional

import httpx

from .state import MinerState, MinerStatus, ServiceState

log = logging.getLogger("phung5_b200.app")


class EngineProber:
    def __init__(self, name: str, base_url: str, model: str = "", timeout: float = 5.0, grace_s: float = 1800.0,
                 client: Optional[httpx.AsyncClient] = None):
        self.name = name
        self.url = base_url.rstrip("/").removesuffix("/v1")
        self.model = model
        self.timeout = timeout
        self.grace_s = grace_s
        self.t0 = time.monotonic()
        self.http = client or httpx.AsyncClient(timeout=timeout)
        self.state = ServiceState.STARTING
        self.last_error = ""
        self.ever_up = False

    async def probe(self) -> ServiceState:
        try:
            r = await self.http.get(self.url + "/health", timeout=self.timeout)
            if r.status_code != 200:
                raise RuntimeError(f"/health {r.status_code}")
            if self.model:
                m = await self.http.get(self.url + "/v1/models", timeout=self.timeout)
                ids = [d.get("id") for d in (m.json().get("data") or [])]
                if self.model not in ids:
                    self.last_error = f"serving {ids}, expected {self.model}"
                    self.state = ServiceState.DOWN
                    return self.state
            self.state = ServiceState.RUNNING
            self.ever_up = True
            self.last_error = ""
        except (httpx.HTTPError, RuntimeError, ValueError) as e:
            self.last_error = f"{type(e).__name__}: {str(e)[:120]}"
            within_grace = time.monotonic() - self.t0 < self.grace_s and not self.ever_up
            self.state = ServiceState.STARTING if within_grace else ServiceState.DOWN
        return self.state


class HealthWatcher:
    def __init__(self, state: MinerState, probers: Dict[str, EngineProber], interval_s: float = 5.0,
                 on_ready: Optional[Callable[[], Awaitable[None]]] = None):
        self.state, self.probers, self.interval = state, probers, interval_s
        self.on_ready = on_ready
        self.ready_done = False
        self._task: Optional[asyncio.Task] = None

    async def tick(self) -> None:
        results = await asyncio.gather(*(p.probe() for p in self.probers.values()))
        for name, st in zip(self.probers, results):
            self.state.set_llm_status(name, st)
        s = self.state
        if s.status == MinerStatus.WARMING_UP and s.models_ready():
            healthy = True
            if not self.ready_done and self.on_ready is not None:
                try:
                    healthy = await self.on_ready() is not False
                except Exception:  # noqa: BLE001 - a failed warm-up does not block READY
                    log.exception("warm-up failed")
            self.ready_done = True
            if not healthy and s.replacements_remaining > 0:
                log.warning("coder probe below its floor; requesting replacement")
                s.status = MinerStatus.REPLACE
            else:
                if not healthy:
                    log.warning("coder probe below its floor but no replacement left; serving anyway")
                s.status = MinerStatus.READY
        elif s.any_down() and s.status in (MinerStatus.READY, MinerStatus.COMPLETE) and s.replacements_remaining > 0:
            log.warning("engine down (%s); requesting replacement",
                        {n: p.last_error for n, p in self.probers.items() if p.state == ServiceState.DOWN})
            s.status = MinerStatus.REPLACE

    async def run(self) -> None:
        while True:
            try:
                await self.tick()
            except Exception:  # noqa: BLE001
                log.exception("health tick failed")
            await asyncio.sleep(self.interval)

    def start(self) -> None:
        self._task = asyncio.create_task(self.run())

    def stop(self) -> None:
        if self._task is not None:
            self._task.cancel()
