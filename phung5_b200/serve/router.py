"""Replica routing: a least-in-flight HTTP proxy and a client-side load-balanced client.

`build_proxy(upstreams)` — one OpenAI-style endpoint in front of several engine servers (one per GPU,
the reference's measured best layout, docker/opt/sgl/lb_proxy.py:1-25): each POST goes to the active
upstream with the fewest requests in flight (ties round-robin). Upstreams can be parked (no new
requests, drain, then POST /sleep on them) and unparked (POST /wake_up, resume routing), the
reference's burst swap (lb_proxy.py /burst/to_judge, /burst/to_coder); a failed swap is undone and,
if the undo fails, the proxy reports "broken" and /health answers 503.
    GET /health, GET /lb_stats, POST /park {"upstreams": [...]}, POST /unpark {...}, GET /park_state

`LoadBalancedClient` — weighted round-robin over replicas with per-task affinity (requests of one task
stay on one replica so its prefix cache hits) and load-aware migration of a task when its replica's
in-flight count exceeds the least-loaded one by a margin (pipeline_service/llm/balancer.py:79-206).
"""
from __future__ import annotations

import asyncio
import contextvars
import itertools
import time
from typing import Callable, Dict, List, Optional

import httpx

affinity_key: contextvars.ContextVar = contextvars.ContextVar("phx_affinity_key", default=None)


class ProxyState:
    def __init__(self, upstreams: List[str]):
        self.up = [u.rstrip("/") for u in upstreams]
        self.inflight = {u: 0 for u in self.up}
        self.sent = {u: 0 for u in self.up}
        self.errors = {u: 0 for u in self.up}
        self.parked: set = set()
        self.broken = False
        self.tick = itertools.count()

    def pick(self) -> Optional[str]:
        act = [u for u in self.up if u not in self.parked]
        if not act:
            return None
        t = next(self.tick)
        best = min(self.inflight[u] for u in act)
        cands = [u for u in act if self.inflight[u] == best]
        return cands[t % len(cands)]


def build_proxy(upstreams: List[str], drain_timeout: float = 120.0, client: Optional[httpx.AsyncClient] = None):
    from starlette.applications import Starlette
    from starlette.requests import Request
    from starlette.responses import JSONResponse, Response
    from starlette.routing import Route

    st = ProxyState(upstreams)
    http = client or httpx.AsyncClient(timeout=httpx.Timeout(900.0, connect=10.0))

    async def health(req: Request):
        if st.broken:
            return JSONResponse({"status": "broken"}, status_code=503)
        ok = True
        for u in st.up:
            if u in st.parked:
                continue
            try:
                r = await http.get(u + "/health", timeout=10.0)
                ok &= r.status_code == 200
            except Exception:
                ok = False
        return JSONResponse({"status": "ok" if ok else "degraded"}, status_code=200 if ok else 503)

    async def stats(req: Request):
        return JSONResponse({"inflight": st.inflight, "sent": st.sent, "errors": st.errors,
                             "parked": sorted(st.parked), "broken": st.broken})

    async def _drain(us):
        t0 = time.time()
        while any(st.inflight[u] for u in us):
            if time.time() - t0 > drain_timeout:
                raise TimeoutError("drain timeout")
            await asyncio.sleep(0.05)

    async def park(req: Request):
        body = await req.json()
        us = [u.rstrip("/") for u in body.get("upstreams", [])]
        done = []
        try:
            st.parked.update(us)
            await _drain(us)
            for u in us:
                r = await http.post(u + "/sleep")
                r.raise_for_status()
                done.append(u)
        except Exception as e:
            try:  # undo exactly what was done
                for u in done:
                    (await http.post(u + "/wake_up")).raise_for_status()
                st.parked.difference_update(us)
            except Exception:
                st.broken = True
            return JSONResponse({"ok": False, "error": repr(e)}, status_code=500)
        return JSONResponse({"ok": True, "parked": sorted(st.parked)})

    async def unpark(req: Request):
        body = await req.json()
        us = [u.rstrip("/") for u in body.get("upstreams", [])]
        try:
            for u in us:
                (await http.post(u + "/wake_up")).raise_for_status()
            st.parked.difference_update(us)
        except Exception as e:
            return JSONResponse({"ok": False, "error": repr(e)}, status_code=500)
        return JSONResponse({"ok": True, "parked": sorted(st.parked)})

    async def park_state(req: Request):
        return JSONResponse({"parked": sorted(st.parked), "active": [u for u in st.up if u not in st.parked]})

    async def proxy(req: Request):
        path = req.url.path + (("?" + req.url.query) if req.url.query else "")
        if req.method == "GET":
            u = st.up[0]
            r = await http.get(u + path)
            return Response(r.content, status_code=r.status_code, media_type=r.headers.get("content-type"))
        u = st.pick()
        if u is None:
            return JSONResponse({"error": "no active upstream"}, status_code=503)
        st.inflight[u] += 1
        st.sent[u] += 1
        try:
            r = await http.post(u + path, content=await req.body(), headers={"content-type": "application/json"})
            return Response(r.content, status_code=r.status_code, media_type=r.headers.get("content-type"))
        except Exception as e:
            st.errors[u] += 1
            return JSONResponse({"error": repr(e)}, status_code=502)
        finally:
            st.inflight[u] -= 1

    routes = [Route("/health", health), Route("/lb_stats", stats), Route("/park", park, methods=["POST"]),
              Route("/unpark", unpark, methods=["POST"]), Route("/park_state", park_state),
              Route("/{path:path}", proxy, methods=["GET", "POST"])]
    app = Starlette(routes=routes)
    app.state.proxy = st
    return app


class LoadBalancedClient:
    """Picks a replica index per call: affinity first (a task sticks to one replica), weighted round
    robin for new tasks, migration when the sticky replica is `migrate_margin` requests busier than the
    least-loaded active replica."""

    def __init__(self, base_urls: List[str], weights: Optional[List[int]] = None, migrate_margin: int = 8,
                 client: Optional[httpx.AsyncClient] = None, headers: Optional[List[dict]] = None,
                 error: Optional[Callable[[int, str], Exception]] = None):
        self.urls = [u.rstrip("/") for u in base_urls]
        self.headers = list(headers or [{} for _ in self.urls])
        self.error = error            # status, body -> the exception a failed call raises (default: httpx's)
        self.weights = list(weights or [1] * len(self.urls))
        self.active = [True] * len(self.urls)
        self.inflight = [0] * len(self.urls)
        self.affinity: Dict[object, int] = {}
        self.margin = migrate_margin
        self.http = client or httpx.AsyncClient(timeout=httpx.Timeout(900.0, connect=10.0))
        self._rebuild()

    def _rebuild(self):
        self.schedule = [i for i, w in enumerate(self.weights) for _ in range(w) if self.active[i]]
        self._rr = itertools.cycle(self.schedule or [0])

    def add_replicas(self, urls: List[str], weights: Optional[List[int]] = None, active: bool = False) -> List[int]:
        idx = []
        for u, w in zip(urls, weights or [1] * len(urls)):
            self.urls.append(u.rstrip("/"))
            self.headers.append({})
            self.weights.append(w)
            self.active.append(active)
            self.inflight.append(0)
            idx.append(len(self.urls) - 1)
        self._rebuild()
        return idx

    def set_active(self, idxs: List[int], flag: bool) -> None:
        for i in idxs:
            self.active[i] = flag
        self._rebuild()

    def _least(self) -> int:
        act = [i for i in range(len(self.urls)) if self.active[i]]
        return min(act, key=lambda i: (self.inflight[i] / max(1, self.weights[i]), i))

    def pick_index(self) -> int:
        key = affinity_key.get()
        if key is not None:
            i = self.affinity.get(key)
            if i is not None and self.active[i]:
                j = self._least()
                if self.inflight[i] - self.inflight[j] > self.margin:
                    self.affinity[key] = j
                    return j
                return i
        i = next(self._rr)
        if not self.active[i]:
            i = self._least()
        if key is not None:
            self.affinity[key] = i
        return i

    async def chat(self, body: dict) -> dict:
        i = self.pick_index()
        self.inflight[i] += 1
        try:
            r = await self.http.post(self.urls[i] + "/v1/chat/completions", json=body, headers=self.headers[i])
            if r.status_code >= 400 and self.error is not None:
                raise self.error(r.status_code, r.text)
            r.raise_for_status()
            return r.json()
        finally:
            self.inflight[i] -= 1


def main(argv=None):
    """python -m phung5_b200.serve.router --port 8001 --upstream http://127.0.0.1:8101 --upstream ..."""
    import argparse

    import uvicorn
    ap = argparse.ArgumentParser()
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, required=True)
    ap.add_argument("--upstream", action="append", required=True)
    ap.add_argument("--drain-timeout", type=float, default=120.0)
    args = ap.parse_args(argv)
    uvicorn.run(build_proxy(args.upstream, args.drain_timeout), host=args.host, port=args.port, log_level="warning")


if __name__ == "__main__":
    main()
