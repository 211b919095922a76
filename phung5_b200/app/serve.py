"""HTTP API of the generation service.

Reference: pipeline_service/serve.py (lifespan :140-170, /generate :190-233, /results :236-252, debug routes,
`_diag_header` :107-137). Routes:

  GET  /health                         200 while the process is up
  GET  /status?replacements_remaining  {"status", "progress", "total", "payload"}; replacements_remaining == 0
                                       on a REPLACE service forces WARMING_UP (generate anyway)
  POST /generate                       {"prompts": [{"stem", "image_url"}], "seed"} -> {"accepted": n};
                                       503 while warming up; the same stems while generating are idempotent;
                                       409 in any other non-accepting state; a new batch cancels a finished one
  GET  /results                        zip of <stem>.js (each prefixed with the `// miner-diag:` line) plus
                                       _failed.json; 409 unless COMPLETE
  GET  /debug/tasks, /debug/tasks/{stem} (202 while pending), /debug/logs, /debug/stats
"""
from __future__ import annotations

import asyncio
import collections
import io
import json
import logging
import os
import zipfile
from contextlib import asynccontextmanager
from typing import Dict, Optional

from fastapi import FastAPI, HTTPException
from fastapi.responses import JSONResponse, Response, StreamingResponse

from .monitor import EngineProber, HealthWatcher
from .pipeline import GenerationPipeline
from .schemas import GenerateAccepted, GenerateRequest, StatusResponse
from .settings import Settings, load_settings
from .state import MinerState, MinerStatus, PipelineTask

log = logging.getLogger("phung5_b200.app")


class RingHandler(logging.Handler):
    def __init__(self, n: int = 2000):
        super().__init__()
        self.lines = collections.deque(maxlen=n)
        self.setFormatter(logging.Formatter("%(asctime)s %(levelname)s %(name)s: %(message)s"))

    def emit(self, record):
        try:
            self.lines.append(self.format(record))
        except Exception:  # noqa: BLE001
            pass


def build_app(settings: Settings, backends: Optional[Dict[str, object]] = None, watch: bool = True,
              preflight: Optional[dict] = None) -> FastAPI:
    state = MinerState()
    pipeline = GenerationPipeline(settings, state, backends=backends)
    ring = RingHandler()
    logging.getLogger("phung5_b200").addHandler(ring)
    lock = asyncio.Lock()

    @asynccontextmanager
    async def lifespan(app: FastAPI):
        state.diag.update(preflight or {})
        pipeline.startup()
        probers = {name: EngineProber(name, c.base_url, "") for name, c in settings.enabled_clients().items()}

        async def on_ready():
            """Coder probe before READY; False (a coder slower than min_tps) asks for a replacement."""
            if settings.warmup:
                return pipeline.probe_ok(await pipeline.run_coder_probe())
            return True

        watcher = HealthWatcher(state, probers, on_ready=on_ready)
        app.state.watcher = watcher
        if watch and probers:
            watcher.start()
        elif not probers:
            await on_ready()
            state.status = MinerStatus.READY
        yield
        watcher.stop()
        t = app.state.generation_task
        if t is not None and not t.done():
            t.cancel()
        pipeline.close()

    app = FastAPI(lifespan=lifespan)
    app.state.generation_task = None
    app.state.miner = state
    app.state.pipeline = pipeline

    @app.get("/health")
    async def health():
        return Response(status_code=200)

    @app.get("/status", response_model=StatusResponse)
    async def status(replacements_remaining: int = 0):
        state.replacements_remaining = replacements_remaining
        if replacements_remaining == 0 and state.status == MinerStatus.REPLACE:
            log.warning("remaining=0 on a REPLACE service: back to WARMING_UP to try generating")
            state.status = MinerStatus.WARMING_UP
        return state.to_status_response()

    @app.post("/generate", response_model=GenerateAccepted)
    async def generate(req: GenerateRequest):
        async with lock:
            if state.status == MinerStatus.WARMING_UP:
                raise HTTPException(503, "Still warming up")
            stems = sorted(p.stem for p in req.prompts)
            if state.status == MinerStatus.GENERATING and sorted(state.batch_stems) == stems:
                return GenerateAccepted(accepted=len(req.prompts))
            if state.status not in (MinerStatus.READY, MinerStatus.COMPLETE):
                return JSONResponse({"detail": f"Cannot accept batch in state {state.status.value}",
                                     "status": state.status.value, "progress": state.progress, "total": state.total},
                                    status_code=409)
            if len(set(stems)) != len(stems):
                raise HTTPException(422, "duplicate stems")
            t = app.state.generation_task
            if t is not None and not t.done():
                t.cancel()
                try:
                    await t
                except (asyncio.CancelledError, asyncio.TimeoutError):
                    pass
            tasks = [PipelineTask(stem=p.stem, image_url=p.image_url, seed=req.seed + settings.pipeline.seed_offset)
                     for p in req.prompts]
            state.reset_for_batch([p.stem for p in req.prompts], req.seed)

            async def run():
                try:
                    await pipeline.run_batch(tasks)
                except asyncio.CancelledError:
                    raise
                except Exception:  # noqa: BLE001
                    log.exception("run_batch crashed")
                finally:
                    if state.status == MinerStatus.GENERATING:
                        state.mark_complete()

            app.state.generation_task = asyncio.create_task(run())
        return GenerateAccepted(accepted=len(tasks))

    @app.get("/results")
    async def results():
        if state.status != MinerStatus.COMPLETE:
            raise HTTPException(409, f"Not complete, current status: {state.status.value}")
        header = state.diag_header()
        buf = io.BytesIO()
        with zipfile.ZipFile(buf, "w", zipfile.ZIP_DEFLATED) as zf:
            for stem, code in state.results.items():
                if not code.startswith("// miner-diag:"):
                    code = header + code
                zf.writestr(f"{stem}.js", code)
            if state.failed:
                zf.writestr("_failed.json", json.dumps([{"stem": s, "reason": r} for s, r in state.failed.items()],
                                                       indent=2))
        buf.seek(0)
        return StreamingResponse(buf, media_type="application/zip")

    @app.get("/debug/tasks")
    async def debug_tasks():
        done = {s: t.view() for s, t in state.tasks.items()}
        inflight = {s: t.view() for s, t in pipeline.current.items() if s not in done}
        return {"status": state.status.value, "batch": state.batch_index, "completed": list(done.values()),
                "in_flight": list(inflight.values()),
                "pending": [s for s in state.batch_stems if s not in done and s not in inflight]}

    @app.get("/debug/tasks/{stem}")
    async def debug_task(stem: str):
        t = state.tasks.get(stem)
        if t is not None:
            return t.view(full=True)
        cur = pipeline.current.get(stem)
        if cur is not None or stem in state.batch_stems:
            return JSONResponse(cur.view() if cur is not None else {"stem": stem, "status": "pending"}, status_code=202)
        raise HTTPException(404, f"unknown stem {stem}")

    @app.get("/debug/logs")
    async def debug_logs(n: int = 200):
        return {"lines": list(ring.lines)[-max(1, min(n, 2000)):]}

    @app.get("/debug/stats")
    async def debug_stats():
        out = {"batch": pipeline.stats.summary(), "header": pipeline.stats.header_parts(), "diag": state.diag}
        if pipeline.renderer is not None:
            out["renderer"] = pipeline.renderer.health()
        if pipeline.checker is not None:
            out["checker"] = pipeline.checker.counts
        return out

    return app


def main(argv=None):
    import argparse

    import uvicorn
    ap = argparse.ArgumentParser(description="phung5_b200 generation service")
    ap.add_argument("--config", default=os.environ.get("PHX_APP_CONFIG"))
    ap.add_argument("--preflight", default=os.environ.get("PHX_PREFLIGHT_JSON"))
    ap.add_argument("--host")
    ap.add_argument("--port", type=int)
    args = ap.parse_args(argv)
    settings = load_settings(args.config)
    pre = None
    if args.preflight and os.path.exists(args.preflight):
        with open(args.preflight) as f:
            pre = json.load(f).get("diag", {})
    logging.basicConfig(level=logging.INFO)
    app = build_app(settings, preflight=pre)
    uvicorn.run(app, host=args.host or settings.api.host, port=args.port or settings.api.port)


if __name__ == "__main__":
    main()
