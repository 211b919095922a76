"""Service boot: host limits -> preflight -> engines -> generation service.

Reference: pipeline_service/run.sh:1-127 (ulimit, renderer mode, OMP_NUM_THREADS=1, preflight, environment
builds, engine spawn, serve.py). Here, in order:
  1. raise the open-file limit to the hard limit; OMP/MKL threads to 1 unless set (the engines and the
     checker pool own the cores);
  2. preflight (`phung5_b200.utils.preflight`): GPU health bench and host facts, written to
     `<log_dir>/preflight.json`; its `diag` feeds the results header;
  3. spawn the local engines of every enabled client that has an `engine` section (`app.spawn`);
  4. run the HTTP service (`app.serve`) in this process; on exit the engines are stopped.

    python -m phung5_b200.app.boot --config configs/pipeline.yaml [--skip-preflight] [--log-dir logs]
"""
from __future__ import annotations

import argparse
import json
import logging
import os
import resource


def raise_nofile() -> int:
    soft, hard = resource.getrlimit(resource.RLIMIT_NOFILE)
    try:
        resource.setrlimit(resource.RLIMIT_NOFILE, (hard, hard))
        return hard
    except (ValueError, OSError):
        return soft


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default=os.environ.get("PHX_APP_CONFIG"))
    ap.add_argument("--log-dir", default="logs")
    ap.add_argument("--skip-preflight", action="store_true")
    ap.add_argument("--no-spawn", action="store_true", help="engines are managed elsewhere")
    args = ap.parse_args(argv)
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    os.environ.setdefault("MKL_NUM_THREADS", "1")
    nofile = raise_nofile()
    logging.basicConfig(level=logging.INFO, format="%(asctime)s %(levelname)s %(name)s: %(message)s")
    log = logging.getLogger("phung5_b200.app")
    os.makedirs(args.log_dir, exist_ok=True)
    from .settings import load_settings
    settings = load_settings(args.config)
    for n in settings.notes:
        log.info("settings: %s", n)
    diag = {"nofile": nofile}
    if settings.benchmark and not args.skip_preflight:
        from ..utils.preflight import run_preflight
        pre = run_preflight(thresholds=settings.preflight.model_dump())
        with open(os.path.join(args.log_dir, "preflight.json"), "w") as f:
            json.dump(pre, f, indent=1)
        diag.update(pre["diag"])
        log.info("preflight ok=%s diag=%s", pre["ok"], pre["diag"])
    spawner = None
    if not args.no_spawn:
        from .spawn import Spawner
        spawner = Spawner(settings, log_dir=args.log_dir)
        for j in spawner.jobs:
            log.info("engine %s: model=%s gpus=%s tp=%d dp=%d port=%d", j.name, j.model, j.gpu_ids, j.tp, j.dp, j.port)
        spawner.start()
    try:
        import uvicorn

        from .serve import build_app
        uvicorn.run(build_app(settings, preflight=diag), host=settings.api.host, port=settings.api.port)
    finally:
        if spawner is not None:
            spawner.stop()


if __name__ == "__main__":
    main()
