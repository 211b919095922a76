"""End-to-end smoke client of the generation service (reference: tests/test_pipeline.py:1-310).

Sends one batch (stems + image URLs, data URLs or local paths), polls /status until COMPLETE (bounded),
downloads /results and reports per-stem outcome, code size and the diag header.

    python -m phung5_b200.app.smoke_client --url http://127.0.0.1:10006 --prompts prompts.txt [--seed 42]
prompts.txt: one "<stem> <image url or path>" per line (a bare path uses its file name as the stem).
"""
from __future__ import annotations

import argparse
import base64
import io
import json
import os
import sys
import time
import zipfile

import httpx


def load_prompts(path: str):
    out = []
    for line in open(path):
        line = line.strip()
        if not line or line.startswith("#"):
            continue
        parts = line.split(None, 1)
        stem, src = (parts[0], parts[1]) if len(parts) == 2 else (os.path.splitext(os.path.basename(parts[0]))[0], parts[0])
        if os.path.exists(src):
            mime = "image/png" if src.lower().endswith(".png") else "image/jpeg"
            src = f"data:{mime};base64," + base64.b64encode(open(src, "rb").read()).decode()
        out.append({"stem": stem, "image_url": src})
    return out


def run(url: str, prompts, seed: int = 42, timeout_s: float = 7200.0, poll_s: float = 5.0, client=None) -> dict:
    cl = client or httpx.Client(base_url=url, timeout=60.0)
    t0 = time.time()
    while True:
        st = cl.get("/status").json()
        if st["status"] in ("ready", "complete"):
            break
        if time.time() - t0 > timeout_s:
            raise TimeoutError(f"service not ready: {st}")
        time.sleep(poll_s)
    r = cl.post("/generate", json={"prompts": prompts, "seed": seed})
    r.raise_for_status()
    t1 = time.time()
    while True:
        st = cl.get("/status").json()
        if st["status"] == "complete":
            break
        if time.time() - t1 > timeout_s:
            raise TimeoutError(f"batch not complete after {timeout_s}s: {st}")
        time.sleep(poll_s)
    z = zipfile.ZipFile(io.BytesIO(cl.get("/results").content))
    files = {n: z.read(n).decode() for n in z.namelist()}
    failed = json.loads(files.pop("_failed.json", "[]"))
    header = next((v.splitlines()[0] for v in files.values()), "")
    return {"wall_s": round(time.time() - t1, 1), "ok": sorted(n[:-3] for n in files), "failed": failed,
            "bytes": {n[:-3]: len(v) for n, v in files.items()}, "header": header}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--url", default="http://127.0.0.1:10006")
    ap.add_argument("--prompts", required=True)
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--timeout", type=float, default=7200.0)
    args = ap.parse_args(argv)
    res = run(args.url, load_prompts(args.prompts), args.seed, args.timeout)
    print(json.dumps(res, indent=1))
    sys.exit(0 if res["ok"] else 1)


if __name__ == "__main__":
    main()
