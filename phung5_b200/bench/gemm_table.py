"""Measure the per-shape FP8 / bf16 GEMM table (ops/gemm_table.json).

    python -m phung5_b200.bench.gemm_table [--out phung5_b200/ops/gemm_table.json] [--iters 7]

For every per-rank linear shape of the served models at tensor parallelism 1/2/4/8 (Llama-3-70B and -8B: qkv,
o, down, the EAGLE head's fc; the bf16 lm_head) and every M bucket (draft rounds, catch-up, verify, prefill
chunks), each tile configuration the kernel offers is timed with CUDA events after warm-up, flushing L2 before
every launch, round-robin with the default choice over three passes (best of each), and the fastest is recorded:
  fp8:  BN 128 / 256 x hardware block scaling (tcgen05 kind::mxf8f6f4) or per-K-block promotion x CTA pairs
        (cta_group::2, BN 256 only) x the split-K tail (hardware-scaled single-CTA tiles)
  bf16: BN 128 / 256 x the split-K tail
The reference keeps the same kind of table for its sm90 CUTLASS FP8 GEMM (docker/opt/v5/wq/kopt_wq.py:92-116,
kopt_wq_table.json: tile, cluster and schedule per (N, K, M)); here the choices are the tcgen05 kernel's.
Results within 2 % of the default choice keep the default (no churn from timing noise).
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from .. import ops
from ..ops import gemm_table
from ..weights.quant import FP8_DTYPE, pow2_scale
from .kernels import time_it

MODELS = {"llama3-70b": dict(h=8192, q=8192, kv=1024, f=28672, v=128256),
          "llama3-8b": dict(h=4096, q=4096, kv=1024, f=14336, v=128256)}
M_BUCKETS = (128, 512, 1024, 4096, 8192)


def shapes():
    out = set()
    for d in MODELS.values():
        for tp in (1, 2, 4, 8):
            out.add(("fp8", (d["q"] + 2 * d["kv"]) // tp, d["h"]))     # qkv
            out.add(("fp8", d["h"], d["q"] // tp))                     # o
            out.add(("fp8", d["h"], d["f"] // tp))                     # down
            out.add(("bf16", d["v"] // tp, d["h"]))                    # lm_head
        out.add(("fp8", d["h"], 2 * d["h"]))                           # EAGLE fc
    return sorted(out)


def fp8_configs(m):
    cfgs = [dict(bn=b, hws=h, pair=False, split=1) for b in (128, 256) for h in (True, False)]
    cfgs += [dict(bn=b, hws=True, pair=False, split=0) for b in (128, 256)]   # automatic split-K tail
    if m > 128:
        cfgs.append(dict(bn=256, hws=True, pair=True, split=1))
    return cfgs


def measure(kind, n, k, m, iters, rounds=3):
    """-> (fastest config, its ms, the default choice's ms). Candidates and the default are timed round-robin
    (`rounds` passes, best of each) so a slow drift of the clock under the power cap favours none of them."""
    dev = "cuda"
    if kind == "fp8":
        xq, xs = ops.act_quant(torch.randn(m, k, device=dev, dtype=torch.bfloat16))
        wq = (torch.randn(n, k, device=dev, dtype=torch.bfloat16) * 0.05).to(FP8_DTYPE)
        ws = pow2_scale(torch.rand((n + 127) // 128, k // 128, device=dev) * 4.48)
        out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        cands = [(c, (lambda c=c: ops.gemm_fp8_block(xq, xs, wq, ws, out=out, bn=c["bn"], hw_scale=c["hws"],
                                                     pair=c["pair"], split=c["split"], use_table=False)))
                 for c in fp8_configs(m)]
        default = lambda: ops.gemm_fp8_block(xq, xs, wq, ws, out=out, use_table=False)
    else:
        x = torch.randn(m, k, device=dev, dtype=torch.bfloat16)
        w = torch.randn(n, k, device=dev, dtype=torch.bfloat16) * 0.05
        out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        cands = [(dict(bn=b, split=sp), (lambda b=b, sp=sp: ops.gemm_bf16(x, w, out=out, bn=b, split=sp, use_table=False)))
                 for b in (128, 256) for sp in (1, 0)]
        default = lambda: ops.gemm_bf16(x, w, out=out, use_table=False)
    best_t = [float("inf")] * len(cands)
    d_ms = float("inf")
    for _ in range(rounds):
        d_ms = min(d_ms, time_it(default, iters))
        for i, (_, fn) in enumerate(cands):
            best_t[i] = min(best_t[i], time_it(fn, iters))
    ops.check_status()
    i = min(range(len(cands)), key=lambda j: best_t[j])
    torch.cuda.empty_cache()
    return cands[i][0], best_t[i], d_ms


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=gemm_table.PATH)
    ap.add_argument("--iters", type=int, default=7)
    args = ap.parse_args()
    table = {"about": "fastest tcgen05 GEMM configuration per (kind, N, K, M bucket); phung5_b200/bench/gemm_table.py",
             "m_buckets": list(M_BUCKETS), "entries": {}}
    for kind, n, k in shapes():
        for m in M_BUCKETS:
            best, best_ms, default_ms = measure(kind, n, k, m, args.iters)
            key = gemm_table.key(kind, n, k, m)
            keep_default = best_ms > 0.98 * default_ms
            table["entries"][key] = {**({} if keep_default else best), "ms": round(min(best_ms, default_ms), 5),
                                     "default_ms": round(default_ms, 5)}
            print(json.dumps({"key": key, **table["entries"][key]}), flush=True)
    os.makedirs(os.path.dirname(os.path.abspath(args.out)), exist_ok=True)
    with open(args.out, "w") as f:
        json.dump(table, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
