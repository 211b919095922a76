"""Headline benchmark: output tokens/s (and p50 TPOT) of Llama-3-70B-shaped block-scaled FP8
speculative decoding with tensor parallelism over the GPUs of one node.

Workload (Llama-3-70B FP8 serving benchmark): 64 requests sharing one 4096-token random prefix plus 512-token unique
random suffixes; an EAGLE-style one-layer draft head builds a 64-node top-k=8 tree (depth 6) per
request per step; the target verifies the tree with cascade attention over the shared prefix;
256 output tokens per request. Weights are random-init (no checkpoints offline), token ids are
synthetic, and the accepted length per request per step is drawn from a seeded Geometric(p=0.3)
capped at 6 (random weights never agree with their drafter; every step still computes the full
draft, verify, target sampling and accept walk).

A "step" is one speculative step of the whole batch. W warm-up steps, then exactly K timed steps
between barriers + device synchronisation, timed with CUDA events on the launching stream; the
per-rank time is reduced with MAX. Inputs are larger than L2 (70 GB of weights per step at TP1).
Then K more steps are timed end to end through the public engine API (host scheduling, pinned H2D
of step inputs, D2H of step results).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "output tok/s at Llama-3-70B FP8 TP8 spec decode, max over ranks; p50 TPOT"
# Mixtral-8x7B FP8 MoE (EP over the GPUs, attention tensor-parallel), k=4 chain speculation, batch 128 x 2048-token
# prompts, 128 output tokens: `--workload mixtral`
MIXTRAL_METRIC = "output tok/s at Mixtral-8x7B FP8 EP8 spec decode (k=4 chain), max over ranks; p50 TPOT"
WORKLOADS = {"mixtral": dict(model="mixtral-8x7b-fp8", batch=128, prefix=0, suffix=2048, out_tokens=128, mode="chain",
                             num_draft=4)}


def reference_arm(args, metric=METRIC):
    """The reference (huypg-zenai/phung5) is an application around external SGLang/vLLM engines: it has no
    setup.py/pyproject (pip refuses to install it) and its inference engines are downloaded at container
    start, so its own serving path cannot run offline here."""
    line = {"impl": "reference",
            "unavailable": "reference is not installable (no setup.py/pyproject.toml) and its SGLang/vLLM "
                           "engines are fetched from the network at start; no offline build of its serving path",
            "metric": metric, "n_gpus": args.gpus}
    print(json.dumps(line))


class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.rows = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout.strip()
                if out:
                    self.rows.append([x.strip() for x in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if len(r) > 5 + i and r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def _write_op_timing(rep, comm, rank, world, steps, ms):
    """PHX_OP_TIMING=1 (eager steps): per (phase, kernel) device ms per step, max over ranks, written as JSON to
    PHX_OP_TIMING_OUT (default op_timing.json) by rank 0."""
    reps = [rep]
    if comm is not None:
        import torch.distributed as dist
        reps = [None] * world
        dist.all_gather_object(reps, rep)
    out = {"steps": steps, "ms_per_step_max": 0.0, "kernels": {}, "phases": {}}
    for r in reps:
        for k, (v, n) in r["kernels"].items():
            cur = out["kernels"].get(k, [0.0, 0])
            out["kernels"][k] = [max(cur[0], round(v / steps, 4)), n // steps]
        for k, v in r["phases"].items():
            out["phases"][k] = max(out["phases"].get(k, 0.0), round(v / steps, 4))
    n_ar = sum(n for k, (v, n) in rep["kernels"].items() if k.endswith("tp_ar_norm"))
    if comm is not None and getattr(comm, "phase", None) is not None:
        ph = comm.phase_report(n_ar)           # this rank's fused-reduction phases (PHX_TP_PHASES=1)
        phs = [None] * world
        import torch.distributed as dist
        dist.all_gather_object(phs, ph)
        out["tp_phases_per_rank"] = phs
    ms_all = [ms] if comm is None else [comm.max_float(ms)]
    out["ms_per_step_max"] = round(ms_all[0] / steps, 3)
    if rank == 0:
        with open(os.environ.get("PHX_OP_TIMING_OUT", "op_timing.json"), "w") as f:
            json.dump(out, f, indent=1, sort_keys=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default=None, choices=[None, *WORKLOADS],
                    help="a named workload preset (overrides model / batch / prompt / spec flags)")
    ap.add_argument("--model", default="llama3-70b-fp8")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--prefix", type=int, default=4096)
    ap.add_argument("--suffix", type=int, default=512)
    ap.add_argument("--out-tokens", type=int, default=256)
    ap.add_argument("--tree-nodes", type=int, default=64)
    ap.add_argument("--topk", type=int, default=8)
    ap.add_argument("--depth", type=int, default=6)
    ap.add_argument("--mode", default="tree", choices=["tree", "chain"])
    ap.add_argument("--num-draft", type=int, default=4)
    ap.add_argument("--comm", default="fused", choices=["nccl", "fused"])
    ap.add_argument("--moe-dispatch", default="reduce", choices=["reduce", "a2a"],
                    help="MoE expert parallelism on the collective path (--comm nccl): all-reduce of every rank's "
                         "expert outputs, or all-to-all dispatch / combine of each rank's own tokens")
    ap.add_argument("--accept", default="geometric", choices=["geometric", "greedy", "sample"],
                    help="geometric: synthetic accept lengths (random weights never agree with their drafter); "
                         "greedy: target argmax along the tree; sample: seeded top-k 50 / top-p 0.9 / T = 1 target "
                         "sampling with the device accept walk (a step-cost comparison, not a throughput line)")
    ap.add_argument("--no-cascade", action="store_true")
    ap.add_argument("--layers", type=int, default=0, help="override layer count (smoke runs only; not a bench value)")
    ap.add_argument("--model-path", default=None, help="HF checkpoint directory instead of random-init weights")
    ap.add_argument("--draft-path", default=None, help="EAGLE head checkpoint directory (with --model-path)")
    args = ap.parse_args()
    metric = METRIC
    if args.workload:
        for k, v in WORKLOADS[args.workload].items():
            setattr(args, k, v)
        metric = MIXTRAL_METRIC

    if args.impl == "reference":
        reference_arm(args, metric)
        return

    from phung5_b200 import ops
    from phung5_b200.config import CacheConfig, DraftConfig, EngineConfig, ParallelConfig, SpecConfig, preset
    from phung5_b200.engine.engine import LLMEngine
    from phung5_b200.engine.oracle import SamplingParams
    from phung5_b200.parallel.comm import NcclCommunicator, init_distributed

    rank, world, local = init_distributed()
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = NcclCommunicator() if world > 1 else None
    if world > 1 and args.comm == "fused":
        from phung5_b200.parallel.fused import FusedCommunicator
        comm = FusedCommunicator()

    target = drafter = None
    if args.model_path:
        from phung5_b200.weights.loader import load_eagle, load_model
        mc, target = load_model(args.model_path, dev, rank, world)
        if args.draft_path:
            drafter = load_eagle(args.draft_path, mc, dev, rank, world)
    else:
        mc = preset(args.model)
    if args.layers:
        mc.num_layers = args.layers
    spec = SpecConfig(mode=args.mode, tree_nodes=args.tree_nodes, topk=args.topk, depth=args.depth,
                      num_draft=args.num_draft, accept="geometric" if args.accept == "geometric" else "exact",
                      accept_p=0.3, accept_cap=6, accept_seed=0)
    # the shared prefix pages are held once (prefix cache); each request adds its suffix, outputs and
    # speculation scratch
    per_req_pages = (args.suffix + args.out_tokens + 2 * args.tree_nodes + 128) // 64 + 3
    num_pages = args.prefix // 64 + args.batch * per_req_pages + 64
    ecfg = EngineConfig(model=mc, spec=spec, draft=DraftConfig(kind="eagle"),
                        parallel=ParallelConfig(tp=world, comm=args.comm, moe_dispatch=args.moe_dispatch),
                        cache=CacheConfig(page_size=64, num_pages=num_pages, enable_cascade=not args.no_cascade),
                        max_prefill_tokens=8192, seed=0)
    t0 = time.time()
    eng = LLMEngine(ecfg, device=dev, comm=comm, target=target, drafter=drafter,
                    max_context=args.prefix + args.suffix + args.out_tokens + 512)
    torch.cuda.synchronize()
    t_init = time.time() - t0

    g = torch.Generator().manual_seed(1234)
    prefix = torch.randint(0, mc.vocab, (args.prefix,), generator=g).tolist() if args.prefix else []
    prompts = [prefix + torch.randint(0, mc.vocab, (args.suffix,), generator=g).tolist() for _ in range(args.batch)]
    sp = (SamplingParams(temperature=1.0, top_k=50, top_p=0.9, seed=7, max_new_tokens=args.out_tokens)
          if args.accept == "sample" else SamplingParams(temperature=0.0, max_new_tokens=args.out_tokens))
    for p in prompts:
        eng.add_request(p, sp)
    t0 = time.time()
    while eng.waiting:
        eng.step()
    torch.cuda.synchronize()
    t_prefill = time.time() - t0

    def barrier():
        if comm is not None:
            comm.barrier()

    for _ in range(args.warmup):
        eng.step()
    ops.check_status(dev)

    # ---- device-timed region ----
    n_before = eng.stats["tokens_out"]
    per_req_before = {r.rid: len(r.out) for r in eng.running}
    l0 = ops.launches()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    phys = int(vis.split(",")[local]) if vis else local
    profile = os.environ.get("PHX_PROFILE_TIMED") == "1"   # ncu --profile-from-start off captures only this
    ops.timing_reset()
    if getattr(comm, "phase", None) is not None:
        comm.phase_report(1)                   # restart the fused-reduction phase counters
    with ClockSampler(phys) as clk:
        if profile:
            torch.cuda.profiler.start()
        ev0.record()
        for _ in range(args.steps):
            eng.step()
        ev1.record()
        torch.cuda.synchronize()
        if profile:
            torch.cuda.profiler.stop()
    barrier()
    launches = ops.launches() - l0
    ms = ev0.elapsed_time(ev1)
    if ops.OP_TIMING:
        _write_op_timing(ops.timing_report(), comm, rank, world, args.steps, ms)
    ms = comm.max_float(ms) if comm is not None else ms
    tokens = eng.stats["tokens_out"] - n_before
    live = [r for r in eng.running]
    tpot = [ms / max(1, len(r.out) - per_req_before.get(r.rid, 0)) for r in live if r.rid in per_req_before]
    ops.check_status(dev)

    # ---- end-to-end region through the public API ----
    from phung5_b200.engine.attn_meta import UPLOADED_BYTES
    h2d0, d2h0 = eng.stats["h2d_bytes"] + UPLOADED_BYTES[0], eng.stats["d2h_bytes"]
    e2e_tokens = 0
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    step_wall = []
    for _ in range(args.steps):
        ts = time.perf_counter()
        for o in eng.step():
            e2e_tokens += len(o.new_tokens)
        step_wall.append(round(1e3 * (time.perf_counter() - ts), 1))
    e2e_s = time.perf_counter() - t0
    if os.environ.get("PHX_STEP_TIMES") == "1" and rank == 0:   # per-step wall ms of the end-to-end region
        print(json.dumps({"e2e_step_wall_ms": step_wall, "graph_replays": eng.stats.get("graph_replays"),
                          "graphs": len(eng._graphs) if eng._graphs is not None else None}), file=sys.stderr)
    e2e_s = comm.max_float(e2e_s) if comm is not None else e2e_s
    h2d = (eng.stats["h2d_bytes"] + UPLOADED_BYTES[0] - h2d0) / args.steps
    d2h = (eng.stats["d2h_bytes"] - d2h0) / args.steps

    value = tokens / (ms / 1e3)
    if rank == 0:
        line = {
            "metric": metric, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp8_block+bf16",
            "data": "synthetic token ids, " + ("checkpoint weights" if args.model_path else "random-init weights")
                    + {"geometric": ", geometric(p=0.3, cap 6) synthetic acceptance",
                       "greedy": ", target-greedy acceptance",
                       "sample": ", seeded target sampling (T 1, top-k 50, top-p 0.9) with the device accept walk"}[args.accept],
            "config": {"model": mc.name + (f"-{mc.num_layers}L" if args.layers else ""), "global_batch": args.batch,
                       "seq_len": args.prefix + args.suffix, "shared_prefix": args.prefix, "suffix": args.suffix,
                       "out_tokens": args.out_tokens, "spec": args.mode,
                       "tree_nodes": args.tree_nodes if args.mode == "tree" else args.num_draft + 1,
                       "topk": args.topk, "depth": args.depth if args.mode == "tree" else args.num_draft, "parallelism": f"tp{world}",
                       "comm": (args.comm + ("+nvls" if getattr(comm, "mc", 0) else "")) if world > 1 else "none",
                       "cascade": not args.no_cascade, "l2": "inputs larger than L2 (weights stream every step)"},
            "p50_tpot_ms": round(statistics.median(tpot), 3) if tpot else None,
            "tokens_per_step": round(tokens / args.steps, 2),
            "e2e": {"value": round(e2e_tokens / e2e_s, 2), "unit": "tok/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h)},
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "init_s": round(t_init, 1), "prefill_s": round(t_prefill, 1),
        }
        if eng.host_times:
            n = 2 * args.steps + args.warmup
            line["host_ms_per_step"] = {k: round(1e3 * v / n, 2) for k, v in eng.host_times.items()}
        print(json.dumps(line))
    if comm is not None:
        import torch.distributed as dist
        eng._graphs = None          # release the step graphs (they hold the fused kernels) before teardown
        del eng
        if hasattr(comm, "close"):
            comm.close()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
