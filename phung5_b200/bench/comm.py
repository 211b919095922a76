"""Tensor-parallel collective microbenchmarks (run under torchrun, one rank per GPU).

    torchrun --nproc-per-node 8 -m phung5_b200.bench.comm [--iters 20]

Times, with CUDA events after warm-up and the maximum over ranks:
  ar_norm  fused reduce-scatter + residual + RMSNorm + FP8 quant + all-gather (csrc/tp_fused.cu) at the verify
           shape (M = 4096 rows of H = 8192) and the draft shape (M = 512);
  gather   the fused candidate exchange (512 rows x top-8 (value, index) + lse);
  nccl     torch.distributed all_reduce of the same [M, H] bf16 partial (the unfused baseline's collective).
--sweep: the fused-kernel sweep instead: AR + residual + RMSNorm + FP8 quant at tokens {1 ... 8192} and
vocab-sharded top-k / top-p sampling at batch {1, 64, 256} x k {1, 8, 50}, each against NCCL + the separate
kernels, timed both as eager launches and as CUDA-graph replays (the engine's step is a graph).
NVLink bytes per ar_norm per GPU: (W-1)/W of the partial rows read (bf16) plus (W-1)/W of the fp8 rows and
scales written; reported against the measured peer-copy bandwidth of 770 GB/s per direction.
o_proj / down_proj + reduction: the fused path (GEMM epilogue stores rows to their owners, reduction over local
slots) against GEMM + pulling reduction, each as a fraction of the path's roofline (the slower of the GEMM's
FLOPs at the fp8 peak and its NVLink bytes at 770 GB/s).
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

from ..parallel.comm import init_distributed
from ..parallel.fused import FusedCommunicator

NVLINK_GBS = 770.0


def _time(fn, iters):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    b.synchronize()
    ms = a.elapsed_time(b) / iters
    t = torch.tensor([ms], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _time_graph(fn, iters):
    """Device time of one call captured in a CUDA graph (replayed `iters` times between events, max over
    ranks): the engine runs these paths inside its step graph, so host launch cost is not part of it. Returns
    (ms, graph); the caller drops the graph before the communicator or process group is torn down."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    dist.barrier()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    ms = _time(g.replay, iters)
    return ms, g


def ar_norm_sweep(comm, world, iters, H=8192, tokens=(1, 16, 128, 512, 1024, 4096, 8192)):
    """Fused-kernel sweep (a): TP all-reduce + residual + RMSNorm + FP8 quant at hidden 8192 over `tokens`, bf16
    partials and residual ~N(0, 1), unit norm weight. Fused: one ar_norm launch (reduce-scatter by peer loads,
    norm + quant of the owned rows, all-gather of the fp8 rows and scales by peer stores). Baseline: NCCL
    all_reduce of the bf16 partial, then the add + RMSNorm + FP8 quant kernel on every rank. Roofline: the bytes
    that must cross NVLink per GPU ((W-1)/W of the bf16 rows in, (W-1)/W of the fp8 rows + scales out) at the
    measured 770 GB/s peer-copy rate."""
    from .. import ops
    dev = comm.device
    w = torch.ones(H, device=dev, dtype=torch.bfloat16)
    rows = []
    for m in tokens:
        g = torch.Generator(device=dev).manual_seed(11 + comm.rank)
        part = torch.randn(m, H, device=dev, dtype=torch.bfloat16, generator=g)
        h0 = torch.randn(m, H, device=dev, dtype=torch.bfloat16, generator=torch.Generator(device=dev).manual_seed(5))

        comm.partial(m).copy_(part)
        comm.h(m).copy_(h0)
        x = part.clone()
        h = h0.clone()

        def nccl():
            dist.all_reduce(x)
            ops.add_rmsnorm_quant(h, x, w, 1e-5)
        f_ms = _time(lambda: comm.ar_norm(m, w, 1e-5), iters)
        mc, comm.mc = comm.mc, 0
        p_ms = _time(lambda: comm.ar_norm(m, w, 1e-5), iters)        # peer loads / stores only
        comm.mc = mc
        n_ms = _time(nccl, iters)
        fg_ms, g1 = _time_graph(lambda: comm.ar_norm(m, w, 1e-5), iters)
        ng_ms, g2 = _time_graph(nccl, iters)
        del g1, g2
        nv = (world - 1) / world * m * H * (2 + 1 + 4 / 128)
        # with NVLS the busier direction carries each GPU's partial rows for the other owners (read by the
        # switch) plus its own result rows once (the switch copies them to every rank)
        nv_mc = ((world - 1) / world * 2 + (1 + 4 / 128) / world) * m * H
        roof = (nv_mc if mc else nv) / NVLINK_GBS / 1e6
        rows.append({"op": "sweep_ar_norm_quant", "tokens": m, "H": H, "nvls": bool(mc), "fused_ms": round(f_ms, 4),
                     "fused_p2p_ms": round(p_ms, 4), "nccl_plus_kernel_ms": round(n_ms, 4),
                     "speedup": round(n_ms / f_ms, 2), "roofline_ms": round(roof, 5),
                     "fused_frac_of_roofline": round(roof / f_ms, 3),
                     "p2p_frac_of_roofline": round(nv / NVLINK_GBS / 1e6 / p_ms, 3),
                     "graph_fused_ms": round(fg_ms, 4), "graph_nccl_plus_kernel_ms": round(ng_ms, 4),
                     "graph_speedup": round(ng_ms / fg_ms, 2)})
    return rows


def sampling_sweep(comm, world, iters, vocab=128256, batches=(1, 64, 256), ks=(1, 8, 50), top_p=0.9):
    """Fused-kernel sweep (b): vocab-sharded top-k / top-p sampling, vocab 128256 split over the ranks, bf16
    logits ~N(0, 2^2), temperature 1, top-p 0.9, batch x k. Fused: per-shard candidates (csrc/sample.cu
    sample_candidates), one in-kernel exchange of the [rows, chunks, KC] candidate lists over NVLink
    (FusedCommunicator.gather), one draw kernel (spec_accept on a one-node tree: the draw of the step's final
    coin). Baseline: NCCL all_gather of the logits shards, re-layout to [B, V], then the same two kernels over
    the full vocab on every rank. Both arms must draw identical tokens. Roofline: the shard read from HBM at
    the measured copy rate plus the candidate bytes each GPU receives at 770 GB/s (microseconds: these sizes
    are launch- and latency-bound)."""
    from .. import ops
    from .kernels import peaks
    dev = comm.device
    vl = vocab // world
    off = comm.rank * vl
    hbm = peaks()["hbm_gbs"]
    rows = []
    for b in batches:
        g = torch.Generator(device=dev).manual_seed(17)
        full = (torch.randn(b, vl * world, device=dev, generator=g) * 2.0).to(torch.bfloat16)
        shard = full[:, off:off + vl].contiguous()
        gbuf = torch.empty(world, b, vl, device=dev, dtype=torch.bfloat16)
        tokens = torch.zeros(b, 1, device=dev, dtype=torch.int64)
        parent = torch.full((b, 1), -1, device=dev, dtype=torch.int64)
        temp = torch.ones(b, device=dev)
        topp = torch.full((b,), top_p, device=dev)
        seed = torch.arange(b, device=dev, dtype=torch.int64) + 7
        committed = torch.zeros(b, device=dev, dtype=torch.int64)
        for k in ks:
            kc = 16 if k <= 16 else 64
            topk = torch.full((b,), k, device=dev, dtype=torch.int32)
            res = {}

            def fused():
                res["f"] = ops.spec_sample_accept(shard, tokens, parent, temp, topk, topp, seed, committed, 0, kc,
                                                  vocab_offset=off, gather=comm.gather)[1]

            def nccl():
                dist.all_gather_into_tensor(gbuf.view(-1), shard.view(-1))
                lay = gbuf.permute(1, 0, 2).reshape(b, world * vl)
                res["n"] = ops.spec_sample_accept(lay, tokens, parent, temp, topk, topp, seed, committed, 0, kc)[1]
            f_ms = _time(fused, iters)
            n_ms = _time(nccl, iters)
            same = bool(torch.equal(res["f"], res["n"]))
            fg_ms, g1 = _time_graph(fused, iters)
            ng_ms, g2 = _time_graph(nccl, iters)
            del g1, g2
            nch = int(ops.ext().sample_chunks(vl))
            roof = (b * vl * 2 / hbm / 1e6) + (world - 1) * b * nch * kc * 8 / NVLINK_GBS / 1e6
            rows.append({"op": "sweep_sampling", "batch": b, "k": k, "top_p": top_p, "vocab_shard": vl,
                         "fused_ms": round(f_ms, 4), "nccl_plus_kernel_ms": round(n_ms, 4),
                         "speedup": round(n_ms / f_ms, 2), "roofline_ms": round(roof, 5),
                         "fused_frac_of_roofline": round(roof / f_ms, 3), "same_tokens": same,
                         "graph_fused_ms": round(fg_ms, 4), "graph_nccl_plus_kernels_ms": round(ng_ms, 4),
                         "graph_speedup": round(ng_ms / fg_ms, 2)})
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--hidden", type=int, default=8192)
    ap.add_argument("--sweep", action="store_true", help="only the fused-kernel sweep (tokens 1..8192, sampling)")
    args = ap.parse_args()
    rank, world, local = init_distributed()
    dev = torch.device("cuda", local)
    H = args.hidden
    comm = FusedCommunicator(max_tokens=8192, hidden=H)
    if args.sweep:
        for sweep in (lambda: ar_norm_sweep(comm, world, args.iters, H), lambda: sampling_sweep(comm, world, args.iters)):
            rows = sweep()
            if rank == 0:
                for o in rows:
                    print(json.dumps({"world": world, **o}), flush=True)
        comm.close()
        dist.destroy_process_group()
        return
    w = torch.ones(H, device=dev, dtype=torch.bfloat16)
    out = []
    for m in (4096, 512):
        comm.partial(m).copy_(torch.randn(m, H, device=dev, dtype=torch.bfloat16))
        comm.h(m).zero_()
        ms = _time(lambda: comm.ar_norm(m, w, 1e-5), args.iters)
        nv = (world - 1) / world * m * H * (2 + 1 + 4 / 128)
        out.append({"op": "ar_norm", "M": m, "H": H, "ms": round(ms, 4),
                    "nvlink_gbs": round(nv / ms / 1e6, 1), "frac_of_770": round(nv / ms / 1e6 / NVLINK_GBS, 3)})
        x = torch.randn(m, H, device=dev, dtype=torch.bfloat16)
        ms = _time(lambda: dist.all_reduce(x), args.iters)
        out.append({"op": "nccl_all_reduce", "M": m, "H": H, "ms": round(ms, 4)})
    # row-parallel projections then the reduction: separate GEMM + pull, vs scatter epilogue + local sum.
    # Roofline of the fused path: the slower of the GEMM at the fp8 peak (2 x the bf16 figure) and the bytes
    # that must cross NVLink (reduce-scatter of bf16 rows + all-gather of fp8 rows and scales) at 770 GB/s.
    from ..models.llama import Linear
    from .. import ops
    from ..weights.quant import quant_weight_block
    from .kernels import peaks
    fp8_tflops = 2 * peaks()["bf16_tflops"]
    m = 4096
    for name, kfull in (("o_proj", 8192), ("down_proj", 28672)):
        kdim = kfull // world
        wq, ws = quant_weight_block(torch.randn(H, kdim, device=dev) * 0.02)
        lin = Linear(wq, ws)
        xq, xs = ops.act_quant(torch.randn(m, kdim, device=dev, dtype=torch.bfloat16))
        comm.h(m).zero_()

        def pull():
            lin((xq, xs), out=comm.partial(m))
            comm.ar_norm(m, w, 1e-5)

        def push():
            comm.project(lin, (xq, xs), m)
            comm.ar_norm(m, w, 1e-5, recv=True)
        flops = 2.0 * m * H * kdim
        nv = (world - 1) / world * m * H * (2 + 1 + 4 / 128)
        roof_ms = max(flops / fp8_tflops / 1e9, nv / NVLINK_GBS / 1e6)
        gemm_ms = _time(lambda: lin((xq, xs), out=comm.partial(m)), args.iters)
        out.append({"op": f"{name}_gemm_alone", "M": m, "K": kdim, "ms": round(gemm_ms, 4)})
        for tag, fn in (("then_ar_norm_pull", pull), ("scatter_then_ar_norm_recv", push)):
            comm.phase_report(1)
            ms = _time(fn, args.iters)
            out.append({"op": f"{name}_{tag}", "M": m, "K": kdim, "ms": round(ms, 4), "roofline_ms": round(roof_ms, 4),
                        "frac_of_roofline": round(roof_ms / ms, 3), **comm.phase_report(args.iters + 3)})
    v = torch.randn(512, 8, device=dev)
    i = torch.randint(0, 1000, (512, 8), device=dev)
    lse = torch.randn(512, 1, device=dev)
    ms = _time(lambda: comm.gather([v, i, lse]), args.iters)
    out.append({"op": "gather_topk8_512", "ms": round(ms, 4)})
    if rank == 0:
        for o in out:
            print(json.dumps({"world": world, **o}))
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
