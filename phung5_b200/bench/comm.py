"""Tensor-parallel collective microbenchmarks (run under torchrun, one rank per GPU).

    torchrun --nproc-per-node 8 -m phung5_b200.bench.comm [--iters 20]

Times, with CUDA events after warm-up and the maximum over ranks:
  ar_norm  fused reduce-scatter + residual + RMSNorm + FP8 quant + all-gather (csrc/tp_fused.cu) at the verify
           shape (M = 4096 rows of H = 8192) and the draft shape (M = 512);
  gather   the fused candidate exchange (512 rows x top-8 (value, index) + lse);
  nccl     torch.distributed all_reduce of the same [M, H] bf16 partial (the unfused baseline's collective).
NVLink bytes per ar_norm per GPU: (W-1)/W of the partial rows read (bf16) plus (W-1)/W of the fp8 rows and
scales written; reported against the measured peer-copy bandwidth of 770 GB/s per direction.
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--hidden", type=int, default=8192)
    args = ap.parse_args()
    rank, world, local = init_distributed()
    dev = torch.device("cuda", local)
    H = args.hidden
    comm = FusedCommunicator(max_tokens=4096, hidden=H)
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
    # row-parallel o_proj (K = 8192 / W) then the reduction: separate GEMM + pull, vs scatter epilogue + local sum
    from ..models.llama import Linear
    from .. import ops
    from ..weights.quant import quant_weight_block
    kdim = 8192 // world
    wq, ws = quant_weight_block(torch.randn(H, kdim, device=dev) * 0.02)
    lin = Linear(wq, ws)
    m = 4096
    xq, xs = ops.act_quant(torch.randn(m, kdim, device=dev, dtype=torch.bfloat16))
    comm.h(m).zero_()

    def pull():
        lin((xq, xs), out=comm.partial(m))
        comm.ar_norm(m, w, 1e-5)

    def push():
        comm.project(lin, (xq, xs), m)
        comm.ar_norm(m, w, 1e-5, recv=True)
    gemm_ms = _time(lambda: lin((xq, xs), out=comm.partial(m)), args.iters)
    out.append({"op": "o_proj_gemm_alone", "M": m, "K": kdim, "ms": round(gemm_ms, 4)})
    out.append({"op": "o_proj_then_ar_norm_pull", "M": m, "K": kdim, "ms": round(_time(pull, args.iters), 4)})
    out.append({"op": "o_proj_scatter_then_ar_norm_recv", "M": m, "K": kdim, "ms": round(_time(push, args.iters), 4)})
    v = torch.randn(512, 8, device=dev)
    i = torch.randint(0, 1000, (512, 8), device=dev)
    lse = torch.randn(512, 1, device=dev)
    ms = _time(lambda: comm.gather([v, i, lse]), args.iters)
    out.append({"op": "gather_topk8_512", "ms": round(ms, 4)})
    if rank == 0:
        for o in out:
            print(json.dumps({"world": world, **o}))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
