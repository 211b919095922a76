"""Tensor-parallel communicators.

`NcclCommunicator` is the baseline: torch.distributed collectives (NCCL on GPU, gloo on CPU) issued
between separate kernels. The fused path (`parallel/fused.py`) replaces the reductions after o_proj
and down_proj with kernels that move the rows themselves over NVLink: peer loads and stores of the
symmetric workspace, or NVLS multimem reductions and broadcasts where the GPUs support multicast.

Vocab-sharded helpers keep the exchange tiny: each rank sends its local top-k (value, global index)
and its local log-sum-exp; the global log-softmax top-k follows exactly from those (the largest k
values overall are among the union of every shard's top k).

The reference has no TP path (every engine runs tensor_parallel_size 1, configuration.yaml:39-116);
its multi-GPU scaling is replica DP behind a proxy (docker/opt/sgl/lb_proxy.py).
"""
from __future__ import annotations

import datetime
import os
from typing import Optional, Tuple

import torch
import torch.distributed as dist

from ..models.llama import Communicator


def init_distributed(backend: Optional[str] = None, timeout_s: float = 120.0) -> Tuple[int, int, int]:
    """Initialise the default process group from torchrun's environment. Returns (rank, world, local_rank)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)
    return rank, world, local


class NcclCommunicator(Communicator):
    def __init__(self, group=None):
        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.size > 1:
            dist.all_reduce(x, group=self.group)
        return x

    def _gather(self, x: torch.Tensor) -> torch.Tensor:
        """[...] -> [world, ...] (gathered as one flat concatenation, the form every backend accepts)."""
        x = x.contiguous()
        flat = torch.empty((self.size * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(flat, x, group=self.group)
        return flat.view((self.size,) + tuple(x.shape))

    def gather(self, parts):
        """All-gather of several tensors: -> [[world, *p.shape] for p in parts]."""
        return [self._gather(p) for p in parts]

    def all_gather_vocab(self, x: torch.Tensor) -> torch.Tensor:
        g = self._gather(x)                       # [tp, rows, V/tp]
        return g.permute(1, 0, 2).reshape(x.shape[0], -1)

    def topk_logprobs_merge(self, v: torch.Tensor, i: torch.Tensor, lse: torch.Tensor, k: int):
        gv, gi, gl = self._gather(v), self._gather(i), self._gather(lse)     # [tp, rows, k] / [tp, rows, 1]
        tot = torch.logsumexp(gl, 0)                                          # [rows, 1]
        vv = gv.permute(1, 0, 2).reshape(v.shape[0], -1)
        ii = gi.permute(1, 0, 2).reshape(v.shape[0], -1)
        tv, ti = torch.topk(vv, k, dim=-1)
        return tv - tot, ii.gather(1, ti)

    def argmax_merge(self, v: torch.Tensor, i: torch.Tensor) -> torch.Tensor:
        gv, gi = self._gather(v), self._gather(i)                             # [tp, rows]
        best = gv.argmax(0)
        return gi.gather(0, best[None])[0]

    def barrier(self):
        if self.size > 1:
            dist.barrier(group=self.group)

    def max_float(self, x: float) -> float:
        if self.size == 1:
            return x
        dev = "cuda" if torch.cuda.is_available() and dist.get_backend(self.group) == "nccl" else "cpu"
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return float(t.item())
