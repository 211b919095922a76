"""Fused tensor-parallel communicator: in-kernel NVLink reductions instead of NCCL collectives.

Every rank allocates one symmetric workspace (torch.distributed._symmetric_memory: cuMem allocations
mapped into every peer, exchanged at rendezvous) holding, for up to `max_tokens` rows:
    partial [M, H] bf16   output of the row-parallel projection (o_proj / down_proj) of this rank
    h       [M, H] bf16   residual stream (identical on every rank)
    y       [M, H] bf16   normalized rows (final norm / bf16 models)
    q       [M, H] e4m3   normalized rows, block-scaled fp8 (input of the next GEMM)
    s       [H/128, Mmax] fp32 scales of q
    flags   [2, W] u32    barrier flags (epochs)
    counter [4] u32       CTA counter of the end barrier, device epoch
    gsrc    [G] bytes     staging block of `gather` (this rank's candidates)
    gdst    [W, G] bytes  every rank's staging block after `gather`
    recv    [W, ceil(M/W), H] bf16  row-parallel projection outputs pushed by each rank for the rows this
                          rank owns (`project`: the GEMM's epilogue stores them over NVLink)
`ar_norm(M, w)` runs csrc/tp_fused.cu: reduce-scatter of the partials with P2P loads, + residual,
RMSNorm, fp8 quant, all-gather of the results with P2P stores, in one kernel. Where the GPUs support
NVLink multicast (NVLS), the reduce-scatter is one multimem.ld_reduce per 16 bytes through the workspace's
multicast address and the all-gather one multimem.st (each rank sends its rows once; the switch copies
them to every rank; used from 8 ranks up, PHX_NVLS=1 / 0 forces it on / off). The engine's model uses
it when the communicator reports `fused = True` (models/llama.py, forward_fused; the EAGLE head's layer
too); anything larger than the workspace keeps the NCCL path of the base class. `gather` exchanges small
blocks (vocab-sharded top-k and argmax candidates) with P2P stores. Barrier epochs are kept on the device,
so every kernel here can be captured in a CUDA graph; no NCCL call remains on the decode path.

`FusedEmulator` gives the same interface on CPU ranks (gloo all-reduce + the op definitions) so the
fused forward's plumbing is tested without GPUs.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from .. import ops
from .comm import NcclCommunicator


GATHER_BYTES = 4 << 20   # verify-row sampling candidates: 4096 rows x 64 x (value, index) = 2 MB


class _Workspace:
    def __init__(self, max_tokens: int, hidden: int, device, world: int, alloc):
        self.mmax, self.h = max_tokens, hidden
        mh = max_tokens * hidden
        off, o = {}, 0
        for name, nbytes in (("partial", 2 * mh), ("h", 2 * mh), ("y", 2 * mh), ("q", mh),
                             ("s", 4 * (hidden // 128) * max_tokens), ("flags", 4 * 2 * world), ("counter", 16),
                             ("gsrc", GATHER_BYTES), ("gdst", GATHER_BYTES * world),
                             ("recv", 2 * hidden * world * ((max_tokens + world - 1) // world))):
            off[name] = o
            o += (nbytes + 255) // 256 * 256
        self.off = off
        self.buf = alloc(o)

    def view(self, name, dtype, shape):
        n = 1
        for d in shape:
            n *= d
        esz = torch.tensor([], dtype=dtype).element_size()
        return self.buf[self.off[name]: self.off[name] + n * esz].view(dtype).view(*shape)


class FusedCommunicator(NcclCommunicator):
    fused = True

    def __init__(self, max_tokens: int = 8192, hidden: int = 8192, group=None):
        super().__init__(group)
        import torch.distributed._symmetric_memory as symm
        dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.ws = _Workspace(max_tokens, hidden, dev, self.size,
                             lambda n: symm.empty(n, dtype=torch.uint8, device=dev))
        grp = self.group or dist.group.WORLD
        self.handle = symm.rendezvous(self.ws.buf, grp.group_name)
        self.peer_base = torch.tensor(list(self.handle.buffer_ptrs), dtype=torch.int64, device=dev)
        # NVLS: the workspace's multicast address (every rank's copy behind one NVSwitch address) when the GPUs
        # and driver support it. Measured on B200 (Llama-3-70B verify rows, M = 4096 x 8192): at 8 ranks the
        # multicast all-gather cuts the reduction's row work from 66 to 15 us; at 2 ranks the peer path is
        # faster (pull mode 0.12 vs 0.19 ms), so by default multicast is used from 8 ranks up. PHX_NVLS=1
        # forces it on (where available), PHX_NVLS=0 off.
        mc = 0
        nv = os.environ.get("PHX_NVLS", "auto")
        if nv == "1" or (nv != "0" and self.size >= 8):
            try:
                mc = int(self.handle.multicast_ptr or 0)
            except (RuntimeError, AttributeError):
                mc = 0
        self.mc = mc
        self.ws.view("flags", torch.int32, (2 * self.size,)).zero_()
        self.ws.view("counter", torch.int32, (4,)).zero_()
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)
        self.max_tokens = max_tokens
        self.hidden = hidden
        # PHX_TP_PHASES=1: the fused reduction sums, per launch, its start-barrier wait and row work over CTAs
        # and its end barrier (device ns; phase_report())
        self.phase = (torch.zeros(4, dtype=torch.int64, device=dev)
                      if os.environ.get("PHX_TP_PHASES") == "1" else None)

    def reset(self) -> None:
        """Collective recovery after a kernel reported a peer timeout (status 4): every rank calls it between
        steps; the barrier flags, CTA counter and device epoch go back to zero on every rank, between two
        host barriers, so the next fused launch starts in step again."""
        dist.barrier(group=self.group)
        torch.cuda.synchronize(self.device)
        self.ws.view("flags", torch.int32, (2 * self.size,)).zero_()
        self.ws.view("counter", torch.int32, (4,)).zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def close(self) -> None:
        """Collective teardown: every rank calls it (between steps, nothing in flight) before the process group is
        destroyed. The symmetric workspace, its peer mappings and its multicast object are released together,
        between two barriers, so no rank unmaps memory a peer is still bound to."""
        dist.barrier(group=self.group)
        torch.cuda.synchronize(self.device)
        self.handle = None
        self.ws = None
        self.peer_base = None
        import gc
        gc.collect()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def partial(self, m: int) -> torch.Tensor:
        return self.ws.view("partial", torch.bfloat16, (m, self.hidden))

    def h(self, m: int) -> torch.Tensor:
        return self.ws.view("h", torch.bfloat16, (m, self.hidden))

    def project(self, lin, x, m: int) -> None:
        """Row-parallel projection (o_proj / down_proj) whose output rows are stored straight into their owner's
        receive slot by the GEMM epilogue (a reduce-scatter's transfer, overlapped with the GEMM); follow with
        `ar_norm(..., recv=True)`."""
        rows_per = (m + self.size - 1) // self.size
        xq, xs = x if lin.fp8 else (x, None)
        bn, hws, pair, _ = ops._table_choice("fp8" if lin.fp8 else "bf16", lin.w.shape[0], xq.shape[1], m, 0, None,
                                             None, True)
        ops.ext().gemm_scatter(xq, xs, lin.w, lin.ws, self.peer_base, self.ws.off["recv"], rows_per, self.rank,
                               ops.status_tensor(self.device), ops.FP8_HW_SCALE if hws is None else hws,
                               ops.GEMM_PAIR if pair is None else pair, bn, ops.SCATTER_BULK)

    def ar_norm(self, m: int, w: torch.Tensor, eps: float, out_bf16: bool = False, push_h: bool = False,
                recv: bool = False):
        """h += sum over ranks of the projection partials (pulled from every rank's `partial`, or, with recv,
        read from the receive slots `project` filled) for the rows this rank owns (every row on every rank with
        push_h); returns the normalized rows on every rank: (q, s) fp8 or y bf16."""
        off = [self.ws.off[k] for k in ("partial", "h", "y", "q", "s", "flags", "counter")]
        ops.ext().tp_ar_norm(self.peer_base, self.rank, self.size, m, self.hidden, eps, w, out_bf16, push_h,
                             ops.status_tensor(self.device), off, m, self.ws.off["recv"] if recv else -1, self.mc,
                             self.phase)
        if out_bf16:
            return self.ws.view("y", torch.bfloat16, (m, self.hidden))
        q = self.ws.view("q", torch.float8_e4m3fn, (m, self.hidden))
        s = self.ws.view("s", torch.float32, (self.hidden // 128, m))
        return q, s


    def phase_report(self, launches: int) -> dict:
        """Mean device microseconds per fused-reduction launch (PHX_TP_PHASES=1): a CTA's wait at the start
        barrier (the peers' arrival skew), its row work, and the end barrier; then the counters restart."""
        if self.phase is None or launches <= 0:
            return {}
        p = self.phase.tolist()
        ctas = max(1, p[3])
        out = {"start_wait_us": round(p[0] / ctas / 1e3, 2), "row_work_us": round(p[1] / ctas / 1e3, 2),
               "end_barrier_us": round(p[2] / launches / 1e3, 2), "ctas_per_launch": round(ctas / launches, 1)}
        self.phase.zero_()
        return out

    def gather(self, parts):
        """All-gather of small tensors (one exchange for all parts): -> [[world, *p.shape] for p in parts]."""
        offs, o = [], 0
        for p in parts:
            offs.append(o)
            o += (p.numel() * p.element_size() + 15) // 16 * 16
        if o > GATHER_BYTES:
            return [super(FusedCommunicator, self)._gather(p) for p in parts]
        src = self.ws.buf[self.ws.off["gsrc"]:]
        for p, a in zip(parts, offs):
            nb = p.numel() * p.element_size()
            src[a:a + nb].copy_(p.contiguous().view(-1).view(torch.uint8))
        off = [self.ws.off[k] for k in ("gsrc", "gdst", "flags", "counter")]
        ops.ext().tp_allgather(self.peer_base, self.rank, self.size, o, ops.status_tensor(self.device), off, self.mc)
        dst = self.ws.buf[self.ws.off["gdst"]: self.ws.off["gdst"] + self.size * o].view(self.size, o)
        out = []
        for p, a in zip(parts, offs):
            nb = p.numel() * p.element_size()
            out.append(dst[:, a:a + nb].contiguous().view(p.dtype).view((self.size,) + tuple(p.shape)))
        return out

    def _gather(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            return super()._gather(x)
        return self.gather([x])[0]

    def topk_logprobs_merge(self, v: torch.Tensor, i: torch.Tensor, lse: torch.Tensor, k: int):
        gv, gi, gl = self.gather([v.float(), i, lse.float()])
        tot = torch.logsumexp(gl, 0)
        vv = gv.permute(1, 0, 2).reshape(v.shape[0], -1)
        ii = gi.permute(1, 0, 2).reshape(v.shape[0], -1)
        tv, ti = torch.topk(vv, k, dim=-1)
        return tv - tot, ii.gather(1, ti)

    def argmax_merge(self, v: torch.Tensor, i: torch.Tensor) -> torch.Tensor:
        gv, gi = self.gather([v.float(), i])
        best = gv.argmax(0)
        return gi.gather(0, best[None])[0]


class FusedEmulator(NcclCommunicator):
    """CPU stand-in with FusedCommunicator's interface: all-reduce + the op definitions."""

    fused = True

    def __init__(self, max_tokens: int = 8192, hidden: int = 256, group=None, dtype=torch.float32):
        super().__init__(group)
        self.max_tokens, self.hidden = max_tokens, hidden
        self._partial = torch.zeros(max_tokens, hidden, dtype=dtype)
        self._h = torch.zeros(max_tokens, hidden, dtype=dtype)

    def partial(self, m):
        return self._partial[:m]

    def h(self, m):
        return self._h[:m]

    def project(self, lin, x, m):
        self._partial[:m].copy_(lin(x))

    def ar_norm(self, m, w, eps, out_bf16=False, push_h=False, recv=False):
        p = self._partial[:m].clone()
        self.all_reduce(p)
        q, s, y = ops.add_rmsnorm_quant(self._h[:m], p, w, eps, quant=not out_bf16, out_bf16=out_bf16)
        return y if out_bf16 else (q, s)
