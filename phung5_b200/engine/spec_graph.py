"""CUDA graph of the speculative step: draft tree rounds, tree selection, verification, acceptance and the
KV move, captured once per batch size and replayed every step.

Everything after the draft catch-up has a fixed shape for a batch of R requests (R*K draft rows per round,
R*N verify rows), so the step is launch- and host-bound only by construction: about 1,300 kernels per step
at 80 layers. Replaying a graph removes the host enqueue (tens of ms per step) and the launch gaps between
dependent kernels. What varies per step is uploaded into static device buffers before the replay, in one
pinned host->device copy:

  page table [R, P] (P = pages of the longest context), committed lengths c [R], root tokens [R],
  synthetic accept lengths [R], per-request shared-prefix length [R], and the cascade pass-1 work
  lists of the draft rounds and of verification, padded with empty tiles (tile item -1: the kernel's
  CTAs for those tiles exit before any barrier).

Per-forward attention metadata is computed on the device inside the graph from c: draft round d has
prefix c+1 and kv_hi = c+1+d*K, verification prefix c and kv_hi = c+N; the main-pass work list is one
item per request with a fixed number of tiles. The catch-up forward (variable length: 1 + accepted tokens
per request) runs eagerly and hands its root logits and features to the graph through static buffers.

Used for greedy, synthetic (geometric) and seeded-sampling acceptance on dense models, at TP1 and on the
fused tensor-parallel communicator (the sampled graph needs every request on the device accept path: greedy or
1 <= top_k <= 64; its per-request temperature, top_k, top_p and seed are static buffers filled per step). MoE
layers are captured too (routing, expert sort and segment offsets are device-side and sync-free); hybrid GDN
models and the NCCL communicator run the same `_spec_core` eagerly.
"""
from __future__ import annotations

import math
from typing import List, Optional

import numpy as np
import torch

from .. import ops
from .attn_meta import AttnMeta, tiles_for


class _StaticMeta:
    def __init__(self, eng, R: int, P: int, buf: dict):
        self.eng, self.R, self.P = eng, R, P
        self.b = buf
        dev = eng.device
        g = eng.target.hq // eng.target.hkv
        rows = ops.attn_rows()
        self.g, self.rows = g, rows
        ar = torch.arange(R, device=dev, dtype=torch.int32)
        self.ar = ar
        self.indptr = torch.arange(R + 1, device=dev, dtype=torch.int32) * P
        self.qs = {n: torch.arange(R + 1, device=dev, dtype=torch.int32) * n for n in (eng.K, eng.N)}
        self.tiles2 = {}
        for n in (eng.K, eng.N):
            tpr = math.ceil(n * g / rows)
            ti = ar.repeat_interleave(tpr)
            tr = (torch.arange(tpr, device=dev, dtype=torch.int32) * rows).repeat(R)
            self.tiles2[n] = (ti, tr, R * tpr)

    def _meta(self, n: int, prefix: torch.Tensor, kv_hi: torch.Tensor, bits: torch.Tensor):
        b = self.b
        meta = AttnMeta(pages=b["pages32"], page_indptr=self.indptr, prefix_len=prefix, kv_len=kv_hi,
                        q_start=self.qs[n], tree=bits, causal=False)
        q0 = self.ar * n
        items2 = torch.stack([q0, torch.full_like(q0, n), self.ar, b["shared"], kv_hi, self.ar], 1).contiguous()
        w2 = (items2, self.tiles2[n])
        w1 = None
        if self.eng.use_cascade:
            w1 = (b[f"items1_{n}"], (b[f"ti1_{n}"], b[f"tr1_{n}"], b[f"ti1_{n}"].numel()))
        return meta, w1, w2

    def draft(self, d: int, bits: torch.Tensor):
        K = self.eng.K
        prefix = self.b["c32"] + 1
        return self._meta(K, prefix, prefix + d * K, bits)

    def verify(self, tbits: torch.Tensor):
        N = self.eng.N
        c32 = self.b["c32"]
        return self._meta(N, c32, c32 + N, tbits)


class SpecGraph:
    def __init__(self, eng, R: int, mode: str = "greedy", kc: int = 0):
        self.eng, self.R = eng, R
        self.mode, self.kc = mode, kc
        dev = eng.device
        ps = eng.ps
        self.P = math.ceil((eng.max_context + 2 * ps) / ps) + 1
        g = eng.target.hq // eng.target.hkv
        rows = ops.attn_rows()
        self.G = max(1, R // 2)                                       # groups have >= 2 requests
        self.T1 = {n: math.ceil(R * n * g / rows) + self.G + 1 for n in (eng.K, eng.N)}
        # packed int32 inputs: pt | c | roots | ngeo | shared | (items1, ti1, tr1) for K then N
        sizes = [("pt", R * self.P), ("c", R), ("roots", R), ("ngeo", R), ("shared", R),
                 ("temp", R), ("topk", R), ("topp", R), ("seed", R)]      # temp / topp hold fp32 bits
        for n in (eng.K, eng.N):
            sizes += [(f"items1_{n}", 6 * self.G), (f"ti1_{n}", self.T1[n]), (f"tr1_{n}", self.T1[n])]
        self.layout, off = {}, 0
        for name, n in sizes:
            self.layout[name] = (off, n)
            off += n
        self.host = torch.empty(off, dtype=torch.int32, pin_memory=True)
        self.hnp = self.host.numpy()
        self.dbuf = torch.zeros(off, dtype=torch.int32, device=dev)
        vloc = eng.tw.lm_head.shape[0]
        self.logits = torch.zeros(R, vloc, dtype=torch.bfloat16, device=dev)
        self.feat = torch.zeros(R, eng.cfg.model.hidden, dtype=torch.bfloat16, device=dev) if eng.eagle else None
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.out: Optional[torch.Tensor] = None
        self.launches_per_replay = 0
        self.replays = 0

    def _view(self, name, shape=None):
        o, n = self.layout[name]
        v = self.dbuf[o:o + n]
        return v.view(*shape) if shape is not None else v

    def _fill(self, reqs, tables, groups, c_h: List[int], ngeo_h) -> None:
        R, P, K, N = self.R, self.P, self.eng.K, self.eng.N
        h = self.hnp
        o, n = self.layout["pt"]
        pt = h[o:o + n].reshape(R, P)
        pt[:] = 0
        pad = tables.padded
        w = min(P, pad.shape[1])
        pt[:, :w] = np.where(pad[:, :w] < 0, 0, pad[:, :w])
        for name, vals in (("c", c_h), ("roots", [r.root for r in reqs]),
                           ("ngeo", ngeo_h.tolist() if ngeo_h is not None else [0] * R)):
            o, n = self.layout[name]
            h[o:o + n] = vals
        if self.mode == "sample":
            for name, vals, dt in (("temp", [r.params.temperature for r in reqs], np.float32),
                                   ("topk", [r.params.top_k for r in reqs], np.int32),
                                   ("topp", [r.params.top_p for r in reqs], np.float32),
                                   ("seed", [r.params.seed & 0xFFFFFFFF for r in reqs], np.uint32)):
                o, n = self.layout[name]
                h[o:o + n] = np.asarray(vals, dtype=dt).view(np.int32)
        shared = [0] * R
        for a, b, L in (groups or []):
            for r in range(a, b + 1):
                shared[r] = L
        o, n = self.layout["shared"]
        h[o:o + n] = shared
        for qn in (K, N):
            items = [[a * qn, (b - a + 1) * qn, a, 0, L, -1] for a, b, L in (groups or [])][: self.G]
            ti, tr = tiles_for(items, self.eng.target.hq // self.eng.target.hkv)
            T1 = self.T1[qn]
            if len(ti) > T1:
                raise RuntimeError(f"cascade pass-1 tiles {len(ti)} exceed the graph's {T1}")
            oi, ni = self.layout[f"items1_{qn}"]
            flat = [x for it in items for x in it]
            h[oi:oi + ni] = 0
            h[oi:oi + len(flat)] = flat
            ot, nt = self.layout[f"ti1_{qn}"]
            h[ot:ot + nt] = -1
            h[ot:ot + len(ti)] = ti
            orr, nr = self.layout[f"tr1_{qn}"]
            h[orr:orr + nr] = 0
            h[orr:orr + len(tr)] = tr

    def _bufs(self) -> dict:
        R, P = self.R, self.P
        b = {"pages32": self._view("pt"), "c32": self._view("c"), "shared": self._view("shared")}
        for n in (self.eng.K, self.eng.N):
            b[f"items1_{n}"] = self._view(f"items1_{n}", (self.G, 6))
            b[f"ti1_{n}"] = self._view(f"ti1_{n}")
            b[f"tr1_{n}"] = self._view(f"tr1_{n}")
        return b

    def _body(self) -> torch.Tensor:
        eng, R, P = self.eng, self.R, self.P
        mp = _StaticMeta(eng, R, P, self._bufs())
        pt = self._view("pt", (R, P)).long()
        c = self._view("c").long()
        roots = self._view("roots").long()
        mode = self.mode
        ngeo = self._view("ngeo").long() if mode == "geometric" else None
        sp = None
        if mode == "sample":
            sp = (self._view("temp").view(torch.float32), self._view("topk"), self._view("topp").view(torch.float32),
                  self._view("seed").long() & 0xFFFFFFFF, self.kc)
        return eng._spec_core(mp, pt, c, roots, self.logits, self.feat, mode, ngeo, sp=sp)

    def _capture(self) -> None:
        eng = self.eng
        st = torch.cuda.Stream(device=eng.device)
        st.wait_stream(torch.cuda.current_stream(eng.device))
        with torch.cuda.stream(st):
            self._body()                                   # warm-up: lazy workspaces, same work as a replay
        torch.cuda.current_stream(eng.device).wait_stream(st)
        g = torch.cuda.CUDAGraph()
        pool = getattr(eng, "_graph_pool", None)
        if pool is None:
            pool = torch.cuda.graph_pool_handle()
            eng._graph_pool = pool
        n0 = ops.launches()
        with torch.cuda.graph(g, pool=pool, stream=st):
            self.out = self._body()
        self.launches_per_replay = ops.launches() - n0
        self.graph = g

    def run(self, reqs, tables, groups, c_h, logits: torch.Tensor, root_feat, ngeo_h) -> torch.Tensor:
        self._fill(reqs, tables, groups, c_h, ngeo_h)
        self.dbuf.copy_(self.host, non_blocking=True)
        self.logits.copy_(logits)
        if self.feat is not None:
            self.feat.copy_(root_feat)
        if self.graph is None:
            self._capture()
        self.graph.replay()
        ops._LAUNCHES[0] += self.launches_per_replay     # kernels launched by the replay
        self.replays += 1
        return self.out
