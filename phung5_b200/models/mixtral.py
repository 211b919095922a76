"""Mixtral-style sparse MoE block (the Mixtral-8x7B EP8 workload) on the grouped tcgen05 GEMMs.

Routing: router logits = x @ W_gate^T (replicated [E, H]); each token takes its top-k experts, weights =
softmax over the selected logits (Mixtral's rule, also the oracle's in models/reference.py).

Expert parallelism: rank r of `ep` ranks owns experts [r*E/ep, (r+1)*E/ep) with full FFN width. Every
rank holds every token (attention is tensor-parallel and its output is all-reduced), so dispatch is a
local selection: the (token, slot) assignments of local experts are sorted by expert on the device
(stable argsort, counts -> offsets, no host round trip); the fp8 rows and scales are gathered once into
expert order, gate/up and down run as grouped GEMMs over the per-expert row segments, and one fused kernel
(ops.moe_combine) sums weight * expert output per token into the buffer the tensor-parallel reduction
reads. The grouped GEMM can also gather rows inside its A loads (rows=, TMA gather4), but at 32 gather
operations per pipeline stage, repeated for every N tile, that measured 2.3x slower than one gather copy. Each rank's output holds only its experts'
contributions; the layer's all-reduce (the same collective as tensor-parallel MLPs) completes it.
Rows beyond the local assignment count are never written by the grouped GEMMs; the combine selects
(not multiplies) them away, so uninitialised rows cannot leak NaN.

`forward_a2a` is the all-to-all alternative (ParallelConfig.moe_dispatch = "a2a", NCCL / gloo collectives):
each rank routes only its own share of the tokens and sends every (token, expert) row to the expert's rank
and back, moving the routed rows instead of every token's full output.

The reference serves no MoE model; this follows the Mixtral-8x7B EP8 workload.
"""
from __future__ import annotations

import zlib
from dataclasses import dataclass
from typing import Dict, Optional

import torch
import torch.distributed as dist

from .. import ops
from ..config import ModelConfig
from ..weights.quant import ensure_pow2, quant_weight_block


@dataclass
class MoEBlock:
    gate: torch.Tensor          # [E, H] router weight (bf16 / fp32), replicated
    w13: torch.Tensor           # [E_local * 2F, H]: per expert gate rows then up rows
    w13_s: Optional[torch.Tensor]
    w2: torch.Tensor            # [E_local * H, F]
    w2_s: Optional[torch.Tensor]
    num_experts: int
    top_k: int
    e_lo: int
    e_local: int
    ffn: int
    hidden: int

    @property
    def fp8(self) -> bool:
        return self.w13_s is not None

    def route(self, xb: torch.Tensor):
        """-> (expert ids [T, k] int64, weights [T, k] fp32)."""
        if xb.is_cuda and xb.dtype == torch.bfloat16 and self.gate.dtype == torch.bfloat16:
            logits = ops.gemm_bf16(xb, self.gate)
        else:
            logits = xb.float() @ self.gate.float().t()
        v, i = torch.topk(logits.float(), self.top_k, dim=-1)
        return i, torch.softmax(v, dim=-1)

    def __call__(self, x_act, xb: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """-> this rank's experts' contribution per token, bf16 [T, H] (written into `out` when given, e.g.
        the fused tensor-parallel reduction's partial buffer)."""
        t = xb.shape[0]
        k, el = self.top_k, self.e_local
        ids, w = self.route(xb)
        flat = ids.reshape(-1) - self.e_lo                         # local expert of each assignment
        local = (flat >= 0) & (flat < el)
        key = torch.where(local, flat, torch.full_like(flat, el))  # non-local assignments sort last
        order = torch.argsort(key, stable=True)                    # permuted position -> assignment
        # counts by scatter-add (torch.bincount reads the maximum back to the host): no synchronisation, so
        # the MoE step can be captured in a CUDA graph
        counts = torch.zeros(el + 1, dtype=torch.int64, device=xb.device).scatter_add_(
            0, key, torch.ones_like(key))[:el]
        offsets = torch.zeros(el + 1, dtype=torch.int32, device=xb.device)
        offsets[1:] = torch.cumsum(counts, 0).to(torch.int32)
        tok = order // k                                          # token of each permuted row
        if self.fp8:
            # dispatch: one gather of the tokens' fp8 rows and scales into expert order (8 MB at 2048 rows x
            # 4096); gathering inside the GEMM's A loads (rows=, TMA gather4) measured 2.3x slower
            xq, xs = x_act
            gu = ops.gemm_grouped((xq[tok], xs[:, tok].contiguous()), self.w13, self.w13_s, offsets, 2 * self.ffn)
        else:
            gu = ops.gemm_grouped(x_act[tok], self.w13, self.w13_s, offsets, 2 * self.ffn)
        aq, as_, ab = ops.silu_mul_quant(gu, quant=self.fp8, out_bf16=not self.fp8)
        y = ops.gemm_grouped((aq, as_) if self.fp8 else ab, self.w2, self.w2_s, offsets, self.hidden)
        # combine: position of every assignment in the permuted order
        pos = torch.empty_like(order)
        pos[order] = torch.arange(order.numel(), device=xb.device)
        pos = pos.view(t, k)
        valid = local.view(t, k)
        if y.is_cuda:
            if out is None:
                out = torch.empty(t, self.hidden, dtype=torch.bfloat16, device=xb.device)
            ops.moe_combine(y, pos, w.float().contiguous(), valid.contiguous(), out)   # one fused kernel
            return out
        g = y[pos.clamp(min=0)]                                    # [T, k, H]
        contrib = torch.where(valid[..., None], g.float() * w[..., None], torch.zeros((), device=xb.device))
        res = contrib.sum(1).to(xb.dtype)
        if out is not None:
            out.copy_(res)
            return out
        return res


    def _expert_rows(self, xb_rows: torch.Tensor, lexp: torch.Tensor) -> torch.Tensor:
        """This rank's experts over rows that all belong to them: row i goes through local expert lexp[i];
        -> [n, H] in the input row order (fp8 experts quantize the bf16 rows here)."""
        el = self.e_local
        n = xb_rows.shape[0]
        order = torch.argsort(lexp, stable=True)
        counts = torch.zeros(el, dtype=torch.int64, device=xb_rows.device).scatter_add_(0, lexp, torch.ones_like(lexp))
        offsets = torch.zeros(el + 1, dtype=torch.int32, device=xb_rows.device)
        offsets[1:] = torch.cumsum(counts, 0).to(torch.int32)
        xs_rows = xb_rows[order]
        act = ops.act_quant(xs_rows) if self.fp8 else xs_rows
        gu = ops.gemm_grouped(act, self.w13, self.w13_s, offsets, 2 * self.ffn)
        aq, as_, ab = ops.silu_mul_quant(gu, quant=self.fp8, out_bf16=not self.fp8)
        y = ops.gemm_grouped((aq, as_) if self.fp8 else ab, self.w2, self.w2_s, offsets, self.hidden)
        out = torch.empty(n, self.hidden, dtype=y.dtype, device=y.device)
        out[order] = y[:n]
        return out

    def forward_a2a(self, xb_rows: torch.Tensor, comm) -> torch.Tensor:
        """Expert parallelism by all-to-all: this rank's own token rows [T_own, H] are routed here, every
        (token, expert) assignment is sent to the rank that owns the expert (one variable-size all-to-all of the
        rows and one of their local expert ids), the receiving rank runs its experts over what it received, the
        outputs return by the reverse all-to-all, and the owner sums them weighted per token. -> [T_own, H].
        Counts are exchanged on the host (a synchronisation: this path is not captured in a graph). Bytes per rank
        are the routed rows only, against every token's full output in the reduction path."""
        W, el, k = comm.size, self.e_local, self.top_k
        t = xb_rows.shape[0]
        dev = xb_rows.device
        ids, w = self.route(xb_rows)                               # [T_own, k]
        flat = ids.reshape(-1)
        dest = flat // el                                          # owning rank of each assignment
        order = torch.argsort(dest, stable=True)                   # assignments grouped by destination rank
        send = torch.zeros(W, dtype=torch.int64, device=dev).scatter_add_(0, dest, torch.ones_like(dest))
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=comm.group)
        send_l, recv_l = send.tolist(), recv.tolist()
        rows = xb_rows[order // k].contiguous()
        lexp = (flat[order] - dest[order] * el).contiguous()
        n_recv = sum(recv_l)
        rows_in = torch.empty(n_recv, self.hidden, dtype=rows.dtype, device=dev)
        lexp_in = torch.empty(n_recv, dtype=lexp.dtype, device=dev)
        dist.all_to_all_single(rows_in, rows, recv_l, send_l, group=comm.group)
        dist.all_to_all_single(lexp_in, lexp, recv_l, send_l, group=comm.group)
        y = self._expert_rows(rows_in, lexp_in) if n_recv else rows_in.new_zeros(0, self.hidden)
        y = y.to(rows.dtype).contiguous()
        back = torch.empty(flat.numel(), self.hidden, dtype=y.dtype, device=dev)
        dist.all_to_all_single(back, y, send_l, recv_l, group=comm.group)
        per = torch.empty_like(back)
        per[order] = back                                          # assignment order again
        return (per.view(t, k, self.hidden).float() * w[..., None]).sum(1).to(xb_rows.dtype)


def _expert_range(cfg: ModelConfig, rank: int, size: int):
    if cfg.num_experts % size:
        raise ValueError(f"{cfg.num_experts} experts do not split over {size} expert-parallel ranks")
    el = cfg.num_experts // size
    return rank * el, el


def pack_moe(cfg: ModelConfig, wd: Dict[str, torch.Tensor], prefix: str, device, rank: int = 0, size: int = 1,
             dtype: torch.dtype = torch.bfloat16) -> MoEBlock:
    """HF Mixtral names: block_sparse_moe.gate.weight, block_sparse_moe.experts.{e}.w1/w3/w2.weight (+ _scale_inv)."""
    fp8 = cfg.quant == "fp8_block"
    e_lo, el = _expert_range(cfg, rank, size)
    p = prefix + "block_sparse_moe."
    w13, s13, w2, s2 = [], [], [], []

    def get(name, want_fp8):
        w, s = wd[name], wd.get(name + "_scale_inv")
        if want_fp8:
            if s is None:
                return quant_weight_block(w.to(device).float())
            return ensure_pow2(w.to(device), s.to(device))
        if s is not None:
            from .reference import dequant_block_fp8
            w = dequant_block_fp8(w, s)
        return w.to(device, dtype), None

    for e in range(e_lo, e_lo + el):
        ep = p + f"experts.{e}."
        for nm in ("w1", "w3"):
            w, s = get(ep + nm + ".weight", fp8)
            w13.append(w)
            s13.append(s)
        w, s = get(ep + "w2.weight", fp8)
        w2.append(w)
        s2.append(s)
    return MoEBlock(gate=wd[p + "gate.weight"].to(device, dtype), w13=torch.cat(w13).contiguous(),
                    w13_s=torch.cat(s13).contiguous() if fp8 else None, w2=torch.cat(w2).contiguous(),
                    w2_s=torch.cat(s2).contiguous() if fp8 else None, num_experts=cfg.num_experts,
                    top_k=cfg.experts_per_token, e_lo=e_lo, e_local=el, ffn=cfg.ffn, hidden=cfg.hidden)


def random_moe(cfg: ModelConfig, device, seed: int, layer: int, rank: int = 0, size: int = 1,
               std: float = 0.02) -> MoEBlock:
    fp8 = cfg.quant == "fp8_block"
    e_lo, el = _expert_range(cfg, rank, size)
    gen = torch.Generator(device=device)

    def rnd(n, k, tag):
        gen.manual_seed(zlib.crc32(repr((seed, layer, tag)).encode()) & 0x7FFFFFFF)
        w = torch.randn(n, k, device=device, generator=gen, dtype=torch.bfloat16) * std
        if fp8:
            return quant_weight_block(w.float())
        return w, None

    w13, s13, w2, s2 = [], [], [], []
    for e in range(e_lo, e_lo + el):
        for nm in ("w1", "w3"):
            w, s = rnd(cfg.ffn, cfg.hidden, (e, nm))
            w13.append(w)
            s13.append(s)
        w, s = rnd(cfg.hidden, cfg.ffn, (e, "w2"))
        w2.append(w)
        s2.append(s)
    gen.manual_seed(zlib.crc32(repr((seed, layer, "gate")).encode()) & 0x7FFFFFFF)
    gate = torch.randn(cfg.num_experts, cfg.hidden, device=device, generator=gen, dtype=torch.bfloat16) * std
    return MoEBlock(gate=gate, w13=torch.cat(w13).contiguous(),
                    w13_s=torch.cat(s13).contiguous() if fp8 else None, w2=torch.cat(w2).contiguous(),
                    w2_s=torch.cat(s2).contiguous() if fp8 else None, num_experts=cfg.num_experts,
                    top_k=cfg.experts_per_token, e_lo=e_lo, e_local=el, ffn=cfg.ffn, hidden=cfg.hidden)
