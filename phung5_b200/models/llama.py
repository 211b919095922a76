"""Engine model for Llama-family decoders (dense SwiGLU; Mixtral MoE in models/mixtral.py).

Weights are packed for the kernels: q/k/v fused into one column-parallel projection, gate/up fused
into one [2F, H] projection (gate rows, then up rows), o/down row-parallel. Under tensor parallelism
rank r keeps heads [r*Hq/tp, (r+1)*Hq/tp) (and the matching KV heads) and FFN columns
[r*F/tp, (r+1)*F/tp); o_proj and down_proj produce partial sums that the communicator reduces.

Per layer (fp8_block):
  (xq, xs) = add_rmsnorm_quant(h, delta, w_in)       h <- h + delta (previous MLP output, reduced)
  qkv      = gemm_fp8_block(xq, xs, Wqkv)            tcgen05
  q        = rope_kv_write(qkv, pos, slots)          k/v -> paged cache
  (aq, as) = paged_attention(q, ...)                 fp8 output, one scale per (token, head)
  o        = gemm_fp8_block(aq, as, Wo)  -> reduce
  (xq, xs) = add_rmsnorm_quant(h, o, w_post)
  (aq, as) = gemm_fp8_swiglu(xq, xs, Wgu)            tcgen05, SwiGLU + fp8 quant in the epilogue
  delta    = gemm_fp8_block(aq, as, Wd)  -> reduce
bf16 models run the same sequence with bf16 activations and gemm_bf16.
The reference runs these layers inside SGLang with its FP8 GEMM table and fused SiLU+quant patches
(docker/opt/v5/wq/kopt_wq.py:92-116, docker/opt/v5/fusedq/fusedq.py:289-329).
"""
from __future__ import annotations

import math
import zlib
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch

from .. import ops
from ..utils import nvtx as _nvtx
from ..config import ModelConfig
from ..weights.quant import FP8_DTYPE, ensure_pow2, quant_weight_block


@dataclass
class Linear:
    """A packed linear layer: bf16 weight [N, K], or fp8 e4m3 [N, K] + fp32 block scales [ceil(N/128), K/128]."""

    w: torch.Tensor
    ws: Optional[torch.Tensor] = None
    # gate/up weights whose 128-row blocks were interleaved (gate j, up j) for the fused SwiGLU epilogue; the
    # plain call still returns the [gate | up] layout
    gu_interleaved: bool = False

    @property
    def fp8(self) -> bool:
        return self.ws is not None

    @property
    def out_features(self) -> int:
        return self.w.shape[0]

    def __call__(self, x, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.fp8:
            xq, xs = x
            if self.gu_interleaved:
                y = ops.gemm_fp8_block(xq, xs, self.w, self.ws)
                m, n = y.shape
                y = y.view(m, n // 256, 2, 128).transpose(1, 2).reshape(m, n)
                return out.copy_(y) if out is not None else y
            return ops.gemm_fp8_block(xq, xs, self.w, self.ws, out=out)
        return ops.gemm_bf16(x, self.w, out=out)

    def swiglu(self, x):
        """Gate/up projection followed by SwiGLU: fp8 -> (q [M, F] e4m3, scales [F/128, M]) from one GEMM whose
        epilogue does the SwiGLU and the quant (weights interleaved in place on the first call); bf16 -> the
        bf16 activation [M, F]."""
        if not self.fp8:
            return ops.silu_mul_quant(self(x), quant=False, out_bf16=True)[2]
        xq, xs = x
        f = self.w.shape[0] // 2
        if xq.is_cuda and ops.SWIGLU_FUSED and ops.FP8_HW_SCALE and f % 128 == 0:
            if not self.gu_interleaved:
                self.w, self.ws = interleave_gate_up(self.w, self.ws)
                self.gu_interleaved = True
            return ops.gemm_fp8_swiglu(xq, xs, self.w, self.ws)
        q, s, _ = ops.silu_mul_quant(self(x), quant=True, out_bf16=False)
        return q, s


def interleave_gate_up(w: torch.Tensor, ws: torch.Tensor):
    """[gate; up] rows (2F x K) and their 128-row block scales -> rows in 128-row blocks gate 0, up 0, gate 1,
    up 1, ... (the layout of the fused SwiGLU epilogue: each 256-wide output tile pairs a gate block with its
    up block)."""
    n, k = w.shape
    f = n // 2
    w2 = w.view(2, f // 128, 128, k).transpose(0, 1).reshape(n, k).contiguous()
    s2 = ws.view(2, f // 128, ws.shape[1]).transpose(0, 1).reshape(ws.shape[0], ws.shape[1]).contiguous()
    return w2, s2


@dataclass
class LayerWeights:
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    qkv: Linear
    o: Linear
    gu: Optional[Linear] = None       # dense MLP
    down: Optional[Linear] = None
    moe: Optional[object] = None      # MoE block (models/mixtral.py)


@dataclass
class ModelWeights:
    cfg: ModelConfig
    embed: torch.Tensor               # [V, H] bf16 (full vocab on every rank)
    layers: List[LayerWeights]
    final_norm: torch.Tensor
    lm_head: torch.Tensor             # [V_local, H] bf16 (vocab-sharded under TP)
    vocab_start: int = 0
    tp_rank: int = 0
    tp_size: int = 1

    @property
    def fp8(self) -> bool:
        return self.layers[0].qkv.fp8


def _shard_rows(t: torch.Tensor, rank: int, size: int) -> torch.Tensor:
    n = t.shape[0] // size
    return t[rank * n: (rank + 1) * n]


def _shard_cols(t: torch.Tensor, rank: int, size: int) -> torch.Tensor:
    n = t.shape[1] // size
    return t[:, rank * n: (rank + 1) * n]


def _pack_linear(parts: List[Tuple[torch.Tensor, Optional[torch.Tensor]]], device, fp8: bool,
                 dtype: torch.dtype = torch.bfloat16) -> Linear:
    """Concatenate row blocks of (weight, scale_inv) pairs; requantize when the checkpoint is not fp8 but
    the model runs fp8. Row blocks must be multiples of 128 rows for fp8 scale alignment."""
    ws_list, ss_list = [], []
    for w, s in parts:
        if fp8:
            if s is None:
                q, s = quant_weight_block(w.to(device).float())
                ws_list.append(q)
                ss_list.append(s)
            else:
                q, s = ensure_pow2(w.to(device), s.to(device))
                ws_list.append(q)
                ss_list.append(s)
        else:
            if s is not None:
                from .reference import dequant_block_fp8
                w = dequant_block_fp8(w, s)
            ws_list.append(w.to(device=device, dtype=dtype))
    w = torch.cat(ws_list, 0).contiguous()
    return Linear(w, torch.cat(ss_list, 0).contiguous() if fp8 else None)


def _get(wd: Dict[str, torch.Tensor], name: str):
    return wd[name], wd.get(name + "_scale_inv")


def _row_shard_pair(pair, rank, size):
    w, s = pair
    w = _shard_rows(w, rank, size)
    if s is not None:
        s = _shard_rows(s, rank, size)
    return w, s


def _col_shard_pair(pair, rank, size):
    w, s = pair
    w = _shard_cols(w, rank, size)
    if s is not None:
        s = _shard_cols(s, rank, size)
    return w, s


def pack_weights(cfg: ModelConfig, wd: Dict[str, torch.Tensor], device, tp_rank: int = 0, tp_size: int = 1,
                 prefix: str = "model.", dtype: torch.dtype = torch.bfloat16) -> ModelWeights:
    """HF-named (optionally fp8 block-scaled) weights -> packed, TP-sharded device weights."""
    fp8 = cfg.quant == "fp8_block"
    assert cfg.num_heads % tp_size == 0 and cfg.num_kv_heads % tp_size == 0 and cfg.ffn % tp_size == 0
    layers = []
    if cfg.quant != "fp8_block":
        fp8 = False
    for i in range(cfg.num_layers):
        p = f"{prefix}layers.{i}."
        qkv = _pack_linear([_row_shard_pair(_get(wd, p + f"self_attn.{n}.weight"), tp_rank, tp_size)
                            for n in ("q_proj", "k_proj", "v_proj")], device, fp8, dtype)
        o = _pack_linear([_col_shard_pair(_get(wd, p + "self_attn.o_proj.weight"), tp_rank, tp_size)], device, fp8, dtype)
        lw = LayerWeights(in_norm=wd[p + "input_layernorm.weight"].to(device, dtype),
                          post_norm=wd[p + "post_attention_layernorm.weight"].to(device, dtype),
                          qkv=qkv, o=o)
        if cfg.is_moe:
            from .mixtral import pack_moe
            lw.moe = pack_moe(cfg, wd, p, device, tp_rank, tp_size, dtype)
        else:
            lw.gu = _pack_linear([_row_shard_pair(_get(wd, p + f"mlp.{n}.weight"), tp_rank, tp_size)
                                  for n in ("gate_proj", "up_proj")], device, fp8, dtype)
            lw.down = _pack_linear([_col_shard_pair(_get(wd, p + "mlp.down_proj.weight"), tp_rank, tp_size)],
                                   device, fp8, dtype)
        layers.append(lw)
    embed = wd[f"{prefix}embed_tokens.weight"].to(device, dtype)
    head = embed if cfg.tie_embeddings else wd["lm_head.weight"]
    vl = cfg.vocab // tp_size
    return ModelWeights(cfg=cfg, embed=embed, layers=layers,
                        final_norm=wd[f"{prefix}norm.weight"].to(device, dtype),
                        lm_head=head[tp_rank * vl:(tp_rank + 1) * vl].to(device, dtype).contiguous(),
                        vocab_start=tp_rank * vl, tp_rank=tp_rank, tp_size=tp_size)


def random_packed_weights(cfg: ModelConfig, device, seed: int = 0, tp_rank: int = 0, tp_size: int = 1,
                          std: float = 0.02) -> ModelWeights:
    """Random-init packed weights generated directly on the device, shard by shard (no host copy of
    the full model: 70B fp8 is generated in seconds). Each rank draws its own shard from a seed
    derived from (seed, layer, tensor, rank)."""
    fp8 = cfg.quant == "fp8_block"
    h, hd = cfg.hidden, cfg.head_dim
    if cfg.num_heads % tp_size or cfg.num_kv_heads % tp_size or cfg.ffn % tp_size:
        raise ValueError(f"{cfg.name}: heads {cfg.num_heads}/{cfg.num_kv_heads} and ffn {cfg.ffn} must divide "
                         f"over {tp_size} tensor-parallel ranks")
    hq, hkv, f = cfg.num_heads // tp_size, cfg.num_kv_heads // tp_size, cfg.ffn // tp_size
    gen = torch.Generator(device=device)

    def rnd(n, k, tag):
        gen.manual_seed(zlib.crc32(repr((seed, tag, tp_rank)).encode()) & 0x7FFFFFFF)
        w = torch.randn(n, k, device=device, generator=gen, dtype=torch.bfloat16) * std
        if fp8:
            q, s = quant_weight_block(w.float())
            del w
            return Linear(q, s)
        return Linear(w)

    layers = []
    for i in range(cfg.num_layers):
        lw = LayerWeights(in_norm=torch.ones(h, device=device, dtype=torch.bfloat16),
                          post_norm=torch.ones(h, device=device, dtype=torch.bfloat16),
                          qkv=rnd((hq + 2 * hkv) * hd, h, (i, "qkv")), o=rnd(h, hq * hd, (i, "o")))
        if cfg.is_moe:
            from .mixtral import random_moe
            lw.moe = random_moe(cfg, device, seed, i, tp_rank, tp_size, std)
        else:
            lw.gu = rnd(2 * f, h, (i, "gu"))
            lw.down = rnd(h, f, (i, "down"))
        layers.append(lw)
        torch.cuda.empty_cache() if torch.device(device).type == "cuda" else None
    gen.manual_seed(seed * 7 + 1)
    embed = torch.randn(cfg.vocab, h, device=device, generator=gen, dtype=torch.bfloat16) * std
    vl = cfg.vocab // tp_size
    gen.manual_seed(seed * 7 + 2 + tp_rank)
    head = torch.randn(vl, h, device=device, generator=gen, dtype=torch.bfloat16) * std
    return ModelWeights(cfg=cfg, embed=embed, layers=layers, final_norm=torch.ones(h, device=device, dtype=torch.bfloat16),
                        lm_head=head, vocab_start=tp_rank * vl, tp_rank=tp_rank, tp_size=tp_size)


# ------------------------------------------------------------------------------------------------
# forward
# ------------------------------------------------------------------------------------------------

@dataclass
class ForwardBatch:
    """Per-forward inputs (device tensors) plus the attention work lists."""

    tokens: torch.Tensor          # int64 [T]
    positions: torch.Tensor       # int32 [T]
    slots: torch.Tensor           # int64 [T] cache slot (page * page_size + offset)
    meta: object                  # AttnMeta
    work1: Optional[tuple] = None  # cascade pass-1 (items, tiles) or None
    work2: tuple = None            # main pass (items, tiles)
    logits_rows: Optional[torch.Tensor] = None  # rows whose logits are needed (None = all)
    gdn: Optional[object] = None  # hybrid models: models.hybrid.GdnBatch (ragged token ranges, state slots, mode)
    mm_rows: Optional[torch.Tensor] = None   # rows whose input embedding is an image feature (models/vision.py)
    mm_feats: Optional[torch.Tensor] = None  # [len(mm_rows), H]

    def embed(self, table: torch.Tensor) -> torch.Tensor:
        """Input embeddings of the batch: token embeddings, image features at the image rows."""
        h = table[self.tokens]
        if self.mm_rows is not None:
            h[self.mm_rows] = self.mm_feats.to(h.dtype)
        return h


class Communicator:
    """Tensor-parallel reduction hook; the single-GPU communicator is the identity."""

    size = 1
    rank = 0

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        return x

    def all_gather_vocab(self, x: torch.Tensor) -> torch.Tensor:
        return x


class LlamaModel:
    """Runs a packed Llama-family model over a paged KV cache."""

    def __init__(self, w: ModelWeights, kv_k: torch.Tensor, kv_v: torch.Tensor, cos_sin: torch.Tensor,
                 comm: Optional[Communicator] = None):
        self.w = w
        self.cfg = w.cfg
        self.kv_k = kv_k  # [L, P, Hkv_local, page, D]
        self.kv_v = kv_v
        self.cos_sin = cos_sin
        self.comm = comm or Communicator()
        self.hq = self.cfg.num_heads // w.tp_size
        self.hkv = self.cfg.num_kv_heads // w.tp_size
        self.scale = 1.0 / math.sqrt(self.cfg.head_dim)
        # MoE layers under expert parallelism on the collective path: False = every rank runs its experts over
        # every token and the outputs are all-reduced; True = all-to-all dispatch of each rank's own tokens
        # (MoEBlock.forward_a2a), outputs all-gathered
        self.moe_a2a = False

    def attention(self, li: int, q: torch.Tensor, fb: ForwardBatch, fp8_out: bool):
        t = q.shape[0]
        dt = q.dtype
        d = self.cfg.head_dim
        kc, vc = self.kv_k[li], self.kv_v[li]
        o_part = lse_part = None
        if fb.work1 is not None:
            o_part = torch.empty(t, self.hq, d, dtype=dt, device=q.device)
            lse_part = torch.full((t, self.hq), float("-inf"), dtype=torch.float32, device=q.device)
            it, tl = fb.work1
            ops.paged_attention(q, kc, vc, fb.meta, self.scale, o_part=o_part, lse_part=lse_part, items=it, tiles=tl)
        it, tl = fb.work2
        if fp8_out:
            oq = torch.empty(t, self.hq * d, dtype=FP8_DTYPE, device=q.device)
            os_ = torch.empty(self.hq, t, dtype=torch.float32, device=q.device)
            ops.paged_attention(q, kc, vc, fb.meta, self.scale, o_in=o_part, lse_in=lse_part, out_q=oq, out_qs=os_,
                                items=it, tiles=tl)
            return (oq, os_)
        out = torch.empty(t, self.hq * d, dtype=dt, device=q.device)
        ops.paged_attention(q, kc, vc, fb.meta, self.scale, o_in=o_part, lse_in=lse_part, out=out, items=it,
                            tiles=tl)
        return out

    def layer(self, li: int, h: torch.Tensor, delta: Optional[torch.Tensor], fb: ForwardBatch) -> torch.Tensor:
        lw = self.w.layers[li]
        cfg = self.cfg
        fp8 = lw.qkv.fp8
        xq, xs, xb = ops.add_rmsnorm_quant(h, delta, lw.in_norm, cfg.rms_eps, quant=fp8, out_bf16=not fp8)
        qkv = lw.qkv((xq, xs) if fp8 else xb)
        q = ops.rope_kv_write(qkv, fb.positions, fb.slots, self.cos_sin, self.kv_k[li], self.kv_v[li], self.hq,
                              self.hkv, cfg.head_dim)
        a = self.attention(li, q, fb, fp8)
        o = self.comm.all_reduce(lw.o(a))
        xq, xs, xb = ops.add_rmsnorm_quant(h, o, lw.post_norm, cfg.rms_eps, quant=fp8,
                                           out_bf16=(not fp8) or lw.moe is not None)
        if lw.moe is not None:
            if self.moe_a2a and self.comm.size > 1:
                return self._moe_a2a(lw.moe, xb)
            return self.comm.all_reduce(lw.moe((xq, xs) if fp8 else xb, xb))
        act = lw.gu.swiglu((xq, xs) if fp8 else xb)          # fp8: SwiGLU + quant in the GEMM epilogue
        return self.comm.all_reduce(lw.down(act))

    def _moe_a2a(self, moe, xb: torch.Tensor) -> torch.Tensor:
        """MoE output for every token via all-to-all dispatch: rank r routes rows [r*per, (r+1)*per) (per =
        ceil(T / W)), then the ranks' results are all-gathered."""
        W, r = self.comm.size, self.comm.rank
        t, hd = xb.shape
        per = (t + W - 1) // W
        lo, hi = min(t, r * per), min(t, (r + 1) * per)
        own = moe.forward_a2a(xb[lo:hi].contiguous(), self.comm)
        buf = torch.zeros(per, hd, dtype=own.dtype, device=xb.device)
        buf[:hi - lo] = own
        return self.comm._gather(buf).reshape(W * per, hd)[:t]

    def forward_fused(self, fb: ForwardBatch, want_hidden: bool = False):
        """Tensor-parallel forward on a fused communicator (parallel/fused.py): the residual stream lives in
        the communicator's symmetric workspace, o_proj / down_proj store each output row into its owner's
        receive slot from the GEMM epilogue (`project`), and one `ar_norm` kernel per reduction adds the
        slots + residual, normalizes, quantizes and all-gathers the rows the next GEMM reads."""
        comm, cfg = self.comm, self.cfg
        m = fb.tokens.shape[0]
        h = comm.h(m)
        h.copy_(fb.embed(self.w.embed))
        fp8 = self.w.layers[0].qkv.fp8
        xq, xs, xb = ops.add_rmsnorm_quant(h, None, self.w.layers[0].in_norm, cfg.rms_eps, quant=fp8, out_bf16=not fp8)
        x = (xq, xs) if fp8 else xb
        n = cfg.num_layers
        for li in range(n):
            _nvtx.push(f"layer{li}")
            lw = self.w.layers[li]
            qkv = lw.qkv(x)
            q = ops.rope_kv_write(qkv, fb.positions, fb.slots, self.cos_sin, self.kv_k[li], self.kv_v[li], self.hq,
                                  self.hkv, cfg.head_dim)
            a = self.attention(li, q, fb, fp8)
            comm.project(lw.o, a, m)
            if lw.moe is not None:
                yb = comm.ar_norm(m, lw.post_norm, cfg.rms_eps, out_bf16=True, recv=True)
                lw.moe(ops.act_quant(yb) if fp8 else yb, yb, out=comm.partial(m))
                recv = False
            else:
                x = comm.ar_norm(m, lw.post_norm, cfg.rms_eps, out_bf16=not fp8, recv=True)
                comm.project(lw.down, lw.gu.swiglu(x), m)   # fp8: SwiGLU + quant in the GEMM epilogue
                recv = True
            last = li == n - 1
            wnext = self.w.final_norm if last else self.w.layers[li + 1].in_norm
            x = comm.ar_norm(m, wnext, cfg.rms_eps, out_bf16=last or not fp8, push_h=last and want_hidden,
                             recv=recv)
            _nvtx.pop()
        rows = x if fb.logits_rows is None else x[fb.logits_rows]
        logits = ops.gemm_bf16(rows, self.w.lm_head)
        return logits, (h if want_hidden else None)

    def forward(self, fb: ForwardBatch, want_hidden: bool = False):
        """Returns (logits [rows, V_local] bf16, final residual h [T, H] bf16 (pre-norm) if want_hidden)."""
        comm = self.comm
        if (getattr(comm, "fused", False) and 0 < fb.tokens.shape[0] <= comm.max_tokens
                and comm.hidden == self.cfg.hidden):
            return self.forward_fused(fb, want_hidden)
        h = fb.embed(self.w.embed)
        delta = None
        for li in range(self.cfg.num_layers):
            _nvtx.push(f"layer{li}")
            delta = self.layer(li, h, delta, fb)
            _nvtx.pop()
        _, _, y = ops.add_rmsnorm_quant(h, delta, self.w.final_norm, self.cfg.rms_eps, quant=False, out_bf16=True)
        rows = y if fb.logits_rows is None else y[fb.logits_rows]
        logits = ops.gemm_bf16(rows, self.w.lm_head)
        return logits, (h if want_hidden else None)
