"""EAGLE-style one-layer draft head on the engine kernels.

Input at position t: z = fc([embed(x_t); f_{t-1}]) where f_{t-1} is the target's last-layer hidden
state (pre-norm) at position t-1 (or the head's own output feature when drafting past committed
tokens); one decoder layer over the head's own paged KV (same page table as the target, separate
tensors); the head's final norm; the target's lm_head. The Llama-3-8B benchmark names this drafter
("1-layer EAGLE-style head fed target hidden state + token embedding"); the reference's coder uses a
DFlash drafter inside SGLang (configuration.yaml:54).
"""
from __future__ import annotations

import zlib
from dataclasses import dataclass
from typing import Dict, Optional

import torch

from .. import ops
from ..config import ModelConfig
from .llama import (ForwardBatch, LayerWeights, Linear, LlamaModel, ModelWeights, _col_shard_pair, _get,
                    _pack_linear, _row_shard_pair)
from ..weights.quant import quant_weight_block


@dataclass
class EagleWeights:
    fc: Linear          # [H, 2H], replicated on every rank
    layer: LayerWeights
    norm: torch.Tensor


def pack_eagle(cfg: ModelConfig, wd: Dict[str, torch.Tensor], device, tp_rank=0, tp_size=1) -> EagleWeights:
    fp8 = cfg.quant == "fp8_block"
    p = "eagle.layers.0."
    layer = LayerWeights(
        in_norm=wd[p + "input_layernorm.weight"].to(device, torch.bfloat16),
        post_norm=wd[p + "post_attention_layernorm.weight"].to(device, torch.bfloat16),
        qkv=_pack_linear([_row_shard_pair(_get(wd, p + f"self_attn.{n}.weight"), tp_rank, tp_size)
                          for n in ("q_proj", "k_proj", "v_proj")], device, fp8),
        o=_pack_linear([_col_shard_pair(_get(wd, p + "self_attn.o_proj.weight"), tp_rank, tp_size)], device, fp8),
        gu=_pack_linear([_row_shard_pair(_get(wd, p + f"mlp.{n}.weight"), tp_rank, tp_size)
                         for n in ("gate_proj", "up_proj")], device, fp8),
        down=_pack_linear([_col_shard_pair(_get(wd, p + "mlp.down_proj.weight"), tp_rank, tp_size)], device, fp8))
    fc = _pack_linear([_get(wd, "eagle.fc.weight")], device, fp8)
    return EagleWeights(fc=fc, layer=layer, norm=wd["eagle.norm.weight"].to(device, torch.bfloat16))


def random_eagle(cfg: ModelConfig, device, seed=1, tp_rank=0, tp_size=1, std=0.02) -> EagleWeights:
    fp8 = cfg.quant == "fp8_block"
    h, hd = cfg.hidden, cfg.head_dim
    hq, hkv, f = cfg.num_heads // tp_size, cfg.num_kv_heads // tp_size, cfg.ffn // tp_size
    gen = torch.Generator(device=device)

    def rnd(n, k, tag, rank_specific=True):
        gen.manual_seed(zlib.crc32(repr((seed, tag, tp_rank if rank_specific else 0)).encode()) & 0x7FFFFFFF)
        w = torch.randn(n, k, device=device, generator=gen, dtype=torch.bfloat16) * std
        if fp8:
            q, s = quant_weight_block(w.float())
            return Linear(q, s)
        return Linear(w)

    layer = LayerWeights(in_norm=torch.ones(h, device=device, dtype=torch.bfloat16),
                         post_norm=torch.ones(h, device=device, dtype=torch.bfloat16),
                         qkv=rnd((hq + 2 * hkv) * hd, h, "qkv"), o=rnd(h, hq * hd, "o"),
                         gu=rnd(2 * f, h, "gu"), down=rnd(h, f, "down"))
    return EagleWeights(fc=rnd(h, 2 * h, "fc", rank_specific=False), layer=layer,
                        norm=torch.ones(h, device=device, dtype=torch.bfloat16))


class EagleHead:
    """Draft head runner. `target` supplies embedding and lm_head (vocab shard)."""

    def __init__(self, ew: EagleWeights, target_w: ModelWeights, kv_k: torch.Tensor, kv_v: torch.Tensor,
                 cos_sin: torch.Tensor, comm=None):
        self.ew = ew
        self.tw = target_w
        mw = ModelWeights(cfg=target_w.cfg, embed=target_w.embed, layers=[ew.layer], final_norm=ew.norm,
                          lm_head=target_w.lm_head, vocab_start=target_w.vocab_start, tp_rank=target_w.tp_rank,
                          tp_size=target_w.tp_size)
        self.runner = LlamaModel(mw, kv_k, kv_v, cos_sin, comm)
        self.cfg = target_w.cfg

    def forward(self, fb: ForwardBatch, hidden_in: torch.Tensor):
        """Returns (logits [rows, V_local], output feature [T, H] (pre-norm)). On a fused communicator the
        feature is a view of its workspace, valid until the next forward."""
        e = self.tw.embed[fb.tokens]
        cat = torch.cat([e, hidden_in.to(torch.bfloat16)], -1)
        if self.ew.fc.fp8:
            z = self.ew.fc(ops.act_quant(cat))
        else:
            z = self.ew.fc(cat)
        comm = self.runner.comm
        m = z.shape[0]
        if getattr(comm, "fused", False) and 0 < m <= comm.max_tokens and comm.hidden == self.cfg.hidden:
            return self._forward_fused(fb, z)
        h = z
        delta = self.runner.layer(0, h, None, fb)
        _, _, y = ops.add_rmsnorm_quant(h, delta, self.ew.norm, self.cfg.rms_eps, quant=False, out_bf16=True)
        rows = y if fb.logits_rows is None else y[fb.logits_rows]
        return ops.gemm_bf16(rows, self.tw.lm_head), h

    def _forward_fused(self, fb: ForwardBatch, z: torch.Tensor):
        """The head's layer on the fused communicator: residual in the symmetric workspace, o_proj / down_proj
        partials reduced by `ar_norm` (+ RMSNorm + quant), the final norm's reduction also gathering the
        residual rows every rank needs as the next round's feature."""
        comm, cfg, lw, r = self.runner.comm, self.cfg, self.ew.layer, self.runner
        m = z.shape[0]
        fp8 = lw.qkv.fp8
        h = comm.h(m)
        h.copy_(z)
        xq, xs, xb = ops.add_rmsnorm_quant(h, None, lw.in_norm, cfg.rms_eps, quant=fp8, out_bf16=not fp8)
        qkv = lw.qkv((xq, xs) if fp8 else xb)
        q = ops.rope_kv_write(qkv, fb.positions, fb.slots, r.cos_sin, r.kv_k[0], r.kv_v[0], r.hq, r.hkv, cfg.head_dim)
        a = r.attention(0, q, fb, fp8)
        comm.project(lw.o, a, m)
        x = comm.ar_norm(m, lw.post_norm, cfg.rms_eps, out_bf16=not fp8, recv=True)
        comm.project(lw.down, lw.gu.swiglu(x), m)      # fp8: SwiGLU + quant in the gate/up GEMM epilogue
        y = comm.ar_norm(m, self.ew.norm, cfg.rms_eps, out_bf16=True, push_h=True, recv=True)
        rows = y if fb.logits_rows is None else y[fb.logits_rows]
        return ops.gemm_bf16(rows, self.tw.lm_head), h
