"""Hybrid decoder (Qwen3-Next style): Gated-DeltaNet linear-attention layers interleaved with full-attention
layers (layer i is full attention iff i % full_attn_every == full_attn_every - 1), every layer followed by a
SwiGLU MLP.

The reference's coder model is such a hybrid served by SGLang with its GDN verify/fold kernels
(docker/opt/kern/braw/kernels.py, a2/kernels.py) and chain (DFlash) speculation; tree verification is not
supported on GDN layers there either (braw/kernels.py:477-478). Here:
  - full-attention layers run exactly like `LlamaModel.layer` over the paged KV (which holds only the
    attention layers);
  - GDN layers keep a conv window and a recurrent state per request slot (`GdnPool`); a forward carries
    `ForwardBatch.gdn = GdnBatch(tok_start, slot, mode)`: "prefill" advances the state over the tokens,
    "verify" leaves it untouched and stashes what `commit(n)` needs to fold the first n tokens in after
    acceptance (models/gdn.py, csrc/gdn.cu).
"""
from __future__ import annotations

import zlib
from dataclasses import dataclass
from typing import List, Optional

import torch

from .. import ops
from ..config import ModelConfig
from .gdn import GDNLayer, random_gdn_layer
from .llama import ForwardBatch, LayerWeights, Linear, LlamaModel, ModelWeights, random_packed_weights


@dataclass
class GdnBatch:
    tok_start: torch.Tensor    # int32 [R+1]
    slot: torch.Tensor         # int32 [R]
    mode: str = "prefill"      # "prefill" | "verify"


@dataclass
class GdnLayerWeights:
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    gdn: GDNLayer
    gu: Linear
    down: Linear


class GdnPool:
    """Conv windows [L, slots, W-1, C] and recurrent states [L, slots, HV, 128, 128] (fp32) of the GDN layers."""

    def __init__(self, n_layers: int, slots: int, channels: int, taps: int, hv: int, device, dtype):
        self.window = torch.zeros(n_layers, slots, taps - 1, channels, dtype=dtype, device=device)
        self.state = torch.zeros(n_layers, slots, hv, 128, 128, dtype=torch.float32, device=device)
        self.free = list(range(slots - 1, -1, -1))

    def alloc(self) -> int:
        if not self.free:
            raise RuntimeError("no free GDN state slot")
        s = self.free.pop()
        self.window[:, s].zero_()
        self.state[:, s].zero_()
        return s

    def release(self, s: int) -> None:
        self.free.append(s)


def gdn_heads(cfg: ModelConfig):
    hv = cfg.gdn_heads
    return max(1, hv // 2), hv


class HybridModel:
    def __init__(self, w: ModelWeights, gdn_layers: List[Optional[GdnLayerWeights]], kv_k, kv_v, cos_sin,
                 pool: GdnPool, comm=None):
        """w.layers holds the full-attention layers in order; gdn_layers[i] is the GDN layer i or None."""
        self.cfg = w.cfg
        self.w = w
        self.attn = LlamaModel(w, kv_k, kv_v, cos_sin, comm)
        self.gdn_layers = gdn_layers
        self.pool = pool
        self.hq, self.hkv = self.attn.hq, self.attn.hkv
        self.comm = self.attn.comm
        self._verify: List[GDNLayer] = []

    def forward(self, fb: ForwardBatch, want_hidden: bool = False):
        cfg, eps = self.cfg, self.cfg.rms_eps
        h = self.w.embed[fb.tokens]
        delta = None
        ai = gi = 0
        gb: GdnBatch = fb.gdn
        self._verify = []
        for li in range(cfg.num_layers):
            gl = self.gdn_layers[li]
            if gl is None:
                delta = self.attn.layer(ai, h, delta, fb)
                ai += 1
                continue
            _, _, xb = ops.add_rmsnorm_quant(h, delta, gl.in_norm, eps, quant=False, out_bf16=True)
            mix = gl.gdn.forward(xb, gb.tok_start, gb.slot, self.pool.window[gi], self.pool.state[gi], mode=gb.mode)
            if gb.mode == "verify":
                self._verify.append((gl.gdn, gi))
            _, _, yb = ops.add_rmsnorm_quant(h, mix.to(h.dtype), gl.post_norm, eps, quant=False, out_bf16=True)
            gu = gl.gu(yb)
            _, _, ab = ops.silu_mul_quant(gu, quant=False, out_bf16=True)
            delta = gl.down(ab)
            gi += 1
        _, _, y = ops.add_rmsnorm_quant(h, delta, self.w.final_norm, eps, quant=False, out_bf16=True)
        rows = y if fb.logits_rows is None else y[fb.logits_rows]
        return ops.gemm_bf16(rows, self.w.lm_head), (h if want_hidden else None)

    def commit(self, n_accept: torch.Tensor) -> None:
        """After a verify forward: fold the first n_accept[r] verified tokens into every GDN layer's state."""
        for layer, gi in self._verify:
            layer.commit(n_accept.to(torch.int32), self.pool.window[gi], self.pool.state[gi])
        self._verify = []


def random_hybrid(cfg: ModelConfig, device, seed: int = 0, dtype=torch.bfloat16, std: float = 0.02):
    """-> (ModelWeights of the attention layers + embeddings, [GdnLayerWeights or None per layer])."""
    if cfg.quant != "bf16":
        raise ValueError("hybrid GDN models are served in bf16")
    full = random_packed_weights(cfg, device, seed=seed)
    attn_layers: List[LayerWeights] = []
    gdn: List[Optional[GdnLayerWeights]] = []
    hk, hv = gdn_heads(cfg)
    for i in range(cfg.num_layers):
        lw = full.layers[i]
        if cfg.layer_is_attention(i):
            attn_layers.append(lw)
            gdn.append(None)
        else:
            g = random_gdn_layer(cfg.hidden, hk, hv, device, seed=zlib.crc32(repr((seed, i)).encode()) & 0xFFFF,
                                 conv_w=cfg.gdn_conv_kernel, std=std, dtype=dtype)
            gdn.append(GdnLayerWeights(lw.in_norm, lw.post_norm, g, lw.gu, lw.down))
    w = ModelWeights(cfg=cfg, embed=full.embed, layers=attn_layers, final_norm=full.final_norm,
                     lm_head=full.lm_head, vocab_start=full.vocab_start, tp_rank=0, tp_size=1)
    if dtype != torch.bfloat16:
        w = _cast(w, dtype)
        gdn = [None if g is None else _cast_gdn(g, dtype) for g in gdn]
    return w, gdn


def _cast(w: ModelWeights, dtype) -> ModelWeights:
    def c(t):
        return t.to(dtype) if isinstance(t, torch.Tensor) and t.is_floating_point() else t
    layers = [LayerWeights(c(l.in_norm), c(l.post_norm), Linear(c(l.qkv.w)), Linear(c(l.o.w)), Linear(c(l.gu.w)),
                           Linear(c(l.down.w))) for l in w.layers]
    return ModelWeights(cfg=w.cfg, embed=c(w.embed), layers=layers, final_norm=c(w.final_norm), lm_head=c(w.lm_head),
                        vocab_start=w.vocab_start, tp_rank=w.tp_rank, tp_size=w.tp_size)


def _cast_gdn(g: GdnLayerWeights, dtype) -> GdnLayerWeights:
    import dataclasses
    L = g.gdn
    gl = dataclasses.replace(L, w_in=Linear(L.w_in.w.to(dtype)), w_ba=L.w_ba.to(dtype), conv_w=L.conv_w.to(dtype),
                             norm_w=L.norm_w.to(dtype), w_out=Linear(L.w_out.w.to(dtype)))
    return GdnLayerWeights(g.in_norm.to(dtype), g.post_norm.to(dtype), gl, Linear(g.gu.w.to(dtype)),
                           Linear(g.down.w.to(dtype)))
