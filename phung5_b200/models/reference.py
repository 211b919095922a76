"""Plain-PyTorch fp32 oracle of the served model families.

This is the correctness reference for every kernel and for the engine: a straightforward, unbatched,
unpaged forward pass over HF-named weights (``model.layers.{i}.self_attn.q_proj.weight`` ...), with a
contiguous per-request KV cache and an explicit boolean attention mask (causal for prefill and
chain verification, ancestor mask for tree verification).

Families: Llama (dense SwiGLU), Mixtral (top-k routed experts, softmax over the selected logits),
the standalone draft LM, and the EAGLE-style draft head (fc([embed; hidden]) -> one decoder layer ->
shared lm_head). FP8 block-scaled checkpoints are dequantized on load (weight * scale_inv per
128x128 block), so the oracle computes in fp32 on the dequantized weights.

The reference itself has no model code (its models run inside SGLang/vLLM, configuration.yaml:39-116);
its kernel self-tests compare against the stock engine path (e.g. docker/opt/v5/fusedq/fusedq.py:139-198).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F

from ..config import ModelConfig

Weights = Dict[str, torch.Tensor]


def dequant_block_fp8(w: torch.Tensor, scale_inv: torch.Tensor, block: int = 128) -> torch.Tensor:
    """fp8 [N, K] with fp32 scale_inv [ceil(N/128), ceil(K/128)] -> fp32 [N, K]."""
    n, k = w.shape
    s = scale_inv.float().repeat_interleave(block, 0)[:n].repeat_interleave(block, 1)[:, :k]
    return w.float() * s


def get_weight(w: Weights, name: str) -> torch.Tensor:
    t = w[name]
    si = w.get(name + "_scale_inv")
    if si is not None:
        return dequant_block_fp8(t, si)
    return t.float()


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * weight.float()


def rope_cos_sin(positions: torch.Tensor, head_dim: int, theta: float) -> Tuple[torch.Tensor, torch.Tensor]:
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    ang = positions.double()[:, None] * inv[None, :]
    return ang.cos().float(), ang.sin().float()


def apply_rope(x: torch.Tensor, positions: torch.Tensor, theta: float) -> torch.Tensor:
    """x [T, H, D]; rotate-half (NeoX/Llama HF) convention."""
    d = x.shape[-1]
    cos, sin = rope_cos_sin(positions.cpu(), d, theta)
    cos, sin = cos.to(x.device)[:, None, :], sin.to(x.device)[:, None, :]
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


@dataclass
class RefKV:
    """Contiguous KV cache of one request: per layer [S, Hkv, D] fp32."""

    k: List[torch.Tensor] = field(default_factory=list)
    v: List[torch.Tensor] = field(default_factory=list)

    def length(self) -> int:
        return 0 if not self.k else self.k[0].shape[0]

    def truncate(self, n: int) -> None:
        self.k = [t[:n] for t in self.k]
        self.v = [t[:n] for t in self.v]

    def keep(self, idx: torch.Tensor) -> None:
        """Keep only rows `idx` (used to compact the accepted path of a verified tree)."""
        self.k = [t[idx] for t in self.k]
        self.v = [t[idx] for t in self.v]

    def clone(self) -> "RefKV":
        return RefKV([t.clone() for t in self.k], [t.clone() for t in self.v])


def causal_mask(prev: int, t: int) -> torch.Tensor:
    """[t, prev + t] bool: query i sees all previous keys and new keys j <= i."""
    m = torch.ones(t, prev + t, dtype=torch.bool)
    m[:, prev:] = torch.tril(torch.ones(t, t, dtype=torch.bool))
    return m


def attention(q, k, v, mask, scale):
    """q [T, Hq, D], k/v [S, Hkv, D], mask [T, S] bool -> [T, Hq, D]."""
    hq, hkv = q.shape[1], k.shape[1]
    rep = hq // hkv
    k = k.repeat_interleave(rep, dim=1)
    v = v.repeat_interleave(rep, dim=1)
    s = torch.einsum("thd,shd->hts", q, k) * scale
    s = s.masked_fill(~mask[None].to(s.device), float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hts,shd->thd", p, v)


def moe_mlp(x: torch.Tensor, w: Weights, pre: str, cfg: ModelConfig) -> torch.Tensor:
    """Mixtral routing: softmax over the top-k router logits, weighted sum of SwiGLU experts."""
    logits = x @ get_weight(w, pre + "block_sparse_moe.gate.weight").t()
    topv, topi = torch.topk(logits, cfg.experts_per_token, dim=-1)
    gates = torch.softmax(topv, dim=-1)
    out = torch.zeros_like(x)
    for e in range(cfg.num_experts):
        rows, slot = (topi == e).nonzero(as_tuple=True)
        if rows.numel() == 0:
            continue
        xe = x[rows]
        ep = pre + f"block_sparse_moe.experts.{e}."
        h = F.silu(xe @ get_weight(w, ep + "w1.weight").t()) * (xe @ get_weight(w, ep + "w3.weight").t())
        out.index_add_(0, rows, (h @ get_weight(w, ep + "w2.weight").t()) * gates[rows, slot][:, None])
    return out


def decoder_layer(x: torch.Tensor, w: Weights, pre: str, cfg: ModelConfig, positions: torch.Tensor,
                  kv: RefKV, li: int, mask: torch.Tensor) -> torch.Tensor:
    t = x.shape[0]
    h = rms_norm(x, w[pre + "input_layernorm.weight"], cfg.rms_eps)
    q = (h @ get_weight(w, pre + "self_attn.q_proj.weight").t()).view(t, cfg.num_heads, cfg.head_dim)
    k = (h @ get_weight(w, pre + "self_attn.k_proj.weight").t()).view(t, cfg.num_kv_heads, cfg.head_dim)
    v = (h @ get_weight(w, pre + "self_attn.v_proj.weight").t()).view(t, cfg.num_kv_heads, cfg.head_dim)
    q = apply_rope(q, positions, cfg.rope_theta)
    k = apply_rope(k, positions, cfg.rope_theta)
    if len(kv.k) <= li:
        kv.k.append(k)
        kv.v.append(v)
    else:
        kv.k[li] = torch.cat([kv.k[li], k], 0)
        kv.v[li] = torch.cat([kv.v[li], v], 0)
    a = attention(q, kv.k[li], kv.v[li], mask, 1.0 / math.sqrt(cfg.head_dim)).reshape(t, cfg.q_size)
    x = x + a @ get_weight(w, pre + "self_attn.o_proj.weight").t()
    h = rms_norm(x, w[pre + "post_attention_layernorm.weight"], cfg.rms_eps)
    if cfg.is_moe:
        m = moe_mlp(h, w, pre, cfg)
    else:
        g = h @ get_weight(w, pre + "mlp.gate_proj.weight").t()
        u = h @ get_weight(w, pre + "mlp.up_proj.weight").t()
        m = (F.silu(g) * u) @ get_weight(w, pre + "mlp.down_proj.weight").t()
    return x + m


class RefModel:
    """fp32 oracle for a Llama/Mixtral-family target or standalone draft LM."""

    def __init__(self, cfg: ModelConfig, weights: Weights):
        self.cfg = cfg
        self.w = weights

    def new_cache(self) -> RefKV:
        return RefKV()

    def forward(self, tokens: torch.Tensor, positions: torch.Tensor, kv: RefKV,
                mask: Optional[torch.Tensor] = None, embeds: Optional[Tuple[torch.Tensor, torch.Tensor]] = None
                ) -> Tuple[torch.Tensor, torch.Tensor]:
        """tokens/positions [T] -> (logits [T, V] fp32, last-layer hidden before the final norm [T, H]).
        embeds: (rows, features) replacing those rows' token embeddings (image inputs)."""
        cfg, w = self.cfg, self.w
        t = tokens.shape[0]
        if mask is None:
            mask = causal_mask(kv.length(), t)
        x = w["model.embed_tokens.weight"].float()[tokens]
        if embeds is not None:
            x[embeds[0]] = embeds[1].float()
        for i in range(cfg.num_layers):
            x = decoder_layer(x, w, f"model.layers.{i}.", cfg, positions, kv, i, mask)
        hn = rms_norm(x, w["model.norm.weight"], cfg.rms_eps)
        head = w["model.embed_tokens.weight"] if cfg.tie_embeddings else w["lm_head.weight"]
        return hn @ head.float().t(), x


class RefEagleHead:
    """One-layer EAGLE-style draft head: z = fc([embed(tok); h_target]); one decoder layer; own final
    norm; the target's lm_head. Weights: ``eagle.fc.weight`` [H, 2H], ``eagle.layers.0.*``,
    ``eagle.norm.weight``; embedding and head are the target's."""

    def __init__(self, cfg: ModelConfig, weights: Weights, target_weights: Weights):
        self.cfg = cfg
        self.w = weights
        self.tw = target_weights

    def new_cache(self) -> RefKV:
        return RefKV()

    def forward(self, tokens: torch.Tensor, hidden: torch.Tensor, positions: torch.Tensor, kv: RefKV,
                mask: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        cfg = self.cfg
        t = tokens.shape[0]
        if mask is None:
            mask = causal_mask(kv.length(), t)
        e = self.tw["model.embed_tokens.weight"].float()[tokens]
        z = torch.cat([e, hidden.float()], -1) @ get_weight(self.w, "eagle.fc.weight").t()
        x = decoder_layer(z, self.w, "eagle.layers.0.", cfg, positions, kv, 0, mask)
        hn = rms_norm(x, self.w["eagle.norm.weight"], cfg.rms_eps)
        head = self.tw["model.embed_tokens.weight"] if cfg.tie_embeddings else self.tw["lm_head.weight"]
        return hn @ head.float().t(), x
