"""Seeded random initialisation of HF-named weights (no checkpoints are available offline).

Produces the same tensor names an HF safetensors checkpoint of the architecture has, so the engine's
loader, the oracle and the tests share one path. For FP8 block-scaled models every linear weight is
quantized with `quant_weight_block` and stored with its ``_scale_inv`` companion, as in FP8
checkpoints.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch

from ..config import ModelConfig
from .quant import quant_weight_block

Weights = Dict[str, torch.Tensor]


def _linear(g: torch.Generator, n: int, k: int, std: float, device) -> torch.Tensor:
    return (torch.randn(n, k, generator=g, dtype=torch.float32) * std).to(device)


def _add_linear(w: Weights, name: str, t: torch.Tensor, fp8: bool) -> None:
    if fp8:
        q, s = quant_weight_block(t)
        w[name] = q
        w[name + "_scale_inv"] = s
    else:
        w[name] = t


def random_weights(cfg: ModelConfig, seed: int = 0, std: float = 0.02, device="cpu",
                   dtype: torch.dtype = torch.float32, fp8: Optional[bool] = None) -> Weights:
    """HF-layout random weights for a Llama/Mixtral model. Norm weights are 1."""
    fp8 = cfg.quant == "fp8_block" if fp8 is None else fp8
    g = torch.Generator().manual_seed(seed)
    w: Weights = {}
    h = cfg.hidden
    w["model.embed_tokens.weight"] = _linear(g, cfg.vocab, h, std, device).to(dtype)
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        w[p + "input_layernorm.weight"] = torch.ones(h, device=device, dtype=dtype)
        w[p + "post_attention_layernorm.weight"] = torch.ones(h, device=device, dtype=dtype)
        for nm, n in (("q_proj", cfg.q_size), ("k_proj", cfg.kv_size), ("v_proj", cfg.kv_size)):
            _add_linear(w, p + f"self_attn.{nm}.weight", _linear(g, n, h, std, device).to(dtype), fp8)
        _add_linear(w, p + "self_attn.o_proj.weight", _linear(g, h, cfg.q_size, std, device).to(dtype), fp8)
        if cfg.is_moe:
            w[p + "block_sparse_moe.gate.weight"] = _linear(g, cfg.num_experts, h, std, device).to(dtype)
            for e in range(cfg.num_experts):
                ep = p + f"block_sparse_moe.experts.{e}."
                _add_linear(w, ep + "w1.weight", _linear(g, cfg.ffn, h, std, device).to(dtype), fp8)
                _add_linear(w, ep + "w3.weight", _linear(g, cfg.ffn, h, std, device).to(dtype), fp8)
                _add_linear(w, ep + "w2.weight", _linear(g, h, cfg.ffn, std, device).to(dtype), fp8)
        else:
            _add_linear(w, p + "mlp.gate_proj.weight", _linear(g, cfg.ffn, h, std, device).to(dtype), fp8)
            _add_linear(w, p + "mlp.up_proj.weight", _linear(g, cfg.ffn, h, std, device).to(dtype), fp8)
            _add_linear(w, p + "mlp.down_proj.weight", _linear(g, h, cfg.ffn, std, device).to(dtype), fp8)
    w["model.norm.weight"] = torch.ones(h, device=device, dtype=dtype)
    if not cfg.tie_embeddings:
        w["lm_head.weight"] = _linear(g, cfg.vocab, h, std, device).to(dtype)
    return w


def random_eagle_weights(cfg: ModelConfig, seed: int = 1, std: float = 0.02, device="cpu",
                         dtype: torch.dtype = torch.float32, fp8: Optional[bool] = None) -> Weights:
    """Weights of a one-layer EAGLE-style head for target `cfg` (embedding and lm_head are shared)."""
    fp8 = cfg.quant == "fp8_block" if fp8 is None else fp8
    g = torch.Generator().manual_seed(seed)
    w: Weights = {}
    h = cfg.hidden
    _add_linear(w, "eagle.fc.weight", _linear(g, h, 2 * h, std, device).to(dtype), fp8)
    p = "eagle.layers.0."
    w[p + "input_layernorm.weight"] = torch.ones(h, device=device, dtype=dtype)
    w[p + "post_attention_layernorm.weight"] = torch.ones(h, device=device, dtype=dtype)
    for nm, n in (("q_proj", cfg.q_size), ("k_proj", cfg.kv_size), ("v_proj", cfg.kv_size)):
        _add_linear(w, p + f"self_attn.{nm}.weight", _linear(g, n, h, std, device).to(dtype), fp8)
    _add_linear(w, p + "self_attn.o_proj.weight", _linear(g, h, cfg.q_size, std, device).to(dtype), fp8)
    _add_linear(w, p + "mlp.gate_proj.weight", _linear(g, cfg.ffn, h, std, device).to(dtype), fp8)
    _add_linear(w, p + "mlp.up_proj.weight", _linear(g, cfg.ffn, h, std, device).to(dtype), fp8)
    _add_linear(w, p + "mlp.down_proj.weight", _linear(g, h, cfg.ffn, std, device).to(dtype), fp8)
    w["eagle.norm.weight"] = torch.ones(h, device=device, dtype=dtype)
    return w
