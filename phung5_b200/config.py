"""Model, speculative-decoding and engine configuration.

One dataclass tree for the whole engine, with named presets for the model shapes the engine serves
(Llama-3-8B/70B, Mixtral-8x7B, a Qwen-style hybrid with Gated-DeltaNet layers, and the tiny CPU test
models), plus the strict 0/1 environment switch idiom of the reference's launch shims
(docker/opt/v5/kopt_shim.sh:50-52: anything but "0"/"1" counts as 0 and is reported).

The reference serves its models through external engines configured by YAML
(configuration.yaml:39-116, validated in pipeline_service/config/settings.py:228-347); here the
engine is in-process and the same information lives in `EngineConfig`.
"""
from __future__ import annotations

import dataclasses
import json
import os
import sys
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional


@dataclass
class ModelConfig:
    """Architecture of one decoder-only transformer.

    arch: "llama" (dense SwiGLU), "mixtral" (top-k routed SwiGLU experts) or "hybrid_gdn"
    (Gated-DeltaNet linear-attention layers interleaved with full-attention layers).
    quant: "bf16" or "fp8_block" (e4m3 weights with fp32 scales per 128x128 block, activations with
    one fp32 scale per token per 128 channels).
    """

    name: str = "tiny"
    arch: str = "llama"
    num_layers: int = 4
    hidden: int = 256
    num_heads: int = 4
    num_kv_heads: int = 4
    head_dim: int = 64
    ffn: int = 688
    vocab: int = 4096
    rope_theta: float = 1e4
    rms_eps: float = 1e-5
    max_position: int = 131072
    tie_embeddings: bool = False
    quant: str = "bf16"
    # MoE
    num_experts: int = 0
    experts_per_token: int = 0
    # hybrid GDN: layer i is full attention iff i % full_attn_every == full_attn_every - 1
    full_attn_every: int = 0
    gdn_heads: int = 0
    gdn_key_dim: int = 128
    gdn_value_dim: int = 128
    gdn_conv_kernel: int = 4

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    def layer_is_attention(self, i: int) -> bool:
        if self.arch != "hybrid_gdn" or self.full_attn_every <= 0:
            return True
        return i % self.full_attn_every == self.full_attn_every - 1

    def param_count(self) -> int:
        h, f = self.hidden, self.ffn
        attn = h * (self.q_size + 2 * self.kv_size) + self.q_size * h
        mlp = 3 * h * f * (self.num_experts if self.is_moe else 1)
        if self.is_moe:
            mlp += h * self.num_experts
        per_layer = attn + mlp + 2 * h
        emb = self.vocab * h * (1 if self.tie_embeddings else 2)
        return self.num_layers * per_layer + emb + h

    def to_dict(self) -> Dict[str, Any]:
        return dataclasses.asdict(self)


@dataclass
class DraftConfig:
    """Draft proposer.

    kind: "model" (a small standalone LM with its own embeddings and head, the CPU fp32 speculative-decode check) or
    "eagle" (a one-layer head fed fc([embed(token); target hidden]) that reuses the target's
    embedding and lm_head, the Llama-3-8B EAGLE benchmark).
    """

    kind: str = "model"
    num_layers: int = 1


@dataclass
class SpecConfig:
    """Speculative decoding schedule.

    mode "chain": k draft tokens in a line. mode "tree": a dynamic top-k tree of `tree_nodes` nodes
    (EAGLE-2 style: `depth` expansions, each keeping the `topk` best frontier nodes by cumulative
    draft log-probability).
    accept: "exact" runs the real target-vs-draft acceptance; "geometric" keeps every step of the
    verification (logits, target sampling, acceptance walk) but replaces the accepted length with a
    seeded Geometric(p) draw capped at `accept_cap`, the synthetic-acceptance workload of the
    benchmark configs (random-init weights never agree with their draft otherwise).
    """

    enabled: bool = True
    mode: str = "chain"
    num_draft: int = 4
    tree_nodes: int = 64
    topk: int = 8
    depth: int = 6
    accept: str = "exact"
    accept_p: float = 0.3
    accept_cap: int = 6
    accept_seed: int = 0


@dataclass
class ParallelConfig:
    tp: int = 1
    ep: int = 1
    # "nccl" = torch.distributed collectives + separate kernels (the baseline);
    # "fused" = in-kernel NVLink peer / multimem collectives (the product).
    comm: str = "fused"
    # MoE expert parallelism on the collective path: "reduce" = every rank runs its experts over every token, then
    # all-reduce; "a2a" = all-to-all dispatch / combine of each rank's own tokens (models/mixtral.py forward_a2a)
    moe_dispatch: str = "reduce"


@dataclass
class CacheConfig:
    page_size: int = 64
    num_pages: int = 0  # 0 = size from memory budget
    mem_fraction: float = 0.85
    enable_prefix_cache: bool = True
    enable_cascade: bool = True
    max_seqs: int = 256  # hybrid GDN models: recurrent state slots (concurrent requests)


@dataclass
class EngineConfig:
    model: ModelConfig = field(default_factory=ModelConfig)
    draft: DraftConfig = field(default_factory=DraftConfig)
    spec: SpecConfig = field(default_factory=SpecConfig)
    parallel: ParallelConfig = field(default_factory=ParallelConfig)
    cache: CacheConfig = field(default_factory=CacheConfig)
    max_running: int = 256
    max_prefill_tokens: int = 8192
    use_cuda_graphs: bool = True
    seed: int = 0

    def to_dict(self) -> Dict[str, Any]:
        return dataclasses.asdict(self)


# ---------------------------------------------------------------------------------------------
# Presets
# ---------------------------------------------------------------------------------------------

PRESETS: Dict[str, ModelConfig] = {
    # the CPU fp32 speculative-decode check target / draft (CPU fp32)
    "tiny": ModelConfig(name="tiny", num_layers=4, hidden=256, num_heads=4, num_kv_heads=4, head_dim=64,
                        ffn=688, vocab=4096, rope_theta=1e4, rms_eps=1e-5),
    "tiny-draft": ModelConfig(name="tiny-draft", num_layers=1, hidden=256, num_heads=4, num_kv_heads=4,
                              head_dim=64, ffn=688, vocab=4096, rope_theta=1e4, rms_eps=1e-5),
    "tiny-moe": ModelConfig(name="tiny-moe", arch="mixtral", num_layers=2, hidden=256, num_heads=4, num_kv_heads=4,
                            head_dim=64, ffn=256, vocab=4096, rope_theta=1e4, num_experts=4, experts_per_token=2),
    "llama3-8b": ModelConfig(name="llama3-8b", num_layers=32, hidden=4096, num_heads=32, num_kv_heads=8,
                             head_dim=128, ffn=14336, vocab=128256, rope_theta=5e5, rms_eps=1e-5),
    "llama3-70b": ModelConfig(name="llama3-70b", num_layers=80, hidden=8192, num_heads=64, num_kv_heads=8,
                              head_dim=128, ffn=28672, vocab=128256, rope_theta=5e5, rms_eps=1e-5),
    "llama3-70b-fp8": ModelConfig(name="llama3-70b-fp8", num_layers=80, hidden=8192, num_heads=64,
                                  num_kv_heads=8, head_dim=128, ffn=28672, vocab=128256, rope_theta=5e5,
                                  rms_eps=1e-5, quant="fp8_block"),
    "mixtral-8x7b-fp8": ModelConfig(name="mixtral-8x7b-fp8", arch="mixtral", num_layers=32, hidden=4096,
                                    num_heads=32, num_kv_heads=8, head_dim=128, ffn=14336, vocab=32000,
                                    rope_theta=1e6, rms_eps=1e-5, quant="fp8_block", num_experts=8,
                                    experts_per_token=2),
    # Qwen3-Next-style hybrid (GDN linear attention, 1 full-attention layer in 4)
    "hybrid-gdn-small": ModelConfig(name="hybrid-gdn-small", arch="hybrid_gdn", num_layers=8, hidden=1024,
                                    num_heads=8, num_kv_heads=2, head_dim=128, ffn=2816, vocab=32000,
                                    rope_theta=1e7, full_attn_every=4, gdn_heads=8),
    "tiny-hybrid": ModelConfig(name="tiny-hybrid", arch="hybrid_gdn", num_layers=4, hidden=256, num_heads=4,
                               num_kv_heads=2, head_dim=64, ffn=688, vocab=4096, full_attn_every=2, gdn_heads=2),
    # small GPU test shapes
    "small-fp8": ModelConfig(name="small-fp8", num_layers=2, hidden=1024, num_heads=8, num_kv_heads=2,
                             head_dim=128, ffn=2816 + 256, vocab=8192, rope_theta=5e5, quant="fp8_block"),
    # 8 KV heads: divides over 2, 4 and 8 tensor-parallel ranks (per-rank FFN 384 = 3 x 128 at 8 ranks)
    "small-fp8-kv8": ModelConfig(name="small-fp8-kv8", num_layers=2, hidden=1024, num_heads=16, num_kv_heads=8,
                                 head_dim=128, ffn=3072, vocab=8192, rope_theta=5e5, quant="fp8_block"),
    "small-bf16": ModelConfig(name="small-bf16", num_layers=2, hidden=1024, num_heads=8, num_kv_heads=2,
                              head_dim=128, ffn=3072, vocab=8192, rope_theta=5e5),
    "small-moe-fp8": ModelConfig(name="small-moe-fp8", arch="mixtral", num_layers=2, hidden=1024, num_heads=8,
                                 num_kv_heads=2, head_dim=128, ffn=1536, vocab=8192, quant="fp8_block",
                                 num_experts=8, experts_per_token=2),
}


def preset(name: str, **overrides) -> ModelConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}")
    return dataclasses.replace(PRESETS[name], **overrides)


# ---------------------------------------------------------------------------------------------
# Strict 0/1 switches
# ---------------------------------------------------------------------------------------------

def switch(name: str, default: bool = False) -> bool:
    """Read an on/off environment switch. Only "0" and "1" are valid; anything else counts as off
    and is reported once on stderr, like the reference shims (v5/kopt_shim.sh:50-52)."""
    v = os.environ.get(name)
    if v is None:
        return default
    if v == "1":
        return True
    if v != "0":
        print(f"!! {name}={v!r} is not 0/1; treated as 0", file=sys.stderr)
    return False


def load_engine_config(path: Optional[str] = None, overrides: Optional[Dict[str, Any]] = None) -> EngineConfig:
    """Build an EngineConfig from an optional YAML/JSON file plus dotted overrides
    (e.g. {"spec.mode": "tree", "model": "llama3-8b"})."""
    data: Dict[str, Any] = {}
    if path:
        with open(path) as f:
            text = f.read()
        if path.endswith((".yaml", ".yml")):
            import yaml
            data = yaml.safe_load(text) or {}
        else:
            data = json.loads(text)
    for k, v in (overrides or {}).items():
        cur = data
        parts = k.split(".")
        for p in parts[:-1]:
            cur = cur.setdefault(p, {})
        cur[parts[-1]] = v
    cfg = EngineConfig()
    m = data.get("model")
    if isinstance(m, str):
        cfg.model = preset(m)
    elif isinstance(m, dict):
        base = preset(m.pop("preset")) if "preset" in m else ModelConfig()
        cfg.model = dataclasses.replace(base, **m)
    for key, cls in (("draft", DraftConfig), ("spec", SpecConfig), ("parallel", ParallelConfig),
                     ("cache", CacheConfig)):
        if key in data:
            setattr(cfg, key, dataclasses.replace(getattr(cfg, key), **data[key]))
    for key in ("max_running", "max_prefill_tokens", "use_cuda_graphs", "seed"):
        if key in data:
            setattr(cfg, key, data[key])
    return cfg
