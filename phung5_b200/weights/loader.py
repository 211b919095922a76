"""HF safetensors checkpoints: config.json -> ModelConfig, sharded weights read lazily per tensor-parallel rank.

A checkpoint directory holds `config.json` and either `model.safetensors` or shards listed by
`model.safetensors.index.json` (`weight_map`: tensor name -> shard file). `open_checkpoint` maps every
shard (safetensors memory-maps the file) and returns a `Checkpoint`, a read-only name -> tensor mapping
whose values are `LazyTensor`s: indexing one (`t[a:b]`, `t[:, a:b]`) reads only that slice from the file,
and `.to(...)` reads the whole tensor. The packers (models.llama.pack_weights, models.mixtral.pack_moe,
models.eagle.pack_eagle) slice row- and column-parallel weights before moving them, so each rank reads
only its shard of every sharded weight; replicated tensors (embedding, norms, the EAGLE fc) are read whole.

FP8 weights:
  * block-scaled (`quantization_config.weight_block_size` [128, 128], companion `<name>_scale_inv`
    [ceil(N/128), K/128] fp32): used as stored; non-power-of-two scales are requantized once at load to the
    power-of-two scales the tensor core applies (weights/quant.py ensure_pow2);
  * per-channel or per-tensor (`<name>_scale` [N, 1], [N] or []): dequantized on read (w * scale in fp32)
    and requantized to 128 x 128 power-of-two block scales by the packer -- one extra e4m3 rounding, since
    the engine's FP8 GEMMs take block scales (per-token x per-channel activations are not served natively).
bf16/fp16/fp32 weights of an fp8 model are quantized by the packer; of a bf16 model, used as bf16.

EAGLE heads (`load_eagle`): a separate directory whose tensors are either prefixed `eagle.` (this
framework's layout) or unprefixed EAGLE checkpoint names (`fc.weight`, `layers.0.*`, `norm.weight`);
both map to the `eagle.*` names pack_eagle reads.

The reference serves pinned HF checkpoints downloaded at container start (configuration.yaml:45-46,
docker/opt/prefetch/prefetch_shim.sh:24-35); this loader reads such a directory from local disk.
"""
from __future__ import annotations

import json
import os
from typing import Dict, Iterator, Mapping, Optional, Tuple

import torch

from ..config import ModelConfig

_FP8 = getattr(torch, "float8_e4m3fn", None)


class LazyTensor:
    """One checkpoint tensor, read from its memory-mapped shard on demand."""

    def __init__(self, handle, name: str, scale: Optional["LazyTensor"] = None):
        self._h, self.name = handle, name
        sl = handle.get_slice(name)
        self.shape = torch.Size(sl.get_shape())
        self._scale = scale           # per-channel / per-tensor fp8 scale: reads return w * scale (fp32)

    def dim(self) -> int:
        return len(self.shape)

    def _apply_scale(self, t: torch.Tensor, rows) -> torch.Tensor:
        if self._scale is None:
            return t
        s = self._scale.read().float()
        if s.numel() > 1:
            s = s.reshape(-1)[rows].reshape(-1, 1)
        return t.float() * s

    def __getitem__(self, idx) -> torch.Tensor:
        t = self._h.get_slice(self.name)[idx]
        rows = idx[0] if isinstance(idx, tuple) else idx
        return self._apply_scale(t, rows if isinstance(rows, slice) else slice(None))

    def read(self) -> torch.Tensor:
        return self._h.get_tensor(self.name)

    def to(self, *args, **kw) -> torch.Tensor:
        return self._apply_scale(self.read(), slice(None)).to(*args, **kw)

    def float(self) -> torch.Tensor:
        return self.to(torch.float32)


class Checkpoint(Mapping):
    """name -> LazyTensor over every shard of a checkpoint directory (see the module docstring)."""

    def __init__(self, path: str, rename=None):
        from safetensors import safe_open
        self.path = path
        index = os.path.join(path, "model.safetensors.index.json")
        if os.path.exists(index):
            with open(index) as f:
                wmap = json.load(f)["weight_map"]
            files = sorted(set(wmap.values()))
        else:
            files = sorted(f for f in os.listdir(path) if f.endswith(".safetensors"))
            if not files:
                raise FileNotFoundError(f"{path}: no model.safetensors or model.safetensors.index.json")
            wmap = None
        self._handles = {f: safe_open(os.path.join(path, f), framework="pt", device="cpu") for f in files}
        raw: Dict[str, Tuple[object, str]] = {}
        for f, h in self._handles.items():
            for k in h.keys():
                if wmap is not None and wmap.get(k, f) != f:
                    continue
                raw[k] = (h, k)
        rename = rename or (lambda k: k)
        self._entries: Dict[str, LazyTensor] = {}
        scales = {k[: -len("_scale")]: v for k, v in raw.items() if k.endswith(".weight_scale")}
        for k, (h, name) in raw.items():
            if k.endswith(".weight_scale") or k.endswith(".input_scale"):
                continue        # folded into the weight (per-channel) / dynamic activation quant (input)
            sc = scales.get(k)
            lt = LazyTensor(h, name, LazyTensor(*scales[k]) if sc is not None else None)
            self._entries[rename(k)] = lt

    def __getitem__(self, k: str) -> LazyTensor:
        return self._entries[k]

    def __iter__(self) -> Iterator[str]:
        return iter(self._entries)

    def __len__(self) -> int:
        return len(self._entries)


def config_from_hf(cfg: dict, name: Optional[str] = None) -> ModelConfig:
    """HF config.json (LlamaForCausalLM / MixtralForCausalLM) -> ModelConfig."""
    mt = cfg.get("model_type", "llama")
    arch = "mixtral" if mt == "mixtral" or cfg.get("num_local_experts") else "llama"
    h = int(cfg["hidden_size"])
    nh = int(cfg["num_attention_heads"])
    q = cfg.get("quantization_config") or {}
    quant = "bf16"
    if q.get("quant_method") in ("fp8", "compressed-tensors", "fbgemm_fp8") or q.get("fmt") == "e4m3":
        quant = "fp8_block"
    return ModelConfig(
        name=name or cfg.get("_name_or_path") or mt, arch=arch, num_layers=int(cfg["num_hidden_layers"]), hidden=h,
        num_heads=nh, num_kv_heads=int(cfg.get("num_key_value_heads", nh)),
        head_dim=int(cfg.get("head_dim") or h // nh), ffn=int(cfg["intermediate_size"]),
        vocab=int(cfg["vocab_size"]), rope_theta=float(cfg.get("rope_theta", 1e4)),
        rms_eps=float(cfg.get("rms_norm_eps", 1e-5)), max_position=int(cfg.get("max_position_embeddings", 131072)),
        tie_embeddings=bool(cfg.get("tie_word_embeddings", False)), quant=quant,
        num_experts=int(cfg.get("num_local_experts", 0) or 0),
        experts_per_token=int(cfg.get("num_experts_per_tok", 0) or 0))


def load_config(path: str) -> ModelConfig:
    with open(os.path.join(path, "config.json")) as f:
        return config_from_hf(json.load(f), name=os.path.basename(os.path.normpath(path)))


def open_checkpoint(path: str) -> Tuple[ModelConfig, Checkpoint]:
    return load_config(path), Checkpoint(path)


def load_model(path: str, device, tp_rank: int = 0, tp_size: int = 1, cfg: Optional[ModelConfig] = None):
    """Checkpoint directory -> (ModelConfig, packed device weights of this rank's shard)."""
    from ..models.llama import pack_weights
    mc, ck = open_checkpoint(path)
    if cfg is not None:
        mc = cfg
    return mc, pack_weights(mc, ck, device, tp_rank=tp_rank, tp_size=tp_size)


def load_eagle(path: str, target_cfg: ModelConfig, device, tp_rank: int = 0, tp_size: int = 1):
    """EAGLE head directory -> EagleWeights for `target_cfg` (see the module docstring for the names)."""
    from ..models.eagle import pack_eagle

    def rename(k: str) -> str:
        return k if k.startswith("eagle.") else "eagle." + (k[len("model."):] if k.startswith("model.") else k)
    return pack_eagle(target_cfg, Checkpoint(path, rename=rename), device, tp_rank=tp_rank, tp_size=tp_size)


def save_checkpoint(weights: Dict[str, torch.Tensor], cfg: ModelConfig, path: str, shards: int = 1) -> None:
    """Write HF-named weights as a (sharded) safetensors checkpoint with its config.json (tests, exports)."""
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    names = list(weights)
    per = (len(names) + shards - 1) // shards
    wmap = {}
    for s in range(shards):
        part = {k: weights[k].contiguous() for k in names[s * per:(s + 1) * per]}
        fn = "model.safetensors" if shards == 1 else f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
        save_file(part, os.path.join(path, fn))
        wmap.update({k: fn for k in part})
    if shards > 1:
        with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
            json.dump({"metadata": {}, "weight_map": wmap}, f)
    hf = {"model_type": "mixtral" if cfg.is_moe else "llama", "hidden_size": cfg.hidden,
          "num_hidden_layers": cfg.num_layers, "num_attention_heads": cfg.num_heads,
          "num_key_value_heads": cfg.num_kv_heads, "head_dim": cfg.head_dim, "intermediate_size": cfg.ffn,
          "vocab_size": cfg.vocab, "rope_theta": cfg.rope_theta, "rms_norm_eps": cfg.rms_eps,
          "tie_word_embeddings": cfg.tie_embeddings, "max_position_embeddings": cfg.max_position}
    if cfg.is_moe:
        hf.update(num_local_experts=cfg.num_experts, num_experts_per_tok=cfg.experts_per_token)
    if cfg.quant == "fp8_block":
        hf["quantization_config"] = {"quant_method": "fp8", "fmt": "e4m3", "weight_block_size": [128, 128],
                                     "activation_scheme": "dynamic"}
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(hf, f, indent=1)
