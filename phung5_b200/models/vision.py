"""Vision tower and image placeholders: image inputs for the serving engine.

The reference's coder and judge are vision-language models fed rendered views and reference photos
(configuration.yaml:39-54, 84-116); the judge's image encoder outputs are cached across requests
(docker/opt/jf: VLLM_ENC_CACHE_TOKENS) and the client sends each image once, then by uuid
(pipeline_service/llm/mm_resend.py:113-170). Here:

  * `VisionTower`: a ViT encoder (patch embedding, pre-norm transformer blocks, learned positions), a 2 x 2
    patch merge and a two-layer projector into the language model's hidden size: an image becomes
    (image_size / patch / merge)^2 feature rows. Weights are seeded random (no checkpoints offline) or loaded
    from safetensors names `vision.*`.
  * `VisionEncoder`: decodes an image (data URL or bytes), runs the tower, and keeps the features in an LRU
    cache keyed by the image's sha1 -- the encoder cache: an image seen before (sent in full or referenced by
    its uuid) is not encoded again.
  * `image_placeholders`: the token ids that stand for an image in the prompt. They are derived from the
    image's digest, so equal images give equal ids (the prefix cache may share them) and different images
    different ids; the engine replaces those rows' token embeddings with the image features during prefill
    (`ForwardBatch.mm_rows / mm_feats`, applied in models.llama).
"""
from __future__ import annotations

import base64
import hashlib
import io
import math
from collections import OrderedDict
from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class VisionConfig:
    image_size: int = 224
    patch: int = 14
    merge: int = 2
    width: int = 256
    depth: int = 2
    heads: int = 4
    out_hidden: int = 256          # the language model's hidden size
    seed: int = 7
    cache_entries: int = 256

    @property
    def tokens(self) -> int:
        g = self.image_size // self.patch // self.merge
        return g * g


class _Block(nn.Module):
    def __init__(self, d: int, heads: int):
        super().__init__()
        self.n1, self.n2 = nn.LayerNorm(d), nn.LayerNorm(d)
        self.qkv, self.proj = nn.Linear(d, 3 * d), nn.Linear(d, d)
        self.fc1, self.fc2 = nn.Linear(d, 4 * d), nn.Linear(4 * d, d)
        self.heads = heads

    def forward(self, x):
        b, n, d = x.shape
        q, k, v = self.qkv(self.n1(x)).view(b, n, 3, self.heads, d // self.heads).permute(2, 0, 3, 1, 4)
        a = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(b, n, d)
        x = x + self.proj(a)
        return x + self.fc2(F.gelu(self.fc1(self.n2(x))))


class VisionTower(nn.Module):
    def __init__(self, cfg: VisionConfig):
        super().__init__()
        self.cfg = cfg
        d, g = cfg.width, cfg.image_size // cfg.patch
        self.patch = nn.Linear(3 * cfg.patch * cfg.patch, d)
        self.pos = nn.Parameter(torch.zeros(g * g, d))
        self.blocks = nn.ModuleList(_Block(d, cfg.heads) for _ in range(cfg.depth))
        self.norm = nn.LayerNorm(d)
        self.proj1 = nn.Linear(d * cfg.merge * cfg.merge, cfg.out_hidden)
        self.proj2 = nn.Linear(cfg.out_hidden, cfg.out_hidden)

    def forward(self, pixels: torch.Tensor) -> torch.Tensor:
        """pixels [B, 3, S, S] (normalised) -> features [B, tokens, out_hidden]."""
        c = self.cfg
        b = pixels.shape[0]
        g = c.image_size // c.patch
        p = F.unfold(pixels, c.patch, stride=c.patch).transpose(1, 2)          # [B, g*g, 3*p*p]
        x = self.patch(p) + self.pos
        for blk in self.blocks:
            x = blk(x)
        x = self.norm(x).view(b, g // c.merge, c.merge, g // c.merge, c.merge, -1)
        x = x.permute(0, 1, 3, 2, 4, 5).reshape(b, (g // c.merge) ** 2, -1)  # 2 x 2 neighbourhoods merged
        return self.proj2(F.gelu(self.proj1(x)))


def random_tower(cfg: VisionConfig, device="cpu", dtype=torch.float32) -> VisionTower:
    with torch.random.fork_rng(devices=[]):
        torch.manual_seed(cfg.seed)
        t = VisionTower(cfg)
        for name, prm in t.named_parameters():
            if prm.dim() > 1:
                nn.init.normal_(prm, std=0.02 if name != "pos" else 0.01)
    return t.eval().to(device=device, dtype=dtype)


_MEAN = torch.tensor([0.485, 0.456, 0.406]).view(3, 1, 1)
_STD = torch.tensor([0.229, 0.224, 0.225]).view(3, 1, 1)


def decode_image(data) -> Tuple[str, torch.Tensor]:
    """bytes, a data URL, or an HxWx3/4 uint8 tensor -> (sha1 digest, float RGB [3, H, W] in [0, 1])."""
    if isinstance(data, torch.Tensor):
        raw = data.contiguous().cpu().numpy().tobytes()
        img = data[..., :3].permute(2, 0, 1).float() / 255.0
        return hashlib.sha1(raw).hexdigest(), img
    if isinstance(data, str):
        if not data.startswith("data:"):
            raise ValueError("only data: URLs are accepted for images")
        digest = hashlib.sha1(data.encode()).hexdigest()
        data = base64.b64decode(data.split(",", 1)[1])
    else:
        digest = hashlib.sha1(data).hexdigest()
    from PIL import Image
    import numpy as np
    with Image.open(io.BytesIO(data)) as im:
        arr = np.asarray(im.convert("RGB"), dtype=np.uint8).copy()
    return digest, torch.from_numpy(arr).permute(2, 0, 1).float() / 255.0


class VisionEncoder:
    """Image -> feature rows, with an LRU encoder cache keyed by the image digest."""

    def __init__(self, cfg: VisionConfig, device="cpu", dtype=torch.float32, tower: Optional[VisionTower] = None):
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dtype
        self.tower = tower if tower is not None else random_tower(cfg, device, dtype)
        self.cache: "OrderedDict[str, torch.Tensor]" = OrderedDict()
        self.stats = {"encoded": 0, "hits": 0, "misses": 0}

    def lookup(self, digest: str) -> Optional[torch.Tensor]:
        f = self.cache.get(digest)
        if f is not None:
            self.cache.move_to_end(digest)
            self.stats["hits"] += 1
        return f

    @torch.inference_mode()
    def encode(self, data, digest: Optional[str] = None) -> Tuple[str, torch.Tensor]:
        """-> (digest, features [tokens, out_hidden]); served from the cache when the image was seen."""
        d, img = decode_image(data)
        digest = digest or d
        f = self.lookup(digest)
        if f is not None:
            return digest, f
        self.stats["misses"] += 1
        s = self.cfg.image_size
        x = F.interpolate(img[None], size=(s, s), mode="bilinear", align_corners=False)
        x = ((x - _MEAN) / _STD).to(self.device, self.dtype)
        f = self.tower(x)[0]
        self.stats["encoded"] += 1
        self.cache[digest] = f
        while len(self.cache) > self.cfg.cache_entries:
            self.cache.popitem(last=False)
        return digest, f


def image_placeholders(digest: str, n: int, vocab: int, reserved: int = 258) -> List[int]:
    """n token ids standing for one image, derived from its digest (in [max(reserved, vocab // 2), vocab))."""
    lo = max(reserved, vocab // 2)
    span = max(1, vocab - lo)
    out = []
    for i in range(n):
        h = hashlib.blake2b(f"{digest}:{i}".encode(), digest_size=8).digest()
        out.append(lo + int.from_bytes(h, "little") % span)
    return out
