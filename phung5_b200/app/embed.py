"""View embedder for the judge's best-view stage and tie-breaks (a DINO-style ViT).

Reference: `DinoEmbedder` (pipeline_service/modules/judge/dino.py:12-156) lazily loads a DINOv3 ViT-S/16
through transformers, embeds PNG views in batches (L2-normalised pooled output), computes cosine
similarities to the prompt image and packs {prompt, view_*} vectors into an npz.

Here: when `model_dir` names a local transformers checkpoint it is loaded with AutoModel (no network);
otherwise a ViT-S/16-shaped encoder (patch 16, width 384, 12 blocks, 6 heads, CLS pooling) is built with
deterministic random weights, so the pipeline and its tests run anywhere. Images are resized to
`image_size` and normalised with ImageNet statistics; the encoder runs in bf16 on CUDA (fp32 on CPU) under
inference mode, in batches of `batch_size`.
"""
from __future__ import annotations

import asyncio
import io
import os
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class EmbedderSettings:
    enabled: bool = True
    model_dir: Optional[str] = None
    device: Optional[str] = None
    batch_size: int = 8
    image_size: int = 224
    width: int = 384
    depth: int = 12
    heads: int = 6
    patch: int = 16
    seed: int = 0


class _Block(nn.Module):
    def __init__(self, d, h):
        super().__init__()
        self.n1 = nn.LayerNorm(d, eps=1e-6)
        self.qkv = nn.Linear(d, 3 * d)
        self.proj = nn.Linear(d, d)
        self.n2 = nn.LayerNorm(d, eps=1e-6)
        self.fc1 = nn.Linear(d, 4 * d)
        self.fc2 = nn.Linear(4 * d, d)
        self.h = h
        self.ls1 = nn.Parameter(torch.full((d,), 1e-1))
        self.ls2 = nn.Parameter(torch.full((d,), 1e-1))

    def forward(self, x):
        b, t, d = x.shape
        q, k, v = self.qkv(self.n1(x)).view(b, t, 3, self.h, d // self.h).permute(2, 0, 3, 1, 4)
        a = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(b, t, d)
        x = x + self.ls1 * self.proj(a)
        return x + self.ls2 * self.fc2(F.gelu(self.fc1(self.n2(x))))


class ViT(nn.Module):
    def __init__(self, s: EmbedderSettings):
        super().__init__()
        d = s.width
        self.patch = nn.Conv2d(3, d, s.patch, s.patch)
        n = (s.image_size // s.patch) ** 2
        self.cls = nn.Parameter(torch.zeros(1, 1, d))
        self.pos = nn.Parameter(torch.zeros(1, n + 1, d))
        self.blocks = nn.ModuleList([_Block(d, s.heads) for _ in range(s.depth)])
        self.norm = nn.LayerNorm(d, eps=1e-6)

    def forward(self, x):
        p = self.patch(x).flatten(2).transpose(1, 2)
        x = torch.cat([self.cls.expand(p.shape[0], -1, -1), p], 1) + self.pos
        for b in self.blocks:
            x = b(x)
        return self.norm(x)[:, 0]


_MEAN = torch.tensor([0.485, 0.456, 0.406]).view(1, 3, 1, 1)
_STD = torch.tensor([0.229, 0.224, 0.225]).view(1, 3, 1, 1)


def _to_tensor(img) -> torch.Tensor:
    """PNG/JPEG bytes or an HxWx{3,4} uint8 tensor -> [3, H, W] float in [0, 1] (alpha over white)."""
    if isinstance(img, (bytes, bytearray)):
        from PIL import Image
        im = Image.open(io.BytesIO(img)).convert("RGBA")
        t = torch.from_numpy(np.asarray(im).copy())
    else:
        t = img.detach().to("cpu")
    t = t.float() / 255.0
    if t.shape[-1] == 4:
        a = t[..., 3:4]
        t = t[..., :3] * a + (1 - a)
    return t.permute(2, 0, 1)


class Embedder:
    def __init__(self, settings: Optional[EmbedderSettings] = None):
        self.s = settings or EmbedderSettings()
        self.model = None
        self.hf = False
        self.device = self.s.device or ("cuda" if torch.cuda.is_available() else "cpu")
        self._lock = asyncio.Lock()
        self.disabled = not self.s.enabled

    def _load(self):
        if self.s.model_dir and os.path.isdir(self.s.model_dir):
            from transformers import AutoModel
            self.model = AutoModel.from_pretrained(self.s.model_dir, local_files_only=True).eval().to(self.device)
            self.hf = True
        else:
            g = torch.random.fork_rng(devices=[])
            with g:
                torch.manual_seed(self.s.seed)
                m = ViT(self.s)
                for p in m.parameters():
                    if p.dim() > 1:
                        nn.init.trunc_normal_(p, std=0.02)
                nn.init.trunc_normal_(m.pos, std=0.02)
            self.model = m.eval().to(self.device)
        if self.device == "cuda":
            self.model = self.model.to(torch.bfloat16)

    def embed_sync(self, images: Sequence) -> np.ndarray:
        """-> [N, D] float32, L2-normalised."""
        if self.model is None:
            self._load()
        out = []
        size = self.s.image_size
        dt = torch.bfloat16 if self.device == "cuda" else torch.float32
        for i in range(0, len(images), max(1, self.s.batch_size)):
            xs = [F.interpolate(_to_tensor(im)[None], size=(size, size), mode="bilinear", align_corners=False)
                  for im in images[i:i + self.s.batch_size]]
            x = ((torch.cat(xs) - _MEAN) / _STD).to(self.device, dt)
            with torch.inference_mode():
                if self.hf:
                    o = self.model(pixel_values=x)
                    v = getattr(o, "pooler_output", None)
                    v = o.last_hidden_state[:, 0] if v is None else v
                else:
                    v = self.model(x)
            out.append(F.normalize(v.float(), dim=-1).cpu().numpy())
        return np.concatenate(out, 0) if out else np.zeros((0, self.s.width), np.float32)

    async def embed(self, images: Sequence) -> Optional[np.ndarray]:
        if self.disabled or not images:
            return None
        async with self._lock:      # one model, one batch at a time
            return await asyncio.to_thread(self.embed_sync, list(images))

    @staticmethod
    def similarities(ref: Optional[np.ndarray], views: np.ndarray) -> List[float]:
        if ref is None or views is None:
            return []
        return [round(float(v), 4) for v in views @ ref]

    @staticmethod
    def pack_npz(ref: Optional[np.ndarray], views: Dict[str, np.ndarray]) -> bytes:
        buf = io.BytesIO()
        arrays = {f"view_{k}": v for k, v in views.items()}
        if ref is not None:
            arrays["prompt"] = ref
        np.savez(buf, **arrays)
        return buf.getvalue()
