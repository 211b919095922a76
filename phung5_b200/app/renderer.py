"""Renderer module: candidate scene JSON -> judge views, gray-background rescue views and the 2x2 preview grid.

Reference: `RendererModule` (pipeline_service/modules/renderer/module.py:66-688) supervises Node/Chrome
sidecars and dispatches renders to slots; `compose_grid` (renderer/grid.py:25) builds the collage;
render_timeouts.py bounds each render. Here the renders are CUDA kernels (csrc/raster.cu) in-process, so a
"slot" is a worker thread with its own CUDA stream: `slots` renders run concurrently, each bounded by
`timeout_s`; a render that raises or times out is counted and reported to the caller, never retried
silently. On a host without a GPU the same code runs the rasterizer's C++ CPU restatement.

Views: "judge" = front views the duel compares (front, +-45 deg, side, back, top-down 60 deg);
"grid" = the four-view orbit (azimuth 24/120/216/312 deg) composed into the 2x2 preview.
"""
from __future__ import annotations

import asyncio
import io
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import torch

from ..render import scene as S

GRID_VIEWS = [(24.0, 15.0), (120.0, 15.0), (216.0, 15.0), (312.0, 15.0)]
JUDGE_VIEWS = [(0.0, 15.0), (45.0, 20.0), (-45.0, 20.0), (90.0, 15.0), (180.0, 15.0), (0.0, 60.0)]
WHITE = (1.0, 1.0, 1.0)
GRAY = (0.5, 0.5, 0.5)


@dataclass
class RendererSettings:
    slots: int = 4
    size: int = 384
    grid_size: int = 256
    grid_gap: int = 4
    timeout_s: float = 30.0
    device: str = "auto"        # "auto" -> cuda when available
    lighting: str = "studio"    # render/scene.py LIGHTING rig (standard-material shading); "lambert": flat rig


def to_png(img: torch.Tensor) -> bytes:
    from PIL import Image
    arr = img.detach().to("cpu").contiguous().numpy()
    out = io.BytesIO()
    Image.fromarray(arr, "RGBA").save(out, format="PNG", compress_level=1)
    return out.getvalue()


def compose_grid(tiles: Sequence[torch.Tensor], gap: int = 4) -> torch.Tensor:
    """Row-major square collage of equal tiles on opaque black with `gap`-pixel gutters."""
    import math
    n = len(tiles)
    if n == 0:
        raise ValueError("no tiles")
    h, w = tiles[0].shape[:2]
    cols = math.ceil(math.sqrt(n))
    rows = math.ceil(n / cols)
    canvas = torch.zeros(rows * h + (rows - 1) * gap, cols * w + (cols - 1) * gap, 4, dtype=torch.uint8,
                         device=tiles[0].device)
    canvas[..., 3] = 255
    for i, t in enumerate(tiles):
        if t.shape[:2] != (h, w):
            raise ValueError(f"grid tile {i} is {tuple(t.shape[:2])}, expected {(h, w)}")
        r, c = divmod(i, cols)
        canvas[r * (h + gap):r * (h + gap) + h, c * (w + gap):c * (w + gap) + w] = t
    return canvas


class RendererModule:
    def __init__(self, settings: Optional[RendererSettings] = None):
        self.s = settings or RendererSettings()
        dev = self.s.device
        if dev == "auto":
            dev = "cuda" if torch.cuda.is_available() else "cpu"
        self.device = dev
        self._pool = ThreadPoolExecutor(max_workers=self.s.slots, thread_name_prefix="render")
        self._local = threading.local()
        self.counts = {"renders": 0, "errors": 0, "timeouts": 0, "views": 0}
        self.seconds = 0.0

    def _stream(self):
        if self.device != "cuda":
            return None
        st = getattr(self._local, "stream", None)
        if st is None:
            st = torch.cuda.Stream()
            self._local.stream = st
        return st

    def _geometry(self, scene: dict):
        tris, cols, mats = S.scene_triangles(scene, with_materials=True)
        return S.normalise(tris), cols, mats

    def render_sync(self, scene: dict, views: Sequence, size: int, background=WHITE, yaw: float = 0.0) -> List[torch.Tensor]:
        """Render `views` [(azimuth, elevation)] of a scene; `yaw` rotates the object about +y first."""
        tris, cols, mats = self._geometry(scene)
        st = self._stream()
        ctx = torch.cuda.stream(st) if st is not None else _null()
        with ctx:
            tris = tris.to(self.device, non_blocking=False)
            cols = cols.to(self.device)
            mats = mats.to(self.device)
            if self.s.lighting == "lambert":
                out = [S.render(tris, cols, S.view_projection(a + yaw, e), size, background=background)
                       for a, e in views]
            else:
                out = [S.render_pbr(tris, cols, mats, a + yaw, e, size, self.s.lighting, background=background)
                       for a, e in views]
            if st is not None:
                st.synchronize()
        return out

    async def render(self, scene: dict, views: Sequence = JUDGE_VIEWS, size: Optional[int] = None,
                     background=WHITE, yaw: float = 0.0) -> List[torch.Tensor]:
        loop = asyncio.get_running_loop()
        t0 = time.monotonic()
        try:
            fut = loop.run_in_executor(self._pool, self.render_sync, scene, list(views), size or self.s.size,
                                       background, yaw)
            out = await asyncio.wait_for(fut, self.s.timeout_s)
        except asyncio.TimeoutError:
            self.counts["timeouts"] += 1
            raise
        except Exception:
            self.counts["errors"] += 1
            raise
        finally:
            self.seconds += time.monotonic() - t0
        self.counts["renders"] += 1
        self.counts["views"] += len(out)
        return out

    async def judge_views(self, scene: dict, gray: bool = True, yaw: float = 0.0) -> Dict[str, List[torch.Tensor]]:
        white = await self.render(scene, JUDGE_VIEWS, background=WHITE, yaw=yaw)
        out = {"white": white}
        if gray:
            out["gray"] = await self.render(scene, JUDGE_VIEWS, background=GRAY, yaw=yaw)
        return out

    async def grid_png(self, scene: dict) -> bytes:
        tiles = await self.render(scene, GRID_VIEWS, size=self.s.grid_size)
        return to_png(compose_grid(tiles, self.s.grid_gap))

    def health(self) -> dict:
        return {"device": self.device, "slots": self.s.slots, **self.counts, "seconds": round(self.seconds, 3)}

    def close(self):
        self._pool.shutdown(wait=False, cancel_futures=True)


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def data_url(png: bytes) -> str:
    import base64
    return "data:image/png;base64," + base64.b64encode(png).decode()
