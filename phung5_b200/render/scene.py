"""Scene previews without a graphics stack: three.js-style scene JSON -> world-space triangles -> the
CUDA rasterizer (csrc/raster.cu; CPU tensors run its C++ restatement, the oracle).

Supported scene JSON (the subset of three.js ObjectLoader JSON that the reference's serializer emits,
pipeline_service/modules/js_checker/validator/serialize_worker.mjs): "geometries" with type
BoxGeometry, SphereGeometry, CylinderGeometry, ConeGeometry, PlaneGeometry, TorusGeometry or
BufferGeometry (data.attributes.position + optional data.index); "materials" with a "color" (int
0xRRGGBB); and an "object" tree whose nodes carry a column-major 4x4 "matrix", "children", and
"geometry"/"material" uuids. Views follow the reference's presets: camera on a sphere of radius 2
around the unit-normalised object, vertical fov 49.1 degrees (renderer/render_service/renderer.js:10-15).
"""
from __future__ import annotations

import math
from typing import Optional, Dict, List, Sequence, Tuple

import torch

from .. import ops


def _box(w=1, h=1, d=1, **_):
    x, y, z = w / 2, h / 2, d / 2
    v = torch.tensor([[-x, -y, -z], [x, -y, -z], [x, y, -z], [-x, y, -z], [-x, -y, z], [x, -y, z], [x, y, z], [-x, y, z]])
    f = [(0, 2, 1), (0, 3, 2), (4, 5, 6), (4, 6, 7), (0, 1, 5), (0, 5, 4), (3, 6, 2), (3, 7, 6), (1, 2, 6), (1, 6, 5),
         (0, 4, 7), (0, 7, 3)]
    return v, torch.tensor(f)


def _grid_faces(rows: int, cols: int, offset: int = 0):
    """Two triangles per cell of a (rows + 1) x (cols + 1) vertex grid stored row by row."""
    faces = []
    w = cols + 1
    for r in range(rows):
        for c in range(cols):
            a, b = offset + r * w + c, offset + r * w + c + 1
            d, e = a + w, b + w
            faces += [(a, d, b), (b, d, e)]
    return faces


def _lathe(profile: List[Tuple[float, float]], seg: int, phiStart: float = 0.0, phiLength: float = 2 * math.pi):
    """Surface of revolution around y of a profile [(radius, y)], over azimuths phiStart .. phiStart + phiLength
    (x = r sin(phi), z = r cos(phi), as three.js's LatheGeometry)."""
    seg = max(1, int(seg))
    verts = []
    for (r, y) in profile:
        for i in range(seg + 1):
            a = phiStart + phiLength * i / seg
            verts.append((r * math.sin(a), y, r * math.cos(a)))
    faces = _grid_faces(len(profile) - 1, seg)
    return torch.tensor(verts, dtype=torch.float32), torch.tensor(faces, dtype=torch.long).view(-1, 3)


def _sphere(radius=1, widthSegments=24, heightSegments=12, phiStart=0.0, phiLength=2 * math.pi, thetaStart=0.0,
            thetaLength=math.pi, **_):
    """A sphere patch: polar angle theta from +y over thetaStart .. +thetaLength, azimuth phi over phiStart ..
    +phiLength (three.js's SphereGeometry: x = -r cos(phi) sin(theta), y = r cos(theta), z = r sin(phi) sin(theta))."""
    W, H = max(3, int(widthSegments)), max(2, int(heightSegments))
    verts = []
    for iy in range(H + 1):
        th = thetaStart + thetaLength * iy / H
        for ix in range(W + 1):
            ph = phiStart + phiLength * ix / W
            verts.append((-radius * math.cos(ph) * math.sin(th), radius * math.cos(th),
                          radius * math.sin(ph) * math.sin(th)))
    return torch.tensor(verts, dtype=torch.float32), torch.tensor(_grid_faces(H, W), dtype=torch.long).view(-1, 3)


def _cylinder(radiusTop=1, radiusBottom=1, height=1, radialSegments=24, heightSegments=1, openEnded=False,
              thetaStart=0.0, thetaLength=2 * math.pi, **_):
    """A (truncated) cone's side over thetaStart .. +thetaLength (x = r sin(theta), z = r cos(theta)), radius
    interpolated from the top (+height/2) to the bottom, plus the two caps unless openEnded."""
    R, Hs = max(3, int(radialSegments)), max(1, int(heightSegments))
    h = height / 2
    verts = []
    for iy in range(Hs + 1):
        v = iy / Hs
        r = radiusTop + (radiusBottom - radiusTop) * v
        y = h - height * v
        for ix in range(R + 1):
            t = thetaStart + thetaLength * ix / R
            verts.append((r * math.sin(t), y, r * math.cos(t)))
    faces = _grid_faces(Hs, R)
    if not openEnded:
        for r, y in ((radiusTop, h), (radiusBottom, -h)):
            if r <= 0:
                continue
            c = len(verts)
            verts.append((0.0, y, 0.0))
            for ix in range(R + 1):
                t = thetaStart + thetaLength * ix / R
                verts.append((r * math.sin(t), y, r * math.cos(t)))
            faces += [(c, c + 1 + ix, c + 2 + ix) for ix in range(R)]
    return torch.tensor(verts, dtype=torch.float32), torch.tensor(faces, dtype=torch.long).view(-1, 3)


def _cone(radius=1, height=1, radialSegments=24, heightSegments=1, openEnded=False, thetaStart=0.0,
          thetaLength=2 * math.pi, **_):
    return _cylinder(0.0, radius, height, radialSegments, heightSegments, openEnded, thetaStart, thetaLength)


def _plane(width=1, height=1, **_):
    x, y = width / 2, height / 2
    return torch.tensor([[-x, -y, 0], [x, -y, 0], [x, y, 0], [-x, y, 0]], dtype=torch.float32), torch.tensor([(0, 1, 2), (0, 2, 3)])


def _torus(radius=1, tube=0.4, radialSegments=12, tubularSegments=32, arc=2 * math.pi, **_):
    """A torus in the xy plane around z, swept over 0 .. arc (three.js's TorusGeometry)."""
    R, T = max(2, int(radialSegments)), max(3, int(tubularSegments))
    verts = []
    for j in range(R + 1):
        v = 2 * math.pi * j / R
        for i in range(T + 1):
            u = arc * i / T
            verts.append(((radius + tube * math.cos(v)) * math.cos(u), (radius + tube * math.cos(v)) * math.sin(u),
                          tube * math.sin(v)))
    return torch.tensor(verts, dtype=torch.float32), torch.tensor(_grid_faces(R, T), dtype=torch.long).view(-1, 3)


_PRIMS = {"BoxGeometry": _box, "SphereGeometry": _sphere, "CylinderGeometry": _cylinder, "ConeGeometry": _cone,
          "PlaneGeometry": _plane, "TorusGeometry": _torus}


def _geometry(g: dict):
    t = g.get("type")
    if t in _PRIMS:
        params = {k: v for k, v in g.items() if k not in ("type", "uuid")}
        return _PRIMS[t](**params)
    if t == "BufferGeometry":
        data = g["data"]
        pos = torch.tensor(data["attributes"]["position"]["array"], dtype=torch.float32).view(-1, 3)
        if data.get("index"):
            idx = torch.tensor(data["index"]["array"]).view(-1, 3)
        else:
            idx = torch.arange(pos.shape[0]).view(-1, 3)
        return pos, idx
    raise ValueError(f"unsupported geometry type {t!r}")


def scene_triangles(scene: dict, with_materials: bool = False):
    """-> (triangles [T, 3, 3] world space, colours [T, 3] linear RGB[, materials [T, 2] (roughness,
    metalness)]); materials default to the standard material's roughness 1, metalness 0."""
    geoms = {g["uuid"]: g for g in scene.get("geometries", [])}
    mats = {m["uuid"]: m for m in scene.get("materials", [])}
    cache: Dict[str, tuple] = {}
    tris, cols, pbr = [], [], []

    def walk(node, parent):
        m = torch.tensor(node.get("matrix", [1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1]), dtype=torch.float32)
        world = parent @ m.view(4, 4).t()            # three.js matrices are column-major
        gid = node.get("geometry")
        if gid is not None and gid in geoms:
            if gid not in cache:
                cache[gid] = _geometry(geoms[gid])
            v, f = cache[gid]
            vh = torch.cat([v, torch.ones(v.shape[0], 1)], 1) @ world.t()
            tris.append(vh[:, :3][f])
            md = mats.get(node.get("material"), {})
            c = md.get("color", 0xCCCCCC)
            rgb = torch.tensor([(c >> 16) & 255, (c >> 8) & 255, c & 255], dtype=torch.float32) / 255.0
            lin = rgb ** 2.2                                    # sRGB material colour -> linear
            if md.get("mapMean") is not None:                  # a texture map tints by its mean texel colour
                lin = lin * torch.tensor(md["mapMean"], dtype=torch.float32)
            vcol = geoms[gid]["data"]["attributes"].get("color") if "data" in geoms[gid] else None
            if md.get("vertexColors") and vcol is not None:
                # vertex colours are linear; a triangle takes the mean of its corners, times the material colour
                per_v = torch.tensor(vcol["array"], dtype=torch.float32).view(-1, 3)
                cols.append(per_v[f].mean(1).clamp(0, 1) * lin)
            else:
                cols.append(lin.expand(f.shape[0], 3))
            md = mats.get(node.get("material"), {})
            pbr.append(torch.tensor([float(md.get("roughness", 1.0)), float(md.get("metalness", 0.0))]).expand(
                f.shape[0], 2))
        for ch in node.get("children", []):
            walk(ch, world)

    walk(scene.get("object", {}), torch.eye(4))
    if not tris:
        empty = (torch.zeros(0, 3, 3), torch.zeros(0, 3))
        return empty + (torch.zeros(0, 2),) if with_materials else empty
    out = (torch.cat(tris), torch.cat(cols))
    return out + (torch.cat(pbr),) if with_materials else out


def normalise(tris: torch.Tensor) -> torch.Tensor:
    """Centre on the bounding box and scale the largest extent to 1 (the reference frames views this way)."""
    if tris.numel() == 0:
        return tris
    p = tris.reshape(-1, 3)
    lo, hi = p.min(0).values, p.max(0).values
    return (tris - (lo + hi) / 2) / float((hi - lo).max().clamp(min=1e-6))


def view_projection(azimuth_deg: float, elevation_deg: float, radius: float = 2.0, fov_deg: float = 49.1,
                    aspect: float = 1.0, near: float = 0.05, far: float = 20.0) -> torch.Tensor:
    az, el = math.radians(azimuth_deg), math.radians(elevation_deg)
    eye = torch.tensor([radius * math.cos(el) * math.sin(az), radius * math.sin(el), radius * math.cos(el) * math.cos(az)])
    f = -eye / eye.norm()
    up = torch.tensor([0.0, 1.0, 0.0])
    s = torch.linalg.cross(f, up)
    s = s / s.norm().clamp(min=1e-6)
    u = torch.linalg.cross(s, f)
    view = torch.eye(4)
    view[0, :3], view[1, :3], view[2, :3] = s, u, -f
    view[:3, 3] = torch.stack([-(s @ eye), -(u @ eye), f @ eye])
    t = 1.0 / math.tan(math.radians(fov_deg) / 2)
    proj = torch.zeros(4, 4)
    proj[0, 0], proj[1, 1] = t / aspect, t
    # view space looks down -z; depth in [0, 1] over [near, far], w = -z
    proj[2, 2] = -far / (far - near)
    proj[2, 3] = -far * near / (far - near)
    proj[3, 2] = -1.0
    return proj @ view


def render(tris: torch.Tensor, cols: torch.Tensor, vp: torch.Tensor, size: int = 256, light=(0.4, 0.8, 0.6),
           ambient: float = 0.35, diffuse: float = 0.9, exposure: float = 1.0, background=(1.0, 1.0, 1.0)) -> torch.Tensor:
    """-> RGBA uint8 [size, size, 4]; CUDA tensors use the GPU rasterizer, CPU tensors its C++ restatement."""
    return ops.ext().raster(tris.float().contiguous(), cols.float().contiguous(), vp.float(), size, size, list(light),
                            ambient, diffuse, exposure, list(background))


# Light rigs for raster_pbr (csrc/raster.cu): lights (direction towards the light, intensity, follows the
# camera), ambient, hemisphere environment (sky, ground linear RGB, intensity). Modelled on the reference's
# page rigs (render_service/object-page.html:37-110): "studio" = key / fill / rim lights over a white-to-grey
# hemisphere, "neutral" = a camera-following key light in a grey room with a bright ceiling, "follow" = ambient +
# a camera-following light.
LIGHTING = {
    "studio": {"lights": [(2, 3, 2, 1.2, 0), (-2, 1, 1, 0.4, 0), (0, 2, -3, 0.3, 0)], "ambient": 0.12,
               "hemi": (1.0, 1.0, 1.0, 0.058, 0.058, 0.058, 0.8)},
    "neutral": {"lights": [(0, 0, 1, 1.1, 1)], "ambient": 0.0, "hemi": (1.2, 1.2, 1.2, 0.32, 0.32, 0.32, 0.9)},
    "follow": {"lights": [(0, 0, 1, 1.5, 1)], "ambient": 0.4, "hemi": (0, 0, 0, 0, 0, 0, 0.0)},
}


def camera_eye(azimuth_deg: float, elevation_deg: float, radius: float = 2.0) -> List[float]:
    az, el = math.radians(azimuth_deg), math.radians(elevation_deg)
    return [radius * math.cos(el) * math.sin(az), radius * math.sin(el), radius * math.cos(el) * math.cos(az)]


def render_pbr(tris: torch.Tensor, cols: torch.Tensor, mats: Optional[torch.Tensor], azimuth_deg: float,
               elevation_deg: float, size: int = 256, lighting: str = "studio", exposure: float = 1.0,
               background=(1.0, 1.0, 1.0)) -> torch.Tensor:
    """Standard-material render (GGX + hemisphere environment) of one view -> RGBA uint8 [size, size, 4]; CUDA
    tensors use the GPU kernel, CPU tensors its C++ restatement."""
    rig = LIGHTING[lighting]
    lights = torch.tensor(rig["lights"], dtype=torch.float32).view(-1, 5)
    m = mats.float().contiguous() if mats is not None else torch.zeros(0, 2, device=tris.device)
    return ops.ext().raster_pbr(tris.float().contiguous(), cols.float().contiguous(), m,
                                view_projection(azimuth_deg, elevation_deg), camera_eye(azimuth_deg, elevation_deg),
                                lights, float(rig["ambient"]), list(rig["hemi"]), exposure, list(background), size, size)


VIEW_PRESETS = {"front4": [(0, 15), (45, 15), (-45, 15), (90, 15)],
                "judge": [(0, 15), (45, 25), (-45, 25), (90, 15), (180, 15), (0, 60)]}


def render_views(scene: dict, preset: str = "front4", size: int = 256, device="cpu") -> List[torch.Tensor]:
    tris, cols = scene_triangles(scene)
    tris = normalise(tris).to(device)
    cols = cols.to(device)
    return [render(tris, cols, view_projection(a, e), size) for a, e in VIEW_PRESETS[preset]]
