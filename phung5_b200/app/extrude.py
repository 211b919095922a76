"""Shape triangulation and extrusion with holes and bevels (the geometry of three.js's ShapeGeometry and
ExtrudeGeometry, built here for the module interpreter's renders and vertex counts).

- Caps: a shape's holes are bridged into its outline (each hole, rightmost first, is joined to the outline by a
  cut from its rightmost vertex to the outline vertex that a ray toward +x reaches first), and the resulting
  single polygon is ear-clipped.
- Extrusion along +z over [0, depth], with three.js's bevel when enabled (its default): `bevelSegments` rings
  on each side between z = -bevelThickness and 0 (and depth .. depth + bevelThickness), the outline pushed out
  by bevelSize * sin(t * pi / 2) + bevelOffset along each vertex's miter direction (holes shrink by the same
  rule), the body at the full bevelSize + bevelOffset, the caps at the bevelOffset outline.
"""
from __future__ import annotations

import math
from typing import Dict, List, Sequence, Tuple

Pt = Tuple[float, float]


def signed_area(poly: Sequence[Pt]) -> float:
    return 0.5 * sum(poly[i][0] * poly[(i + 1) % len(poly)][1] - poly[(i + 1) % len(poly)][0] * poly[i][1]
                     for i in range(len(poly)))


def clean(poly: Sequence[Sequence[float]]) -> List[Pt]:
    """Drop repeated consecutive points and a closing copy of the first point."""
    out: List[Pt] = []
    for p in poly:
        q = (float(p[0]), float(p[1]))
        if not out or abs(q[0] - out[-1][0]) + abs(q[1] - out[-1][1]) > 1e-12:
            out.append(q)
    if len(out) > 1 and abs(out[0][0] - out[-1][0]) + abs(out[0][1] - out[-1][1]) <= 1e-12:
        out.pop()
    return out


def _cross(o: Pt, a: Pt, b: Pt) -> float:
    return (a[0] - o[0]) * (b[1] - o[1]) - (a[1] - o[1]) * (b[0] - o[0])


def _in_tri(p: Pt, a: Pt, b: Pt, c: Pt) -> bool:
    d1, d2, d3 = _cross(a, b, p), _cross(b, c, p), _cross(c, a, p)
    return not ((d1 < 0 or d2 < 0 or d3 < 0) and (d1 > 0 or d2 > 0 or d3 > 0))


def ear_clip(poly: Sequence[Pt]) -> List[Tuple[int, int, int]]:
    """Triangles (indices into poly, counter-clockwise) of a simple polygon given counter-clockwise; falls back to
    a fan when no ear is found (degenerate input)."""
    idx = list(range(len(poly)))
    out: List[Tuple[int, int, int]] = []
    guard = 0
    while len(idx) > 3 and guard < 4 * len(poly) + 16:
        guard += 1
        found = False
        for k in range(len(idx)):
            i0, i1, i2 = idx[k - 1], idx[k], idx[(k + 1) % len(idx)]
            a, b, c = poly[i0], poly[i1], poly[i2]
            if _cross(a, b, c) <= 1e-15:
                continue
            if any(_in_tri(poly[j], a, b, c) for j in idx if j not in (i0, i1, i2) and poly[j] not in (a, b, c)):
                continue
            out.append((i0, i1, i2))
            idx.pop(k)
            found = True
            break
        if not found:
            break
    for k in range(1, len(idx) - 1):
        out.append((idx[0], idx[k], idx[k + 1]))
    return out


def bridge_holes(outer: List[Pt], holes: List[List[Pt]]) -> List[Pt]:
    """One simple polygon from a counter-clockwise outline and clockwise holes."""
    poly = list(outer)
    for hole in sorted(holes, key=lambda h: -max(p[0] for p in h)):
        hi = max(range(len(hole)), key=lambda i: (hole[i][0], -hole[i][1]))
        hx, hy = hole[hi]
        best, best_x = None, math.inf
        for i in range(len(poly)):
            a, b = poly[i], poly[(i + 1) % len(poly)]
            if (a[1] - hy) * (b[1] - hy) > 0 or a[1] == b[1]:
                continue
            x = a[0] + (hy - a[1]) * (b[0] - a[0]) / (b[1] - a[1])
            if hx <= x < best_x:
                best_x = x
                best = i if a[0] >= b[0] else (i + 1) % len(poly)
        if best is None:
            best = min(range(len(poly)), key=lambda i: (poly[i][0] - hx) ** 2 + (poly[i][1] - hy) ** 2)
        ring = hole[hi:] + hole[:hi] + [hole[hi]]
        poly = poly[:best + 1] + ring + [poly[best]] + poly[best + 1:]
    return poly


def triangulate(outer: Sequence[Sequence[float]], holes: Sequence[Sequence[Sequence[float]]] = ()
                ) -> Tuple[List[Pt], List[Tuple[int, int, int]]]:
    """(vertices, triangles) of a shape with holes, counter-clockwise as seen from +z."""
    o = clean(outer)
    if len(o) < 3:
        return o, []
    if signed_area(o) < 0:
        o = o[::-1]
    hs = []
    for h in holes:
        h = clean(h)
        if len(h) >= 3:
            hs.append(h[::-1] if signed_area(h) > 0 else h)
    poly = bridge_holes(o, hs) if hs else o
    return poly, ear_clip(poly)


def miter(poly: List[Pt]) -> List[Pt]:
    """Per-vertex offset directions that move every edge of a counter-clockwise ring outward by one unit (clockwise
    rings, the holes, move inward: away from the solid either way)."""
    n = len(poly)
    out = []
    for i in range(n):
        p0, p1, p2 = poly[i - 1], poly[i], poly[(i + 1) % n]
        e1 = (p1[0] - p0[0], p1[1] - p0[1])
        e2 = (p2[0] - p1[0], p2[1] - p1[1])
        l1, l2 = math.hypot(*e1) or 1.0, math.hypot(*e2) or 1.0
        n1 = (e1[1] / l1, -e1[0] / l1)
        n2 = (e2[1] / l2, -e2[0] / l2)
        d = 1.0 + n1[0] * n2[0] + n1[1] * n2[1]
        if d < 1e-6:
            out.append(n1)
        else:
            m = ((n1[0] + n2[0]) / d, (n1[1] + n2[1]) / d)
            k = math.hypot(*m)
            if k > 4.0:                     # a very sharp corner: cap the miter length
                m = (m[0] * 4.0 / k, m[1] * 4.0 / k)
            out.append(m)
    return out


def extrude(outer, holes=(), depth: float = 1.0, bevel: bool = True, thickness: float = 0.2,
            size: float = 0.1, offset: float = 0.0, segments: int = 3):
    """(vertices [(x, y, z)], triangles) of an extruded shape; depth 0 and no bevel gives the flat shape."""
    o = clean(outer)
    if len(o) < 3:
        return [], []
    if signed_area(o) < 0:
        o = o[::-1]
    hs = []
    for h in holes:
        h = clean(h)
        if len(h) >= 3:
            hs.append(h[::-1] if signed_area(h) > 0 else h)
    rings = [o] + hs
    moves = [miter(r) for r in rings]
    segments = max(1, int(segments))
    if not bevel:
        thickness = size = offset = 0.0
    # rings of the side surface, front to back: (z, outward push)
    layers: List[Tuple[float, float]] = []
    if bevel and thickness > 0:
        for b in range(segments):
            t = b / segments
            layers.append((-thickness * math.cos(t * math.pi / 2), size * math.sin(t * math.pi / 2) + offset))
    layers.append((0.0, size + offset))
    if depth > 0:
        layers.append((depth, size + offset))
    if bevel and thickness > 0:
        for b in range(segments - 1, -1, -1):
            t = b / segments
            layers.append((depth + thickness * math.cos(t * math.pi / 2), size * math.sin(t * math.pi / 2) + offset))
    verts: List[Tuple[float, float, float]] = []
    faces: List[Tuple[int, int, int]] = []

    def ring_at(r: int, z: float, push: float) -> int:
        base = len(verts)
        for (x, y), (mx, my) in zip(rings[r], moves[r]):
            verts.append((x + mx * push, y + my * push, z))
        return base

    # caps at the front and back layers (the bevel's starting outline)
    cap_rings = [[(x + mx * layers[0][1], y + my * layers[0][1]) for (x, y), (mx, my) in zip(rings[r], moves[r])]
                 for r in range(len(rings))]
    poly = bridge_holes(cap_rings[0], cap_rings[1:]) if len(cap_rings) > 1 else cap_rings[0]
    tris = ear_clip(poly)
    lookup: Dict[Pt, int] = {}
    # two caps facing out of the solid; a flat shape (one layer) is a single face toward +z with no side walls
    caps = ((layers[0][0], False), (layers[-1][0], True)) if len(layers) > 1 else ((layers[0][0], True),)
    for zc, back in caps:
        lookup = {}
        idx = []
        for p in poly:
            if p not in lookup:
                lookup[p] = len(verts)
                verts.append((p[0], p[1], zc))
            idx.append(lookup[p])
        for a, b, c in tris:
            faces.append((idx[a], idx[b], idx[c]) if back else (idx[c], idx[b], idx[a]))
    if len(layers) == 1:
        return verts, faces
    # side walls between consecutive layers, for the outline and every hole
    for r in range(len(rings)):
        n = len(rings[r])
        prev = None
        for z, push in layers:
            cur = ring_at(r, z, push)
            if prev is not None:
                for i in range(n):
                    j = (i + 1) % n
                    faces += [(prev + i, prev + j, cur + j), (prev + i, cur + j, cur + i)]
            prev = cur
    return verts, faces
