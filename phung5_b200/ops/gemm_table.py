"""Per-shape GEMM configuration table (measured by phung5_b200/bench/gemm_table.py, stored as gemm_table.json).

An entry maps (kind, N, K, M bucket) to the tile configuration that measured fastest: BN (128 / 256), and for
fp8 whether the tensor core applies the block scales (hardware scaling) or the epilogue promotes per K block,
and whether 256 x 256 tiles run on CTA pairs. M is bucketed to the nearest measured size at or above it (the
largest bucket beyond). Missing entries (or a missing file) leave the kernel's own heuristic in charge.
PHX_GEMM_TABLE=0 disables the table.
"""
from __future__ import annotations

import json
import os
from typing import Optional

PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "gemm_table.json")
_TABLE = {"loaded": False, "entries": {}, "buckets": []}
ENABLED = os.environ.get("PHX_GEMM_TABLE", "1") != "0"


def _bucket(m: int, buckets) -> int:
    for b in buckets:
        if m <= b:
            return b
    return buckets[-1] if buckets else m


def key(kind: str, n: int, k: int, m: int, buckets=None) -> str:
    bs = buckets if buckets is not None else (_TABLE["buckets"] or [m])
    return f"{kind}:{n}:{k}:{_bucket(m, bs)}"


def _load() -> None:
    _TABLE["loaded"] = True
    if not os.path.exists(PATH):
        return
    with open(PATH) as f:
        t = json.load(f)
    _TABLE["entries"] = t.get("entries", {})
    _TABLE["buckets"] = sorted(t.get("m_buckets", []))


def lookup(kind: str, n: int, k: int, m: int) -> Optional[dict]:
    """-> {"bn": ..., ["hws": ..., "pair": ...]} or None (use the kernel's default)."""
    if not ENABLED:
        return None
    if not _TABLE["loaded"]:
        _load()
    if not _TABLE["entries"]:
        return None
    e = _TABLE["entries"].get(key(kind, n, k, m))
    if not e or "bn" not in e:
        return None
    return e
