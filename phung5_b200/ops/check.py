"""Bounds-check debug mode of the native ops (PHX_CHECK_BOUNDS=1, or `with bounds_checks():`).

The C++ bindings check shapes, dtypes and strides before a launch, but not the VALUES of the index data that
drives the kernels' loads and stores (page tables, KV slots, positions, work lists, expert offsets, tree parents):
a wrong value there is an out-of-range access on the device, or two CTAs writing the same rows (a race that
shows as nondeterministic output). In this mode every op validates that data on the host before it launches:

- every index lies inside the buffer it addresses (the first bad element is named in the error);
- no two writers share a target: KV slots written by one `rope_kv_write` are distinct, and the query rows of
  one attention pass's work items are disjoint, as are its (item, first row) tiles;
- the TMA operands of the GEMMs start on 16-byte boundaries with 16-byte multiple row strides, and the scales
  handed to the hardware block-scaled path are powers of two.

The checks read device tensors back (a synchronisation per op), so they are for small-shape debug runs (the
kernel self-test, the test suite), not for serving. Inside a CUDA graph capture they are skipped (nothing may
synchronise there): run the eager step to check the captured one, which launches the same kernels on the same
data. Both the CUDA ops and their CPU definitions are checked, so CPU runs of the engine exercise every rule.
"""
from __future__ import annotations

import contextlib
import os
from typing import Optional, Sequence

import torch

ON = [os.environ.get("PHX_CHECK_BOUNDS", "0") == "1"]
CHECKS = [0]          # number of op calls validated so far


class BoundsError(ValueError):
    """Index data or operand layout that would make a kernel access memory outside its buffers or race."""


@contextlib.contextmanager
def bounds_checks(on: bool = True):
    old = ON[0]
    ON[0] = on
    try:
        yield
    finally:
        ON[0] = old


def active() -> bool:
    if not ON[0]:
        return False
    if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
        return False
    CHECKS[0] += 1
    return True


def _fail(op: str, what: str) -> None:
    raise BoundsError(f"{op}: {what}")


def _range(op: str, name: str, t: torch.Tensor, lo: int, hi: int, allow: Optional[int] = None) -> None:
    """All values of t in [lo, hi) (values equal to `allow` are accepted as well); names the first bad one."""
    if t is None or t.numel() == 0:
        return
    v = t.reshape(-1).long()
    bad = (v < lo) | (v >= hi)
    if allow is not None:
        bad &= v != allow
    if bool(bad.any()):
        i = int(bad.nonzero()[0, 0])
        ok = f"[{lo}, {hi})" + (f" or {allow}" if allow is not None else "")
        _fail(op, f"{name}[{i}] = {int(v[i])} outside {ok}")


def _distinct(op: str, name: str, t: torch.Tensor) -> None:
    if t is None or t.numel() < 2:
        return
    s, _ = t.reshape(-1).long().sort()
    dup = s[1:] == s[:-1]
    if bool(dup.any()):
        i = int(dup.nonzero()[0, 0])
        _fail(op, f"{name} value {int(s[i])} appears more than once (two writers of one target)")


def _nondecreasing(op: str, name: str, t: torch.Tensor) -> None:
    v = t.reshape(-1).long()
    if v.numel() > 1 and bool((v[1:] < v[:-1]).any()):
        i = int((v[1:] < v[:-1]).nonzero()[0, 0])
        _fail(op, f"{name} decreases at {i + 1}: {int(v[i])} -> {int(v[i + 1])}")


def _tma(op: str, name: str, t: torch.Tensor) -> None:
    """A TMA operand: 16-byte aligned base, unit inner stride, row stride a multiple of 16 bytes."""
    if t is None or not t.is_cuda:
        return
    if t.data_ptr() % 16:
        _fail(op, f"{name} starts at {t.data_ptr():#x}, not on a 16-byte boundary")
    if t.dim() >= 2 and (t.stride(-1) != 1 or (t.stride(-2) * t.element_size()) % 16):
        _fail(op, f"{name} strides {tuple(t.stride())} ({t.element_size()}-byte elements): a row must be "
                  f"contiguous and start on a 16-byte boundary")


def _shape(op: str, name: str, t: torch.Tensor, shape: Sequence[int]) -> None:
    if t is not None and tuple(t.shape) != tuple(shape):
        _fail(op, f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")


def _pow2(op: str, name: str, s: torch.Tensor) -> None:
    if s is None or s.numel() == 0:
        return
    f = s.float().reshape(-1)
    m, _ = torch.frexp(f)
    bad = ~torch.isfinite(f) | (f <= 0) | (m != 0.5)
    if bool(bad.any()):
        i = int(bad.nonzero()[0, 0])
        _fail(op, f"{name}[{i}] = {float(f[i])!r} is not a positive power of two (hardware block scaling)")


# ------------------------------------------------------------------------------------------------
# per-op rules
# ------------------------------------------------------------------------------------------------

def gemm_fp8_block(xq, xs, wq, ws, out, hws: bool) -> None:
    op = "gemm_fp8_block"
    m, k = xq.shape
    n = wq.shape[0]
    if k % 128:
        _fail(op, f"K = {k} is not a multiple of the 128-wide scale block")
    _shape(op, "xs", xs, (k // 128, m))
    _shape(op, "wq", wq, (n, k))
    _shape(op, "ws", ws, ((n + 127) // 128, k // 128))
    _shape(op, "out", out, (m, n))
    for name, t in (("xq", xq), ("wq", wq), ("out", out)):
        _tma(op, name, t)
    if hws:
        _pow2(op, "xs", xs)
        _pow2(op, "ws", ws)


def gemm_bf16(x, w, out) -> None:
    op = "gemm_bf16"
    m, k = x.shape
    if w.shape[1] != k:
        _fail(op, f"x has K = {k}, w has K = {w.shape[1]}")
    _shape(op, "out", out, (m, w.shape[0]))
    for name, t in (("x", x), ("w", w), ("out", out)):
        _tma(op, name, t)


def gemm_grouped(x_rows: int, w, n: int, offsets, rows) -> None:
    op = "gemm_grouped"
    if n <= 0 or w.shape[0] % n:
        _fail(op, f"weight rows {w.shape[0]} are not a multiple of the group width n = {n}")
    g = w.shape[0] // n
    if offsets.numel() != g + 1:
        _fail(op, f"offsets has {offsets.numel()} entries for {g} groups (need {g + 1})")
    m = x_rows if rows is None else rows.numel()
    _range(op, "offsets", offsets, 0, m + 1)
    _nondecreasing(op, "offsets", offsets)
    if rows is not None:
        _range(op, "rows", rows, 0, x_rows)


def moe_combine(y, pos, w, local, out) -> None:
    op = "moe_combine"
    if pos.shape != w.shape or pos.shape != local.shape:
        _fail(op, f"pos {tuple(pos.shape)}, w {tuple(w.shape)} and local {tuple(local.shape)} differ")
    if out.shape[0] != pos.shape[0]:
        _fail(op, f"out has {out.shape[0]} rows for {pos.shape[0]} tokens")
    _range(op, "pos (local entries)", pos[local.bool()], 0, y.shape[0])


def topk_logprobs(logits, k: int, temperature: float) -> None:
    op = "topk_logprobs"
    if not 1 <= k <= min(16, logits.shape[-1]):
        _fail(op, f"k = {k} outside [1, min(16, vocab {logits.shape[-1]})]")
    if not temperature > 0:
        _fail(op, f"temperature {temperature} must be > 0 (k = 1 for greedy)")


def spec_sample_accept(logits, tokens, parent, top_k, temp, depth: int, kc: int, vocab_offset: int) -> None:
    op = "spec_sample_accept"
    R, N = tokens.shape
    if logits.shape[0] != R * N:
        _fail(op, f"{logits.shape[0]} logits rows for {R} requests x {N} nodes")
    if not 0 <= depth < N:
        _fail(op, f"depth {depth} outside [0, {N})")
    if bool((parent[:, 0] != -1).any()):
        _fail(op, "node 0 of every tree must be its root (parent -1)")
    if N > 1:
        # a node's parent precedes it: the accept walk visits nodes in index order
        j = torch.arange(1, N, device=parent.device)
        bad = (parent[:, 1:] < 0) | (parent[:, 1:] >= j[None, :])
        if bool(bad.any()):
            r, c = (int(x) for x in bad.nonzero()[0])
            _fail(op, f"parent[{r}, {c + 1}] = {int(parent[r, c + 1])} is not an earlier node")
    sampled = temp.float() > 0
    _range(op, "top_k (sampled requests)", top_k[sampled], 1, kc + 1)
    _range(op, "tokens (drafts)", tokens[:, 1:], 0, 1 << 31)


def rope_kv_write(qkv, pos, slots, cos_sin, k_cache, hq: int, hkv: int, d: int) -> None:
    op = "rope_kv_write"
    m = qkv.shape[0]
    if qkv.shape[1] != (hq + 2 * hkv) * d:
        _fail(op, f"qkv width {qkv.shape[1]} != (hq + 2 hkv) d = {(hq + 2 * hkv) * d}")
    if pos.numel() != m:
        _fail(op, f"{pos.numel()} positions for {m} rows")
    _range(op, "pos", pos, 0, cos_sin.shape[0])
    if slots is not None and k_cache is not None:
        if slots.numel() != m:
            _fail(op, f"{slots.numel()} slots for {m} rows")
        cap = k_cache.shape[0] * k_cache.shape[2]
        _range(op, "slots", slots, 0, cap, allow=-1)
        _distinct(op, "slots", slots[slots >= 0])


def attention(q, k_cache, meta, items, tiles, group_size: int, rows: int) -> None:
    """One attention pass: page tables, key ranges, work items and (if given) tiles (engine/attn_meta.py
    layout: item = [q0, qn, table_req, kv_lo, kv_hi, mask_req]; tile = (item, first row of its qn x group rows))."""
    op = "paged_attention"
    ps = k_cache.shape[2]
    n_pages = k_cache.shape[0]
    T = q.shape[0]
    R = meta.page_indptr.numel() - 1
    ip = meta.page_indptr.long().cpu()
    _nondecreasing(op, "page_indptr", ip)
    if int(ip[0]) != 0 or int(ip[-1]) > meta.pages.numel():
        _fail(op, f"page_indptr spans [{int(ip[0])}, {int(ip[-1])}) of {meta.pages.numel()} page entries")
    _range(op, "pages", meta.pages[: int(ip[-1])], 0, n_pages)
    cap = (ip[1:] - ip[:-1]) * ps            # keys that request r's page list can hold
    qs = meta.q_start.long().cpu()
    _nondecreasing(op, "q_start", qs)
    if int(qs[-1]) > T:
        _fail(op, f"q_start ends at {int(qs[-1])} beyond {T} query rows")
    plen = meta.prefix_len.long().cpu()
    it = (items.long().cpu() if isinstance(items, torch.Tensor) else torch.tensor(items, dtype=torch.long)).reshape(-1, 6)
    live = []
    for i, (q0, qn, treq, lo, hi, mreq) in enumerate(it.tolist()):
        if qn == 0:
            continue
        if q0 < 0 or q0 + qn > T:
            _fail(op, f"item {i} rows [{q0}, {q0 + qn}) outside [0, {T})")
        if not 0 <= treq < R:
            _fail(op, f"item {i} page table of request {treq} outside [0, {R})")
        if not 0 <= lo <= hi <= int(cap[treq]):
            _fail(op, f"item {i} keys [{lo}, {hi}) outside request {treq}'s {int(cap[treq]) // ps} pages "
                      f"of {ps} keys")
        if not -1 <= mreq < R:
            _fail(op, f"item {i} mask request {mreq} outside [-1, {R})")
        if mreq >= 0:
            a, b = int(qs[mreq]), int(qs[mreq + 1])
            if q0 < a or q0 + qn > b:
                _fail(op, f"item {i} rows [{q0}, {q0 + qn}) are not request {mreq}'s rows [{a}, {b})")
            if not meta.causal:
                if meta.tree is None:
                    _fail(op, f"item {i} needs the tree ancestor masks (non-causal pass with a mask request)")
                if hi - int(plen[mreq]) > 64:
                    _fail(op, f"item {i}: {hi - int(plen[mreq])} tree keys exceed the 64-bit ancestor mask")
        live.append((q0, q0 + qn, i))
    live.sort()
    for (a0, a1, i), (b0, b1, j) in zip(live, live[1:]):
        if b0 < a1:
            _fail(op, f"items {i} and {j} both write query rows [{b0}, {min(a1, b1)}) (race)")
    if tiles is None:
        return
    ti, tr, nt = tiles
    ti = ti.long().cpu()[:nt]
    tr = tr.long().cpu()[:nt]
    _range(op, "tile_item", ti, 0, it.shape[0], allow=-1)
    seen = set()
    for t, (i, r0) in enumerate(zip(ti.tolist(), tr.tolist())):
        if i < 0:
            continue
        nrows = int(it[i, 1]) * group_size
        if r0 < 0 or r0 >= max(nrows, 1) or r0 % rows:
            _fail(op, f"tile {t}: first row {r0} of item {i} is outside [0, {nrows}) or not a multiple of {rows}")
        if (i, r0) in seen:
            _fail(op, f"tile {t} repeats item {i} rows from {r0} (two CTAs writing one tile: race)")
        seen.add((i, r0))


def add_rmsnorm_quant(h, delta, w, quant: bool) -> None:
    op = "add_rmsnorm_quant"
    m, hd = h.shape
    if quant and hd % 128:
        _fail(op, f"hidden {hd} is not a multiple of the 128-wide scale block")
    if w.numel() != hd:
        _fail(op, f"weight has {w.numel()} entries for hidden {hd}")
    if delta is not None:
        _shape(op, "delta", delta, (m, hd))


def silu_mul_quant(gu, quant: bool) -> None:
    op = "silu_mul_quant"
    f2 = gu.shape[1]
    if f2 % 2 or (quant and (f2 // 2) % 128):
        _fail(op, f"[gate | up] width {f2}: each half must be a multiple of 128 for block-scaled output")
