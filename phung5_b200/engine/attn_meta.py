"""Attention metadata and work lists for the paged attention kernel (csrc/attention.cu).

A batch holds R requests; request r contributes tokens [q_start[r], q_start[r+1]) (prefill chunk,
decode token, or verify tree nodes) and owns the page list pages[page_indptr[r]:page_indptr[r+1]].
Its KV holds kv_len[r] keys: prefix_len[r] committed keys visible to all its new tokens, then the
new tokens themselves, visible causally (prefill / chain) or by the 64-bit ancestor mask (tree).

Cascade attention (the reference's verify cascade, docker/opt/v5/casc/kopt_casc.py:42-202): requests
that share the first L pages (L*64 keys, from the prefix cache) form a group. Pass 1 attends the
group's rows to the shared keys once and writes (O, LSE); pass 2 attends each request to its own
keys [L*64, kv_len) and merges in registers. Grouping is computed on the host from page-table
identity (the reference probes req_to_token at fixed depths on device, kopt_casc.py:56-79; here the
page tables are host-owned, so exact longest-common-prefix is free).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch

ROWS_PER_TILE = 64


UPLOADED_BYTES = [0]   # host->device bytes moved by upload() (reported per step by the benchmark)


def upload(data, dtype, device) -> torch.Tensor:
    """Host list / tensor -> device tensor without a stream synchronisation: CUDA destinations go through
    pinned memory with a non-blocking copy (a pageable copy would wait for all queued GPU work)."""
    t = data if isinstance(data, torch.Tensor) else torch.tensor(data, dtype=dtype)
    t = t.to(dtype)
    if torch.device(device).type == "cuda":
        UPLOADED_BYTES[0] += t.numel() * t.element_size()
        return t.pin_memory().to(device, non_blocking=True)
    return t.to(device)


@dataclass
class AttnMeta:
    pages: torch.Tensor          # int32 [sum pages]
    page_indptr: torch.Tensor    # int32 [R+1]
    prefix_len: torch.Tensor     # int32 [R]
    kv_len: torch.Tensor         # int32 [R]
    q_start: torch.Tensor        # int32 [R+1]
    tree: Optional[torch.Tensor]  # int64 [T] ancestor bitmasks, or None
    causal: bool
    # host copies used to build work lists
    h_page_indptr: List[int] = None
    h_pages: List[int] = None
    h_prefix_len: List[int] = None
    h_kv_len: List[int] = None
    h_q_start: List[int] = None

    @property
    def num_reqs(self) -> int:
        return len(self.h_kv_len)

    @property
    def num_tokens(self) -> int:
        return self.h_q_start[-1]


def make_meta(page_lists: Sequence[Sequence[int]], prefix_len: Sequence[int], q_lens: Sequence[int],
              tree: Optional[torch.Tensor], causal: bool, device) -> AttnMeta:
    indptr = [0]
    flat: List[int] = []
    for pl in page_lists:
        flat.extend(pl)
        indptr.append(len(flat))
    qs = [0]
    for n in q_lens:
        qs.append(qs[-1] + n)
    kv = [p + n for p, n in zip(prefix_len, q_lens)]
    i32 = torch.int32
    return AttnMeta(
        pages=upload(flat if flat else [0], i32, device), page_indptr=upload(indptr, i32, device),
        prefix_len=upload(list(prefix_len), i32, device), kv_len=upload(kv, i32, device),
        q_start=upload(qs, i32, device), tree=None if tree is None else upload(tree, torch.int64, device),
        causal=causal, h_page_indptr=indptr, h_pages=flat, h_prefix_len=list(prefix_len), h_kv_len=kv,
        h_q_start=qs)


def cascade_groups(meta: AttnMeta, page_size: int, min_shared_pages: int = 1, min_group: int = 2
                   ) -> List[Tuple[int, int, int]]:
    """Greedy grouping of consecutive requests by their longest common page prefix.
    Returns [(r_first, r_last, shared_keys)] with shared_keys a multiple of page_size and not beyond
    any member's committed prefix (new tokens are never in a shared page)."""
    groups = []
    r, n = 0, meta.num_reqs
    pages = meta.h_pages
    ip = meta.h_page_indptr

    def committed_pages(i):
        return meta.h_prefix_len[i] // page_size

    while r < n:
        best_end, best_len = r, 0
        lcp = committed_pages(r)
        e = r + 1
        while e < n:
            cp = min(lcp, committed_pages(e))
            k = 0
            a0, b0 = ip[r], ip[e]
            while k < cp and pages[a0 + k] == pages[b0 + k]:
                k += 1
            if k < min_shared_pages:
                break
            lcp = k
            best_end, best_len = e, k
            e += 1
        if best_end - r + 1 >= min_group and best_len >= min_shared_pages:
            groups.append((r, best_end, best_len * page_size))
            r = best_end + 1
        else:
            r += 1
    return groups


def build_items(meta: AttnMeta, group_size: int, groups: Optional[List[Tuple[int, int, int]]] = None):
    """Work lists. Returns (pass1_items or None, pass2_items); each is a list of 6-int items
    [q0, qn, table_req, kv_lo, kv_hi, mask_req]."""
    shared = [0] * meta.num_reqs
    p1 = None
    if groups:
        p1 = []
        for a, b, L in groups:
            q0, q1 = meta.h_q_start[a], meta.h_q_start[b + 1]
            p1.append([q0, q1 - q0, a, 0, L, -1])
            for r in range(a, b + 1):
                shared[r] = L
    p2 = []
    for r in range(meta.num_reqs):
        q0, q1 = meta.h_q_start[r], meta.h_q_start[r + 1]
        if q1 > q0:
            p2.append([q0, q1 - q0, r, shared[r], meta.h_kv_len[r], r])
    return p1, p2


def tiles_for(items: List[List[int]], group_size: int, rows: Optional[int] = None):
    if rows is None:
        from .. import ops
        rows = ops.attn_rows()
    ti, tr = [], []
    for i, it in enumerate(items):
        nrows = it[1] * group_size
        for r0 in range(0, nrows, rows):
            ti.append(i)
            tr.append(r0)
    return ti, tr


def pack_work(items: List[List[int]], group_size: int, device, pad_tiles: int = 0, rows: Optional[int] = None):
    ti, tr = tiles_for(items, group_size, rows)
    n = len(ti)
    if pad_tiles > n:
        ti = ti + [-1] * (pad_tiles - n)
        tr = tr + [0] * (pad_tiles - n)
    flat_items = [x for it in (items if items else [[0] * 6]) for x in it]
    ti = ti if ti else [-1]
    tr = tr if tr else [0]
    both = upload(flat_items + ti + tr, torch.int32, device)          # one copy for the three arrays
    ni, nt = len(flat_items), len(ti)
    return both[:ni].view(-1, 6), (both[ni:ni + nt], both[ni + nt:], max(n, pad_tiles))


def attention_reference(q, k_cache, v_cache, meta: AttnMeta, scale, items, o_in=None, lse_in=None, o_part=None,
                        lse_part=None, out=None, out_q=None, out_qs=None):
    """Plain-torch definition of one attention pass over a work list (fp32 math)."""
    from ..weights.quant import FP8_MAX, pow2_scale
    t_all, hq, d = q.shape
    hkv = k_cache.shape[1]
    ps = k_cache.shape[2]
    g = hq // hkv
    it_list = items.tolist() if isinstance(items, torch.Tensor) else items
    for q0, qn, treq, kv_lo, kv_hi, mreq in it_list:
        if qn == 0:
            continue
        pl = meta.h_pages[meta.h_page_indptr[treq]: meta.h_page_indptr[treq + 1]]
        keys = torch.arange(kv_lo, kv_hi)
        pg = torch.tensor(pl, dtype=torch.long)[keys // ps]
        off = keys % ps
        kk = k_cache[pg, :, off, :].float()  # [S, hkv, d]
        vv = v_cache[pg, :, off, :].float()
        qq = q[q0: q0 + qn].float()  # [n, hq, d]
        kk = kk.repeat_interleave(g, 1)
        vv = vv.repeat_interleave(g, 1)
        s = torch.einsum("nhd,shd->nhs", qq, kk) * scale
        vis = torch.ones(qn, kv_hi - kv_lo, dtype=torch.bool)
        if mreq >= 0:
            plen = meta.h_prefix_len[mreq]
            li = torch.arange(q0, q0 + qn) - meta.h_q_start[mreq]
            rel = keys[None, :] - plen
            if meta.causal:
                newvis = rel <= li[:, None]
            else:
                bits = meta.tree[q0: q0 + qn].cpu()
                relc = rel.clamp(min=0, max=63)
                newvis = ((bits[:, None] >> relc) & 1).bool()
            vis = (rel < 0) | newvis
        s = s.masked_fill(~vis[:, None, :].to(s.device), float("-inf"))
        m = s.amax(-1)
        if o_in is not None:
            lse0 = lse_in[q0: q0 + qn].float()
            m = torch.maximum(m, lse0)
        msafe = torch.where(torch.isinf(m), torch.zeros_like(m), m)
        p = torch.exp(s - msafe[..., None])
        l = p.sum(-1)
        acc = torch.einsum("nhs,shd->nhd", p, vv)
        if o_in is not None:
            w0 = torch.exp(lse0 - msafe)
            acc = acc + w0[..., None] * o_in[q0: q0 + qn].float()
            l = l + w0
        o = torch.where(l[..., None] > 0, acc / l.clamp(min=1e-30)[..., None], torch.zeros_like(acc))
        lse = torch.where(l > 0, msafe + torch.log(l.clamp(min=1e-30)), torch.full_like(l, float("-inf")))
        if o_part is not None:
            o_part[q0: q0 + qn] = o.to(o_part.dtype)
            lse_part[q0: q0 + qn] = lse
        if out is not None:
            out.view(t_all, hq, d)[q0: q0 + qn] = o.to(out.dtype)
        if out_q is not None:
            amax = o.abs().amax(-1)
            sc = pow2_scale(amax)
            out_q.view(t_all, hq, d)[q0: q0 + qn] = (o / sc[..., None]).clamp(-FP8_MAX, FP8_MAX).to(out_q.dtype)
            out_qs[:, q0: q0 + qn] = sc.t()


class PageTables:
    """Page tables of one scheduling step's requests, uploaded once and shared by every forward of the
    step (draft catch-up, every draft round, verify): only the small per-request arrays (prefix length,
    query lengths) are uploaded per forward, in one packed copy. Cascade groups are computed once, with a
    vectorised longest-common-prefix over the padded page matrix."""

    def __init__(self, page_lists: Sequence[Sequence[int]], device, page_size: int):
        import numpy as np
        self.device = device
        self.ps = page_size
        self.h_indptr = [0]
        self.h_pages: List[int] = []
        for pl in page_lists:
            self.h_pages.extend(pl)
            self.h_indptr.append(len(self.h_pages))
        i32 = dict(dtype=torch.int32)
        both = upload(self.h_pages + self.h_indptr, torch.int32, device)
        n = len(self.h_pages)
        self.pages = both[:n] if n else torch.zeros(1, dtype=torch.int32, device=device)
        self.page_indptr = both[n:]
        lmax = max((len(pl) for pl in page_lists), default=0)
        self.padded = np.full((len(page_lists), max(lmax, 1)), -1, dtype=np.int64)
        for r, pl in enumerate(page_lists):
            self.padded[r, :len(pl)] = pl

    def padded_device(self, device, dtype=torch.int64) -> torch.Tensor:
        """[R, max pages] page table on the device (unused entries 0)."""
        import numpy as np
        return upload(torch.from_numpy(np.where(self.padded < 0, 0, self.padded)), dtype, device)

    def groups(self, committed: Sequence[int], min_shared_pages: int = 1, min_group: int = 2):
        """Consecutive requests sharing >= min_shared_pages committed pages: [(r_first, r_last, keys)]."""
        import numpy as np
        R = self.padded.shape[0]
        if R < min_group:
            return []
        cp = np.asarray(committed, dtype=np.int64) // self.ps
        lim = np.minimum(cp[1:], cp[:-1])                                   # [R-1]
        cols = np.arange(self.padded.shape[1])[None, :]
        eq = (self.padded[1:] == self.padded[:-1]) & (cols < lim[:, None]) & (self.padded[1:] >= 0)
        lcp = np.where(eq.all(1), eq.shape[1], eq.argmin(1))                # consecutive LCP in pages
        out, r = [], 0
        while r < R:
            e, shared = r, None
            while e + 1 < R and lcp[e] >= min_shared_pages:
                shared = lcp[e] if shared is None else min(shared, lcp[e])
                e += 1
            if e - r + 1 >= min_group and shared is not None and shared >= min_shared_pages:
                out.append((r, e, int(shared) * self.ps))
                r = e + 1
            else:
                r += 1
        return out

    def meta(self, prefix_len: Sequence[int], q_lens: Sequence[int], tree: Optional[torch.Tensor],
             causal: bool) -> AttnMeta:
        qs = [0]
        for n in q_lens:
            qs.append(qs[-1] + n)
        kv = [p + n for p, n in zip(prefix_len, q_lens)]
        packed = upload(list(prefix_len) + kv + qs, torch.int32, self.device)
        R = len(prefix_len)
        return AttnMeta(pages=self.pages, page_indptr=self.page_indptr, prefix_len=packed[:R], kv_len=packed[R:2 * R],
                        q_start=packed[2 * R:], tree=tree, causal=causal, h_page_indptr=self.h_indptr,
                        h_pages=self.h_pages, h_prefix_len=list(prefix_len), h_kv_len=kv, h_q_start=qs)
