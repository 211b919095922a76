"""The allocation-free cascade attention entry point (csrc/phx_noalloc.h), called through its exported C
symbol, must match the regular entry point (ops.paged_attention, which allocates its partial buffers
through torch) on two calls in a row. It exists for callers that cannot allocate device memory at call
time (allocator hooks, fixed-budget runtimes, plain C hosts); this file is collected last so that a
stop-at-first-failure run has already run every other test."""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _lib():
    import phung5_b200._C as C  # loads the extension's torch dependencies first
    lib = ctypes.CDLL(C.__file__)
    f = lib.phx_cascade_attention_noalloc
    vp, i32 = ctypes.c_void_p, ctypes.c_int32
    f.argtypes = [vp] * 8 + [vp, vp, vp, i32, vp, vp, vp, i32, i32, i32, i32, i32, ctypes.c_float, vp, vp, vp, vp]
    f.restype = ctypes.c_int
    lib.phx_noalloc_strerror.restype = ctypes.c_char_p
    lib.phx_noalloc_strerror.argtypes = [ctypes.c_int]
    return lib


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _case(seed, q_lens, prefix, shared_pages):
    from tests.test_kernels_gpu import _paged_case, _to
    q, kc, vc, meta = _paged_case(seed, q_lens, prefix, tree=True, shared_pages=shared_pages)
    return q.to(DEV), kc.to(DEV), vc.to(DEV), meta, _to(meta, DEV)


def _regular(q, kc, vc, meta, gm, scale):
    from phung5_b200 import ops
    from phung5_b200.engine.attn_meta import build_items, cascade_groups, pack_work
    from phung5_b200.weights.quant import FP8_DTYPE
    t, hq = q.shape[0], q.shape[1]
    g = hq // kc.shape[1]
    p1, p2 = build_items(meta, g, cascade_groups(meta, 64) or None)
    out = torch.zeros(t, hq * 128, device=DEV, dtype=torch.bfloat16)
    oq = torch.zeros(t, hq * 128, device=DEV, dtype=FP8_DTYPE)
    osc = torch.zeros(hq, t, device=DEV)
    op = lp = None
    if p1:
        op = torch.zeros(t, hq, 128, device=DEV, dtype=torch.bfloat16)
        lp = torch.full((t, hq), float("-inf"), device=DEV)
        it, tl = pack_work(p1, g, DEV)
        ops.paged_attention(q, kc, vc, gm, scale, o_part=op, lse_part=lp, items=it, tiles=tl)
    it, tl = pack_work(p2, g, DEV)
    ops.paged_attention(q, kc, vc, gm, scale, o_in=op, lse_in=lp, out=out, out_q=oq, out_qs=osc, items=it, tiles=tl)
    return out, oq, osc, p1, p2


def _noalloc(lib, q, kc, vc, meta, gm, scale, p1, p2):
    from phung5_b200.engine.attn_meta import pack_work
    from phung5_b200.weights.quant import FP8_DTYPE
    t, hq, hkv = q.shape[0], q.shape[1], kc.shape[1]
    g = hq // hkv
    w1 = pack_work(p1, g, DEV, rows=64) if p1 else None      # the entry point's kernel tiles 64 rows
    it2, (ti2, tr2, n2) = pack_work(p2, g, DEV, rows=64)
    out = torch.zeros(t, hq * 128, device=DEV, dtype=torch.bfloat16)
    oq = torch.zeros(t, hq * 128, device=DEV, dtype=FP8_DTYPE)
    osc = torch.zeros(hq, t, device=DEV)
    if w1:
        it1, (ti1, tr1, n1) = w1
    else:
        it1 = ti1 = tr1 = None
        n1 = 0
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.phx_cascade_attention_noalloc(
        _ptr(q), _ptr(kc), _ptr(vc), _ptr(gm.pages), _ptr(gm.page_indptr), _ptr(gm.prefix_len), _ptr(gm.q_start),
        _ptr(gm.tree), _ptr(it1), _ptr(ti1), _ptr(tr1), n1, _ptr(it2), _ptr(ti2), _ptr(tr2), n2, t, hq, hkv, 0,
        scale, _ptr(out), _ptr(oq), _ptr(osc), stream)
    torch.cuda.synchronize()
    return rc, out, oq, osc


def test_noalloc_matches_regular_entry_point_twice():
    lib = _lib()
    scale = 1 / math.sqrt(128)
    cases = [_case(4, [64, 64, 9], [640, 700, 520], 8),      # shared prefix: both passes
             _case(6, [64, 33, 64, 5], [900, 130, 260, 1100], 2)]
    for q, kc, vc, meta, gm in cases:   # two calls in a row; the second reuses the scratch
        out, oq, osc, p1, p2 = _regular(q, kc, vc, meta, gm, scale)
        rc, out2, oq2, osc2 = _noalloc(lib, q, kc, vc, meta, gm, scale, p1, p2)
        assert rc == 0, lib.phx_noalloc_strerror(rc)
        rel = ((out2.float() - out.float()).norm() / out.float().norm()).item()
        assert rel < 1e-2, rel
        deq = oq.float() * osc.t().repeat_interleave(128, 1)
        deq2 = oq2.float() * osc2.t().repeat_interleave(128, 1)
        assert ((deq2 - deq).norm() / deq.norm()).item() < 4e-2


def _partly_shared_case(seed):
    """Requests 0 and 1 share their first six pages; request 2 shares nothing, so the prefix pass covers
    none of its rows."""
    from phung5_b200.engine.attn_meta import make_meta
    from tests.test_kernels_gpu import _to
    g = torch.Generator().manual_seed(seed)
    q_lens, prefix, hq, hkv, ps = [64, 40, 50], [600, 620, 300], 8, 2, 64
    need = [(p + n + ps - 1) // ps for p, n in zip(prefix, q_lens)]
    npages = 6 + (need[0] - 6) + (need[1] - 6) + need[2] + 1
    perm = torch.randperm(npages, generator=g).tolist()
    lists = [perm[:6] + perm[6:need[0]], perm[:6] + perm[need[0]:need[0] + need[1] - 6]]
    lists.append(perm[need[0] + need[1] - 6:need[0] + need[1] - 6 + need[2]])
    kc = torch.randn(npages, hkv, ps, 128, generator=g).bfloat16()
    vc = torch.randn(npages, hkv, ps, 128, generator=g).bfloat16()
    q = torch.randn(sum(q_lens), hq, 128, generator=g).bfloat16()
    bits = []
    for n in q_lens:            # a chain per request: node i sees nodes 0..i
        bits += [(1 << (i + 1)) - 1 - ((1 << 64) if i == 63 else 0) for i in range(n)]
    meta = make_meta(lists, prefix, q_lens, torch.tensor(bits, dtype=torch.int64), causal=False, device="cpu")
    return q.to(DEV), kc.to(DEV), vc.to(DEV), meta, _to(meta, DEV)


def test_noalloc_ignores_stale_partials_of_a_larger_call():
    """A large cascade call fills the shared array; a smaller call whose prefix pass covers only some requests
    must not pick up the earlier call's partials for the other rows (their LSE is reset to -inf)."""
    lib = _lib()
    scale = 1 / math.sqrt(128)
    big = _case(9, [64, 64, 64, 64], [900, 960, 700, 1000], 10)
    small = _partly_shared_case(10)
    for q, kc, vc, meta, gm in (big, small):
        out, oq, osc, p1, p2 = _regular(q, kc, vc, meta, gm, scale)
        if q is small[0]:
            assert p1, "the small case must still run a prefix pass for requests 0 and 1"
        rc, out2, _, _ = _noalloc(lib, q, kc, vc, meta, gm, scale, p1, p2)
        assert rc == 0, lib.phx_noalloc_strerror(rc)
        rel = ((out2.float() - out.float()).norm() / out.float().norm()).item()
        assert rel < 1e-2, rel
        per_row = ((out2.float() - out.float()).norm(dim=1) / out.float().norm(dim=1)).max().item()
        assert per_row < 3e-2, per_row


def test_noalloc_rejects_oversized_calls():
    lib = _lib()
    q, kc, vc, meta, gm = _case(4, [64, 64, 9], [640, 700, 520], 8)
    big_t = 32768 // q.shape[1] + 1
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    dummy = torch.zeros(16, dtype=torch.int32, device=DEV)
    rc = lib.phx_cascade_attention_noalloc(
        _ptr(q), _ptr(kc), _ptr(vc), _ptr(gm.pages), _ptr(gm.page_indptr), _ptr(gm.prefix_len), _ptr(gm.q_start),
        _ptr(gm.tree), None, None, None, 0, _ptr(dummy), _ptr(dummy), _ptr(dummy), 1, big_t, q.shape[1],
        kc.shape[1], 0, 0.1, _ptr(q), None, None, stream)
    assert rc == 1
    assert b"PHX_NOALLOC_MAX_ROWS" in lib.phx_noalloc_strerror(rc)
