"""Numerics of the sm_100a kernels against plain-PyTorch fp32 references of the same ops."""
import math

import pytest
import torch

from phung5_b200 import ops
from phung5_b200.engine.attn_meta import build_items, cascade_groups, make_meta, pack_work
from phung5_b200.weights.quant import FP8_DTYPE, dequant_act_block, gemm_fp8_block_ref, quant_act_block, quant_weight_block

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp(min=1e-12)).item()


@pytest.fixture(autouse=True)
def _status():
    yield
    ops.check_status()


@pytest.mark.parametrize("m,n,k,bn", [(128, 256, 256, 0), (200, 384, 512, 0), (1000, 1280, 1024, 256),
                                      (64, 128, 128, 128), (513, 1024, 2048, 128), (4096, 2048, 1024, 0),
                                      (96, 4000, 512, 0), (33, 200, 256, 256)])
def test_gemm_fp8_block(m, n, k, bn):
    g = torch.Generator(device=DEV).manual_seed(m + n + k)
    x = torch.randn(m, k, device=DEV, generator=g)
    w = torch.randn(n, k, device=DEV, generator=g) * 0.05
    xq, xs = quant_act_block(x)
    wq, ws = quant_weight_block(w)
    out = ops.gemm_fp8_block(xq, xs, wq, ws, bn=bn)
    torch.cuda.synchronize()
    ref = gemm_fp8_block_ref(xq, xs, wq, ws)
    assert _rel(out, ref) < 5e-3
    assert (out.float() - ref).abs().max().item() <= 0.02 * ref.abs().max().item()


def test_gemm_fp8_block_persistent_small_grid():
    # few CTAs -> every CTA walks many tiles through both TMEM accumulators
    m, n, k = 512, 1024, 1024
    x = torch.randn(m, k, device=DEV)
    w = torch.randn(n, k, device=DEV) * 0.05
    xq, xs = quant_act_block(x)
    wq, ws = quant_weight_block(w)
    out = ops.gemm_fp8_block(xq, xs, wq, ws, bn=256, max_ctas=3)
    ref = gemm_fp8_block_ref(xq, xs, wq, ws)
    assert _rel(out, ref) < 5e-3


@pytest.mark.parametrize("m,n,k,bn", [(200, 384, 512, 128), (300, 512, 1024, 256), (4096, 1280, 1024, 0),
                                      (77, 1000, 256, 0), (1000, 2048, 8192, 256)])
def test_gemm_fp8_hw_scale_matches_promotion(m, n, k, bn):
    """The tensor core's UE8M0 block scaling (kind::mxf8f6f4) equals the software per-K-block promotion, and
    both match the fp32 oracle; the quantizers' scales are powers of two."""
    from phung5_b200.weights.quant import is_pow2
    g = torch.Generator(device=DEV).manual_seed(3 * m + n + k)
    x = torch.randn(m, k, device=DEV, generator=g) * torch.rand(m, 1, device=DEV, generator=g) * 4
    w = torch.randn(n, k, device=DEV, generator=g) * 0.05
    xq, xs = quant_act_block(x)
    wq, ws = quant_weight_block(w)
    assert is_pow2(xs) and is_pow2(ws)
    hw = ops.gemm_fp8_block(xq, xs, wq, ws, bn=bn, hw_scale=True)
    sw = ops.gemm_fp8_block(xq, xs, wq, ws, bn=bn, hw_scale=False)
    ops.check_status()
    ref = gemm_fp8_block_ref(xq, xs, wq, ws)
    assert _rel(hw, ref) < 5e-3 and _rel(hw, sw) < 5e-3


@pytest.mark.parametrize("m,n,k,max_ctas", [(300, 512, 1024, 0), (129, 768, 512, 0), (4096, 1280, 1024, 0),
                                            (1024, 2048, 2048, 4), (4096, 8192, 1024, 0)])
def test_gemm_fp8_cta_pair_matches_single_cta(m, n, k, max_ctas):
    """256 x 256 tiles on CTA pairs (tcgen05 cta_group::2, each CTA staging half of A and half of B) give the
    single-CTA result: rows past M in the second CTA, a 2-pair persistent grid walking many tiles."""
    g = torch.Generator(device=DEV).manual_seed(m * 7 + n + k)
    x = torch.randn(m, k, device=DEV, generator=g)
    w = torch.randn(n, k, device=DEV, generator=g) * 0.05
    xq, xs = quant_act_block(x)
    wq, ws = quant_weight_block(w)
    one = ops.gemm_fp8_block(xq, xs, wq, ws, bn=256, max_ctas=max_ctas, hw_scale=True, pair=False)
    two = ops.gemm_fp8_block(xq, xs, wq, ws, bn=256, max_ctas=max_ctas, hw_scale=True, pair=True)
    ops.check_status()
    ref = gemm_fp8_block_ref(xq, xs, wq, ws)
    assert _rel(two, ref) < 5e-3 and _rel(two, one) < 1e-3


@pytest.mark.parametrize("kind,m,n,k,bn,split", [
    ("fp8", 512, 1280, 8192, 256, 0),     # draft qkv at TP8: 20 tiles -> 7 parts each
    ("fp8", 4096, 1280, 8192, 256, 0),    # verify qkv at TP8: 148 whole tiles + 12 tiles in 12 parts
    ("fp8", 300, 1032, 4096, 128, 5),     # ragged M and N, forced part count
    ("fp8", 77, 256, 2048, 256, 0),
    ("bf16", 512, 1280, 4096, 256, 0),
    ("bf16", 200, 520, 2048, 128, 3)])
def test_gemm_split_k_tail(kind, m, n, k, bn, split):
    """Grids whose last wave leaves most SMs idle split the remaining tiles over K: every part stores an fp32
    partial, meets the tile's other parts and sums a share of the tile. Equals the unsplit kernel to fp32
    summation order and the fp32 oracle; repeated calls reuse the workspace counters (reset by the last part);
    the split result is deterministic."""
    g = torch.Generator(device=DEV).manual_seed(m + 3 * n + k)
    x = torch.randn(m, k, device=DEV, generator=g)
    w = torch.randn(n, k, device=DEV, generator=g) * 0.05
    if kind == "fp8":
        xq, xs = quant_act_block(x)
        wq, ws = quant_weight_block(w)
        run = lambda sp: ops.gemm_fp8_block(xq, xs, wq, ws, bn=bn, hw_scale=True, split=sp)
        ref = gemm_fp8_block_ref(xq, xs, wq, ws)
    else:
        xb, wb = x.bfloat16(), w.bfloat16()
        run = lambda sp: ops.gemm_bf16(xb, wb, bn=bn, split=sp)
        ref = xb.float() @ wb.float().t()
    whole = run(1)
    parts = [run(split) for _ in range(3)]
    ops.check_status()
    assert _rel(parts[0], ref) < 5e-3 and _rel(parts[0], whole) < 2e-3
    assert torch.equal(parts[0], parts[1]) and torch.equal(parts[1], parts[2])


def test_split_gemm_and_topk_replay_in_cuda_graph():
    """The split-K tail's static workspace and counters, and the top-k kernels, work inside a captured CUDA graph:
    two replays on changed inputs equal eager launches bit for bit (the counters are back at zero after every
    launch)."""
    g = torch.Generator(device=DEV).manual_seed(11)
    x = torch.randn(512, 8192, device=DEV, generator=g)
    w = torch.randn(1280, 8192, device=DEV, generator=g) * 0.05
    xq, xs = quant_act_block(x)
    wq, ws = quant_weight_block(w)
    logits = (torch.randn(512, 128256, device=DEV, generator=g) * 2).bfloat16()
    out = torch.empty(512, 1280, device=DEV, dtype=torch.bfloat16)
    res = {}

    def body():
        ops.gemm_fp8_block(xq, xs, wq, ws, out=out, bn=256, hw_scale=True, split=0)
        res["topk"] = ops.topk_logprobs(logits, 8)
        res["argmax"] = ops.topk_logprobs(logits, 1, with_lse=False)
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        body()
    torch.cuda.current_stream().wait_stream(st)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        body()
    for _ in range(2):
        xq.copy_(quant_act_block(torch.randn(512, 8192, device=DEV, generator=g))[0])
        logits.copy_((torch.randn(512, 128256, device=DEV, generator=g) * 2).bfloat16())
        graph.replay()
        torch.cuda.synchronize()
        got = [out.clone()] + [t.clone() for t in res["topk"]] + [t.clone() for t in res["argmax"]]
        ref_out = ops.gemm_fp8_block(xq, xs, wq, ws, bn=256, hw_scale=True, split=0)
        ref = [ref_out] + list(ops.topk_logprobs(logits, 8)) + list(ops.topk_logprobs(logits, 1, with_lse=False))
        ops.check_status()
        for a, b in zip(got, ref):
            assert torch.equal(a, b)


def test_gemm_fp8_hw_scale_flags_non_pow2_scales():
    """A weight scale that is not a power of two cannot be a UE8M0 value: the hardware-scaled GEMM records it in
    the status word; the promotion path takes any fp32 scale."""
    x = torch.randn(256, 512, device=DEV)
    w = torch.randn(256, 512, device=DEV) * 0.05
    xq, xs = quant_act_block(x)
    wq, ws = quant_weight_block(w)
    ws = ws * 1.3
    ops.gemm_fp8_block(xq, xs, wq, ws, hw_scale=True)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="power of two"):
        ops.check_status()
    out = ops.gemm_fp8_block(xq, xs, wq, ws, hw_scale=False)
    ops.check_status()
    assert _rel(out, gemm_fp8_block_ref(xq, xs, wq, ws)) < 5e-3


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (300, 640, 1024), (2048, 4096, 4096), (77, 128256, 512),
                                   (50, 4000, 4096), (130, 200, 128)])
def test_gemm_bf16(m, n, k):
    x = torch.randn(m, k, device=DEV).bfloat16()
    w = (torch.randn(n, k, device=DEV) * 0.05).bfloat16()
    out = ops.gemm_bf16(x, w)
    ref = x.float() @ w.float().t()
    assert _rel(out, ref) < 5e-3


def _deq_close(q, s, ref, tol=1.0 / 15):
    from phung5_b200.weights.quant import is_pow2
    assert is_pow2(s)                     # every activation scale is exact in UE8M0
    deq = dequant_act_block(q.float().to(FP8_DTYPE) if q.dtype != FP8_DTYPE else q, s)
    m, k = ref.shape
    blk_amax = ref.abs().view(m, k // 128, 128).amax(-1, keepdim=True).clamp(min=1e-6)
    err = ((deq - ref).abs().view(m, k // 128, 128) / blk_amax).max().item()
    assert err <= tol, err


@pytest.mark.parametrize("m,h", [(1, 256), (7, 1024), (333, 8192), (64, 4096), (5, 1152)])
def test_add_rmsnorm_quant(m, h):
    hx = torch.randn(m, h, device=DEV).bfloat16()
    dx = torch.randn(m, h, device=DEV).bfloat16()
    w = (1 + 0.1 * torch.randn(h, device=DEV)).bfloat16()
    h_cpu, d_cpu, w_cpu = hx.cpu().clone(), dx.cpu(), w.cpu()
    quant = h % 128 == 0
    q, qs, y = ops.add_rmsnorm_quant(hx, dx, w, 1e-5, quant=quant, out_bf16=True)
    _, _, yr = ops.add_rmsnorm_quant(h_cpu, d_cpu, w_cpu, 1e-5, quant=False, out_bf16=True)
    assert torch.equal(hx.cpu(), h_cpu)  # residual add is exact bf16 round of the fp32 sum
    assert _rel(y.cpu(), yr) < 1e-2
    hf = h_cpu.float()
    yref = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-5) * w_cpu.float()
    if quant:
        _deq_close(q.cpu(), qs.cpu(), yref)


@pytest.mark.parametrize("m,f", [(1, 128), (37, 3584), (256, 14336)])
def test_silu_mul_quant(m, f):
    gu = torch.randn(m, 2 * f, device=DEV).bfloat16()
    q, qs, y = ops.silu_mul_quant(gu, quant=True, out_bf16=True)
    g, u = gu[:, :f].float().cpu(), gu[:, f:].float().cpu()
    a = (torch.nn.functional.silu(g) * u).bfloat16()
    assert _rel(y.cpu(), a) < 1e-2
    _deq_close(q.cpu(), qs.cpu(), a.float())


def test_act_quant():
    x = torch.randn(99, 1024, device=DEV).bfloat16()
    q, qs = ops.act_quant(x)
    _deq_close(q.cpu(), qs.cpu(), x.float().cpu())


@pytest.mark.parametrize("hq,hkv,d", [(8, 2, 128), (4, 4, 64), (5, 1, 128)])
def test_rope_kv_write(hq, hkv, d):
    ps, npages = 64, 10
    m = 37
    qkv = torch.randn(m, (hq + 2 * hkv) * d, device=DEV).bfloat16()
    pos = torch.randint(0, 4000, (m,), device=DEV, dtype=torch.int32)
    slots = torch.randperm(npages * ps, device=DEV)[:m].to(torch.int64)
    slots[3] = -1
    cs = ops.rope_table(4096, d, 5e5, DEV)
    kc = torch.zeros(npages, hkv, ps, d, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    qo = ops.rope_kv_write(qkv, pos, slots, cs, kc, vc, hq, hkv, d)
    kc2, vc2 = kc.cpu().zero_(), vc.cpu().zero_()
    qo2 = ops.rope_kv_write(qkv.cpu(), pos.cpu(), slots.cpu(), cs.cpu(), kc2, vc2, hq, hkv, d)
    assert _rel(qo.cpu(), qo2) < 1e-2
    assert _rel(kc.cpu(), kc2) < 1e-2
    assert torch.equal(vc.cpu(), vc2)


def _paged_case(seed, q_lens, prefix, hq=8, hkv=2, shared_pages=0, tree=False):
    """Random paged KV for R requests; the first `shared_pages` pages are shared by all requests."""
    g = torch.Generator().manual_seed(seed)
    d, ps = 128, 64
    r = len(q_lens)
    kv_len = [p + n for p, n in zip(prefix, q_lens)]
    need = [(k + ps - 1) // ps for k in kv_len]
    npages = shared_pages + sum(n - shared_pages for n in need) + 1
    perm = torch.randperm(npages, generator=g).tolist()
    shared = perm[:shared_pages]
    nxt = shared_pages
    page_lists = []
    for n in need:
        own = perm[nxt: nxt + n - shared_pages]
        nxt += n - shared_pages
        page_lists.append(shared + own)
    kc = torch.randn(npages, hkv, ps, d, generator=g).bfloat16()
    vc = torch.randn(npages, hkv, ps, d, generator=g).bfloat16()
    t = sum(q_lens)
    q = torch.randn(t, hq, d, generator=g).bfloat16()
    tree_bits = None
    if tree:
        bits = []
        for n in q_lens:
            par = [-1] + [int(torch.randint(0, i, (1,), generator=g)) for i in range(1, n)]
            for i in range(n):
                b, j = 0, i
                while j >= 0:
                    b |= 1 << j
                    j = par[j]
                bits.append(b - (1 << 64) if b >= (1 << 63) else b)
        tree_bits = torch.tensor(bits, dtype=torch.int64)
    meta = make_meta(page_lists, prefix, q_lens, tree_bits, causal=not tree, device="cpu")
    return q, kc, vc, meta


def _to(meta, dev):
    import dataclasses
    return dataclasses.replace(meta, pages=meta.pages.to(dev), page_indptr=meta.page_indptr.to(dev),
                               prefix_len=meta.prefix_len.to(dev), kv_len=meta.kv_len.to(dev),
                               q_start=meta.q_start.to(dev), tree=None if meta.tree is None else meta.tree.to(dev))


@pytest.mark.parametrize("impl", ["tc", "mma"])
@pytest.mark.parametrize("case", ["prefill", "decode", "tree", "cascade_tree", "long_prefix", "gqa1"])
def test_paged_attention(case, impl):
    hq, hkv = 8, 2
    if case == "prefill":
        q, kc, vc, meta = _paged_case(1, [100, 7, 64], [0, 130, 64])
    elif case == "decode":
        q, kc, vc, meta = _paged_case(2, [1, 1, 1, 1], [1, 500, 64, 4000])
    elif case == "tree":
        q, kc, vc, meta = _paged_case(3, [64, 17], [300, 1024], tree=True)
    elif case == "cascade_tree":
        q, kc, vc, meta = _paged_case(4, [64, 64, 9], [640, 700, 520], tree=True, shared_pages=8)
    elif case == "long_prefix":
        q, kc, vc, meta = _paged_case(5, [64, 64, 64, 64], [4096 + 520, 4096 + 512, 4096 + 700, 4096 + 300],
                                      tree=True, shared_pages=64)
    else:
        q, kc, vc, meta = _paged_case(7, [33, 5], [200, 64], hq=4, hkv=4)
        hq, hkv = 4, 4
    scale = 1 / math.sqrt(128)
    t = q.shape[0]
    groups = cascade_groups(meta, 64) if case == "cascade_tree" else None
    if case == "cascade_tree":
        assert groups and groups[0][2] == 8 * 64
    if case == "long_prefix":
        groups = cascade_groups(meta, 64)
    p1, p2 = build_items(meta, hq // hkv, groups)
    # reference
    out_ref = torch.zeros(t, hq * 128)
    oq_ref = torch.zeros(t, hq * 128, dtype=FP8_DTYPE)
    os_ref = torch.zeros(hq, t)
    o_part = torch.zeros(t, hq, 128)
    lse_part = torch.full((t, hq), float("-inf"))
    if p1:
        ops.paged_attention(q, kc, vc, meta, scale, o_part=o_part, lse_part=lse_part, items=p1)
    ops.paged_attention(q, kc, vc, meta, scale, o_in=o_part if p1 else None, lse_in=lse_part if p1 else None,
                        out=out_ref, out_q=oq_ref, out_qs=os_ref, items=p2)
    # gpu
    gm = _to(meta, DEV)
    qg, kg, vg = q.to(DEV), kc.to(DEV), vc.to(DEV)
    out = torch.zeros(t, hq * 128, device=DEV, dtype=torch.bfloat16)
    oq = torch.zeros(t, hq * 128, device=DEV, dtype=FP8_DTYPE)
    osc = torch.zeros(hq, t, device=DEV)
    op = torch.zeros(t, hq, 128, device=DEV, dtype=torch.bfloat16)
    lp = torch.full((t, hq), float("-inf"), device=DEV)
    rows = ops.attn_rows(impl)
    if p1:
        it, tl = pack_work(p1, hq // hkv, DEV, rows=rows)
        ops.paged_attention(qg, kg, vg, gm, scale, o_part=op, lse_part=lp, items=it, tiles=tl, impl=impl)
    it, tl = pack_work(p2, hq // hkv, DEV, rows=rows)
    ops.paged_attention(qg, kg, vg, gm, scale, o_in=op if p1 else None, lse_in=lp if p1 else None, out=out,
                        out_q=oq, out_qs=osc, items=it, tiles=tl, impl=impl)
    torch.cuda.synchronize()
    assert _rel(out.cpu(), out_ref) < 1e-2
    deq = (oq.cpu().float().view(t, hq, 128) * osc.cpu().t()[..., None]).view(t, hq * 128)
    assert _rel(deq, out_ref) < 4e-2


@pytest.mark.parametrize("r,v,k,t", [(512, 128256, 8, 1.0), (4096, 16032, 1, 1.0), (7, 32000, 16, 0.7),
                                     (3, 1000, 4, 1.0), (64, 4001, 8, 1.3)])
def test_topk_logprobs(r, v, k, t):
    g = torch.Generator(device=DEV).manual_seed(r + v)
    x = (torch.randn(r, v, device=DEV, generator=g) * 2).bfloat16()
    if v == 4001:
        x = x[:, :4000]          # non-16-byte-aligned row stride
    lp, idx, lse = ops.topk_logprobs(x, k, temperature=t)
    xf = x.float() / t
    ref_lse = torch.logsumexp(xf, -1)
    rv, ri = torch.topk(xf, k, dim=-1)
    assert torch.allclose(lse, ref_lse, atol=1e-3, rtol=1e-5)
    assert torch.allclose(lp, rv - ref_lse[:, None], atol=1e-3)
    # indices agree up to exact ties in bf16
    got = xf.gather(1, idx)
    assert torch.equal(got, rv)


@pytest.mark.parametrize("r,v,k,mode", [(64, 128256, 8, "ints"), (16, 40000, 16, "const"), (33, 16032, 4, "ints"),
                                        (5, 20000, 1, "const")])
def test_topk_heavy_ties_lowest_index_first(r, v, k, mode):
    """Rows with massive ties (small integers, or one constant value, which overflows the threshold filter's
    candidate buffer): the k best by (value desc, index asc), as a stable descending sort orders them."""
    g = torch.Generator(device=DEV).manual_seed(r * 3 + v)
    if mode == "ints":
        x = torch.randint(-3, 4, (r, v), device=DEV, generator=g).bfloat16()
    else:
        x = torch.full((r, v), 1.5, device=DEV).bfloat16()
        x[:, ::7] = -2.0
    lp, idx, lse = ops.topk_logprobs(x, k)
    ops.check_status()
    order = torch.sort(-x.float(), dim=-1, stable=True).indices[:, :k]
    assert torch.equal(idx, order)
    assert torch.allclose(lse, torch.logsumexp(x.float(), -1), atol=1e-3, rtol=1e-5)


@pytest.mark.parametrize("sizes,n,k", [([100, 0, 300, 7, 256], 512, 1024), ([513], 384, 256), ([0, 0, 64], 256, 512),
                                       ([40] * 8, 3072, 1024)])
def test_gemm_grouped(sizes, n, k):
    g = len(sizes)
    m = sum(sizes) + 50                       # tail rows past the last group are never written
    x = torch.randn(m, k, device=DEV)
    xq, xs = quant_act_block(x)
    ws_list, s_list = [], []
    for e in range(g):
        q_, s_ = quant_weight_block(torch.randn(n, k, device=DEV) * 0.05)
        ws_list.append(q_)
        s_list.append(s_)
    wq, ws = torch.cat(ws_list), torch.cat(s_list)
    off = torch.tensor([0] + list(torch.tensor(sizes).cumsum(0)), dtype=torch.int32, device=DEV)
    out = torch.full((m, n), 7.0, device=DEV, dtype=torch.bfloat16)
    ops.gemm_grouped((xq, xs), wq, ws, off, n, out=out)
    torch.cuda.synchronize()
    o = off.tolist()
    for e in range(g):
        a, b = o[e], o[e + 1]
        if b > a:
            ref = gemm_fp8_block_ref(xq[a:b], xs[:, a:b], ws_list[e], s_list[e])
            assert _rel(out[a:b], ref) < 5e-3
    assert (out[o[-1]:].float() == 7.0).all()
    # bf16 grouped
    xb = x.bfloat16()
    wb = torch.cat([w_.float() * 0 + torch.randn_like(w_.float()) * 0.05 for w_ in ws_list]).bfloat16()
    outb = ops.gemm_grouped(xb, wb, None, off, n)
    for e in range(g):
        a, b = o[e], o[e + 1]
        if b > a:
            assert _rel(outb[a:b], xb[a:b].float() @ wb[e * n:(e + 1) * n].float().t()) < 5e-3


def test_gdn_kernels_match_definitions():
    from phung5_b200.models.gdn import random_gdn_layer
    torch.manual_seed(0)
    layer_c = random_gdn_layer(512, 2, 4, "cpu", seed=3, dtype=torch.float32)
    layer_g = random_gdn_layer(512, 2, 4, DEV, seed=3, dtype=torch.bfloat16)
    lens = [5, 1, 9]
    ts = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    slot = torch.tensor([2, 0, 1], dtype=torch.int32)
    x = torch.randn(sum(lens), 512)
    win = torch.randn(3, 3, layer_c.conv_channels) * 0.1
    st = torch.randn(3, 4, 128, 128) * 0.01
    wg, sg = win.to(DEV, torch.bfloat16), st.to(DEV)
    wc, sc = win.to(torch.bfloat16).float(), st.clone()
    xb = x.to(DEV, torch.bfloat16)
    y_g = layer_g.forward(xb, ts.to(DEV), slot.to(DEV), wg, sg, mode="verify")
    y_c = layer_c.forward(xb.float().cpu(), ts, slot, wc, sc, mode="verify")
    assert _rel(y_g.float().cpu(), y_c) < 3e-2
    n = torch.tensor([3, 1, 0], dtype=torch.int32)
    layer_g.commit(n.to(DEV), wg, sg)
    layer_c.commit(n, wc, sc)
    torch.cuda.synchronize()
    assert _rel(sg.cpu(), sc) < 2e-2
    assert _rel(wg.float().cpu(), wc) < 1e-2
    # prefill mode (state written in the kernel)
    y2 = layer_g.forward(xb, ts.to(DEV), slot.to(DEV), wg, sg, mode="prefill")
    y2c = layer_c.forward(xb.float().cpu(), ts, slot, wc, sc, mode="prefill")
    assert _rel(y2.float().cpu(), y2c) < 3e-2 and _rel(sg.cpu(), sc) < 3e-2


@pytest.mark.parametrize("write_state", [False, True])
def test_gdn_recurrent_many_requests(write_state):
    """Many (request, value head) items and token counts from 0 to 37 (chunks of 16, a partial chunk, an empty
    request): outputs, stash and written states against the plain-torch definition."""
    from phung5_b200.ops import gdn as G
    g = torch.Generator().manual_seed(5)
    R, HK, HV = 40, 4, 8
    lens = [(i * 7) % 38 for i in range(R)]
    ts = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    T = int(ts[-1])
    q = torch.randn(T, HK, 128, generator=g).bfloat16()
    k = torch.randn(T, HK, 128, generator=g).bfloat16()
    v = torch.randn(T, HV, 128, generator=g).bfloat16()
    gg = -torch.rand(T, HV, generator=g) * 0.5
    beta = torch.rand(T, HV, generator=g)
    slot = torch.randperm(R + 3, generator=g)[:R].to(torch.int32)
    state = torch.randn(R + 3, HV, 128, 128, generator=g) * 0.02
    st_c = state.clone()
    out_c, stash_c = G.gdn_recurrent(q.float(), k.float(), v.float(), gg, beta, st_c, ts, slot, 0.088, write_state)
    st_g = state.to(DEV)
    out_g, stash_g = G.gdn_recurrent(q.to(DEV), k.to(DEV), v.to(DEV), gg.to(DEV), beta.to(DEV), st_g, ts.to(DEV),
                                     slot.to(DEV), 0.088, write_state)
    ops.check_status()
    assert _rel(out_g.float().cpu(), out_c) < 2e-2
    assert _rel(stash_g[0].cpu(), stash_c[0]) < 1e-3 and _rel(stash_g[1].cpu(), stash_c[1]) < 2e-2
    assert torch.equal(stash_g[2].cpu(), stash_c[2])
    assert _rel(st_g.cpu(), st_c) < (2e-2 if write_state else 1e-7)


@pytest.mark.parametrize("t,sizes,n,k", [(300, [120, 0, 333, 47], 512, 1024), (64, [5, 70], 256, 256)])
def test_gemm_grouped_row_gather_equals_gathered_copy(t, sizes, n, k):
    """The grouped GEMM's A loads gather activation rows by index (TMA gather4, the MoE dispatch fused into
    the GEMM): bitwise the result of running it on the explicitly gathered copy."""
    g = torch.Generator(device=DEV).manual_seed(t + n)
    x = torch.randn(t, k, device=DEV, generator=g)
    xq, xs = quant_act_block(x)
    m = sum(sizes)
    rows = torch.randint(0, t, (m,), device=DEV, generator=g, dtype=torch.int32)
    ws_list, s_list = zip(*[quant_weight_block(torch.randn(n, k, device=DEV, generator=g) * 0.05) for _ in sizes])
    wq, ws = torch.cat(ws_list), torch.cat(s_list)
    off = torch.tensor([0] + list(torch.tensor(sizes).cumsum(0)), dtype=torch.int32, device=DEV)
    got = ops.gemm_grouped((xq, xs), wq, ws, off, n, rows=rows)
    ref = ops.gemm_grouped((xq[rows.long()], xs[:, rows.long()].contiguous()), wq, ws, off, n)
    ops.check_status()
    assert torch.equal(got, ref)


def test_moe_block_fp8_matches_oracle_and_routes_identically():
    from phung5_b200.config import preset
    from phung5_b200.models.llama import pack_weights
    from phung5_b200.models.reference import moe_mlp
    from phung5_b200.weights.init import random_weights
    cfg = preset("small-moe-fp8")
    w = random_weights(cfg, seed=0, std=0.02)
    blk = pack_weights(cfg, w, DEV).layers[0].moe
    xb = torch.randn(64, cfg.hidden).bfloat16().to(DEV)
    y = blk(ops.act_quant(xb), xb).float().cpu()
    ref = moe_mlp(xb.float().cpu(), w, "model.layers.0.", cfg)
    assert ((y - ref).norm(dim=-1) / ref.norm(dim=-1)).max().item() < 0.08
    ids, _ = blk.route(xb)
    ref_ids = torch.topk(xb.float().cpu() @ w["model.layers.0.block_sparse_moe.gate.weight"].float().t(), 2, -1).indices
    assert torch.equal(ids.cpu().sort(-1).values, ref_ids.sort(-1).values)


def test_rasterizer_matches_cpu_restatement():
    from phung5_b200.render.scene import normalise, render, scene_triangles, view_projection
    from tests.test_render_cpu import SCENE
    tris, cols = scene_triangles(SCENE)
    tris = normalise(tris)
    g = torch.Generator().manual_seed(0)
    extra = torch.rand(2000, 3, 3, generator=g) - 0.5                  # many overlapping triangles
    tris = torch.cat([tris, extra * 0.8])
    cols = torch.cat([cols, torch.rand(2000, 3, generator=g)])
    for az, el in [(0, 15), (70, 30), (200, -20)]:
        vp = view_projection(az, el)
        a = render(tris.to(DEV), cols.to(DEV), vp, 256).cpu()
        b = render(tris, cols, vp, 256)
        diff = (a.int() - b.int()).abs().amax(-1)
        # edge-coverage or last-bit differences (device FMA contraction vs host) on a few pixels only
        assert (diff > 2).float().mean().item() < 0.01


def test_standard_material_rasterizer_matches_cpu_restatement():
    from phung5_b200.render.scene import normalise, render_pbr, scene_triangles
    from tests.test_render_cpu import SCENE
    tris, cols, mats = scene_triangles(SCENE, with_materials=True)
    tris = normalise(tris)
    g = torch.Generator().manual_seed(1)
    extra = torch.rand(2000, 3, 3, generator=g) - 0.5
    tris = torch.cat([tris, extra * 0.8])
    cols = torch.cat([cols, torch.rand(2000, 3, generator=g)])
    mats = torch.cat([mats, torch.rand(2000, 2, generator=g)])
    for (az, el), rig in zip([(0, 15), (70, 30), (200, -20)], ["studio", "neutral", "follow"]):
        a = render_pbr(tris.to(DEV), cols.to(DEV), mats.to(DEV), az, el, 256, rig).cpu()
        b = render_pbr(tris, cols, mats, az, el, 256, rig)
        diff = (a.int() - b.int()).abs().amax(-1)
        assert (diff > 2).float().mean().item() < 0.01


def test_selftest_cli_passes():
    from phung5_b200.ops import selftest
    res = selftest.run()
    assert all(v["ok"] for v in res.values()), res


@pytest.mark.parametrize("bulk", [True, False])
@pytest.mark.parametrize("fp8,m,n,k,hws", [(True, 4096, 8192, 1024, True), (True, 300, 1024, 512, True),
                                           (False, 200, 512, 256, False), (True, 77, 256, 128, True),
                                           (True, 300, 1024, 512, False), (True, 4096, 8192, 3584, True)])
def test_gemm_scatter_epilogue(fp8, m, n, k, hws, bulk):
    """The row-parallel projection's scatter epilogue: row r lands in buffer owner(r) = r // rows_per at slot
    [rank][r - owner * rows_per]. Four local buffers stand in for the peers' receive regions."""
    world, rank = 4, 1
    rows_per = (m + world - 1) // world
    x = torch.randn(m, k, device=DEV)
    w = torch.randn(n, k, device=DEV) * 0.05
    bufs = [torch.full((world, rows_per, n), 3.0, device=DEV, dtype=torch.bfloat16) for _ in range(world)]
    base = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=DEV)
    if fp8:
        xq, xs = quant_act_block(x)
        wq, ws = quant_weight_block(w)
        ops.ext().gemm_scatter(xq, xs, wq, ws, base, 0, rows_per, rank, ops.status_tensor(DEV), hws, False, 0, bulk)
        ref = ops.gemm_fp8_block(xq, xs, wq, ws, hw_scale=hws, split=1)     # the scatter epilogue never splits K
    else:
        xb, wb = x.bfloat16(), w.bfloat16()
        ops.ext().gemm_scatter(xb, None, wb, None, base, 0, rows_per, rank, ops.status_tensor(DEV), False, False, 0,
                               bulk)
        ref = ops.gemm_bf16(xb, wb, split=1)
    torch.cuda.synchronize()
    for o in range(world):
        r0, r1 = o * rows_per, min(m, (o + 1) * rows_per)
        got = bufs[o][rank, : r1 - r0]
        assert torch.equal(got, ref[r0:r1])                    # same kernel math: bitwise
        assert bool((bufs[o][rank, r1 - r0:] == 3.0).all())    # nothing past the owner's rows
        for other in range(world):
            if other != rank:
                assert bool((bufs[o][other] == 3.0).all())     # other ranks' slots untouched


def test_kernels_are_deterministic():
    """Same inputs, same bits: GEMMs (fp8 and bf16), the fused norm/quant, top-k and paged attention are run
    twice; no kernel here reduces with atomics, so any difference would be a race."""
    x = torch.randn(1000, 1024, device=DEV)
    w = torch.randn(1280, 1024, device=DEV) * 0.05
    xq, xs = quant_act_block(x)
    wq, ws = quant_weight_block(w)
    runs = []
    for _ in range(2):
        out = [ops.gemm_fp8_block(xq, xs, wq, ws).clone(), ops.gemm_bf16(x.bfloat16(), w.bfloat16()).clone()]
        h = x[:, :512].bfloat16().clone()
        q, s, y = ops.add_rmsnorm_quant(h, x[:, 512:].bfloat16(), torch.ones(512, device=DEV, dtype=torch.bfloat16),
                                        1e-5, quant=True, out_bf16=True)
        out += [h, q.view(torch.uint8), s, y]
        lp, idx, lse = ops.topk_logprobs(out[1], 8)
        out += [lp, idx, lse]
        qa, kc, vc, meta = _paged_case(9, [64, 17], [300, 500], tree=True)
        gm = _to(meta, DEV)
        _, p2 = build_items(meta, 4)
        it, tl = pack_work(p2, 4, DEV)
        o = torch.zeros(qa.shape[0], 8 * 128, device=DEV, dtype=torch.bfloat16)
        ops.paged_attention(qa.to(DEV), kc.to(DEV), vc.to(DEV), gm, 1 / math.sqrt(128), out=o, items=it, tiles=tl)
        out.append(o)
        torch.cuda.synchronize()
        runs.append(out)
    for a, b in zip(*runs):
        assert torch.equal(a, b)


@pytest.mark.parametrize("r,v", [(4096, 128256), (7, 1000)])
def test_argmax_without_lse(r, v):
    x = (torch.randn(r, v, device=DEV) * 2).bfloat16()
    val, idx, lse = ops.topk_logprobs(x, 1, with_lse=False)
    rv, ri = torch.topk(x.float(), 1, dim=-1)
    assert torch.equal(val, rv) and torch.equal(lse, torch.zeros_like(lse))
    assert torch.equal(x.float().gather(1, idx), rv)


@pytest.mark.parametrize("t,k,h", [(300, 2, 4096), (17, 8, 1024), (64, 1, 256)])
def test_moe_combine_matches_definition(t, k, h):
    """The fused MoE combine equals the weighted gather-sum of expert rows, skips non-local slots (whose rows
    hold garbage) and writes into a strided output."""
    g = torch.Generator(device=DEV).manual_seed(t + k)
    mp = t * k + 5
    y = torch.randn(mp, h, device=DEV, generator=g).bfloat16()
    pos = torch.randperm(t * k, device=DEV, generator=g).view(t, k)
    w = torch.rand(t, k, device=DEV, generator=g)
    local = torch.rand(t, k, device=DEV, generator=g) > 0.3
    y[pos[~local]] = float("nan")                              # unwritten rows of non-local slots
    buf = torch.full((t, h + 64), 5.0, device=DEV, dtype=torch.bfloat16)
    out = buf[:, :h]
    ops.moe_combine(y, pos, w, local, out)
    torch.cuda.synchronize()
    yf = y.float().nan_to_num(0.0)
    ref = (torch.where(local[..., None], yf[pos] * w[..., None], torch.zeros((), device=DEV))).sum(1)
    assert _rel(out, ref) < 1e-2 and torch.isfinite(out.float()).all()
    assert bool((buf[:, h:] == 5.0).all())


@pytest.mark.parametrize("m,f,k", [(300, 384, 1024), (77, 128, 256), (4096, 3584, 8192)])
def test_gemm_swiglu_epilogue_equals_gemm_then_silu_quant(m, f, k):
    """The gate/up GEMM with the SwiGLU + FP8 quant epilogue (weights interleaved in 128-row blocks) is bitwise
    the plain GEMM's bf16 [gate | up] output followed by silu_mul_quant; the interleaved Linear's plain call
    still returns the [gate | up] layout."""
    from phung5_b200.models.llama import Linear
    g = torch.Generator(device=DEV).manual_seed(m + f + k)
    x = torch.randn(m, k, device=DEV, generator=g)
    w = torch.randn(2 * f, k, device=DEV, generator=g) * 0.05
    xq, xs = quant_act_block(x)
    wq, ws = quant_weight_block(w)
    gu = ops.gemm_fp8_block(xq, xs, wq, ws, bn=256, hw_scale=True, split=1)   # the SwiGLU epilogue never splits K
    q_ref, s_ref, _ = ops.silu_mul_quant(gu, quant=True, out_bf16=False)
    lin = Linear(wq.clone(), ws.clone())
    fused = ops.SWIGLU_FUSED
    ops.SWIGLU_FUSED = True
    try:
        q, s = lin.swiglu((xq, xs))
    finally:
        ops.SWIGLU_FUSED = fused
    ops.check_status()
    assert lin.gu_interleaved
    assert torch.equal(q.view(torch.uint8), q_ref.view(torch.uint8)) and torch.equal(s, s_ref)
    assert _rel(lin((xq, xs)), gu) < 1e-3
