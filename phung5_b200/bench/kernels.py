"""Per-kernel microbenchmarks with roofline fractions.

    python -m phung5_b200.bench.kernels [--kernel NAME ...] [--iters 10] [--impl reference]

--impl reference times the reference's own Triton kernels (imported unmodified from baseline/_ref) next to
ours at the same shapes: bf16 top-k of logits / T, verify-row target candidates, GDN target verify.

Each case is timed with CUDA events on the current stream after 3 warm-up launches, flushing L2
(a 512 MB write) before every timed launch, and reported as achieved TFLOP/s or GB/s and as the fraction
of the measured peaks in MEASURED_PEAKS.json (copy bandwidth, cuBLAS bf16 burst); fp8 tensor work is
compared against twice the measured bf16 rate (the dense fp8:bf16 ratio of the part).
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

from .. import ops
from ..engine.attn_meta import build_items, cascade_groups, make_meta, pack_work
from ..weights.quant import FP8_DTYPE, pow2_scale

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


_FLUSH = {}


def flush_l2(dev):
    buf = _FLUSH.get(dev)
    if buf is None:
        buf = _FLUSH[dev] = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device=dev)
    buf.fill_(1)


def time_it(fn, iters=10, warmup=3, dev="cuda"):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        flush_l2(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    times.sort()
    return times[len(times) // 2]


def case_gemm_fp8(m, n, k, bn=0):
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    xq, xs = ops.act_quant(x)
    wq = (torch.randn(n, k, device="cuda", dtype=torch.bfloat16) * 0.05).to(FP8_DTYPE)
    ws = pow2_scale(torch.rand((n + 127) // 128, k // 128, device="cuda") * 4.48)   # ~1e-2, UE8M0-exact
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    fn = lambda: ops.gemm_fp8_block(xq, xs, wq, ws, out=out, bn=bn)
    return fn, 2.0 * m * n * k, "fp8"


def case_gemm_scatter_local(m, n, k, world=8, bulk=True):
    """The row-parallel projection's scatter epilogue with W local buffers standing in for the ranks' receive
    slots: the epilogue's cost without NVLink (compare with the plain GEMM of the same shape)."""
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    xq, xs = ops.act_quant(x)
    wq = (torch.randn(n, k, device="cuda", dtype=torch.bfloat16) * 0.05).to(FP8_DTYPE)
    ws = pow2_scale(torch.rand((n + 127) // 128, k // 128, device="cuda") * 4.48)
    rows_per = (m + world - 1) // world
    bufs = [torch.empty(world, rows_per, n, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    base = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device="cuda")
    st = ops.status_tensor(x.device)
    fn = lambda: ops.ext().gemm_scatter(xq, xs, wq, ws, base, 0, rows_per, 1, st, ops.FP8_HW_SCALE, False, 0, bulk)
    fn.keep = bufs
    return fn, 2.0 * m * n * k, "fp8"


def case_moe_gate_up_gather(tokens, per_expert, n, k, gather=True):
    """One expert's gate/up grouped GEMM with the dispatch inside the A loads (TMA gather4 of token rows), or
    (gather=False) an explicit row gather of the fp8 activations and scales followed by the plain grouped GEMM."""
    x = torch.randn(tokens, k, device="cuda", dtype=torch.bfloat16)
    xq, xs = ops.act_quant(x)
    wq = (torch.randn(n, k, device="cuda", dtype=torch.bfloat16) * 0.05).to(FP8_DTYPE)
    ws = pow2_scale(torch.rand((n + 127) // 128, k // 128, device="cuda") * 4.48)
    rows = torch.randint(0, tokens, (per_expert,), device="cuda", dtype=torch.int32)
    off = torch.tensor([0, per_expert], dtype=torch.int32, device="cuda")
    out = torch.empty(per_expert, n, device="cuda", dtype=torch.bfloat16)
    if gather:
        fn = lambda: ops.gemm_grouped((xq, xs), wq, ws, off, n, out=out, rows=rows)
    else:
        rl = rows.long()
        fn = lambda: ops.gemm_grouped((xq[rl], xs[:, rl].contiguous()), wq, ws, off, n, out=out)
    return fn, 2.0 * per_expert * n * k, "fp8"


def case_moe_combine(t, k, h):
    """Fused MoE combine: t tokens x top-k expert rows of width h -> bf16 [t, h]."""
    y = torch.randn(t * k, h, device="cuda", dtype=torch.bfloat16)
    pos = torch.randperm(t * k, device="cuda").view(t, k)
    w = torch.rand(t, k, device="cuda")
    local = torch.ones(t, k, device="cuda", dtype=torch.bool)
    out = torch.empty(t, h, device="cuda", dtype=torch.bfloat16)
    fn = lambda: ops.moe_combine(y, pos, w, local, out)
    return fn, t * k * h * 2 + t * h * 2, "bytes"


def case_gemm_swiglu(m, f, k, fused=True):
    """Gate/up projection + SwiGLU + FP8 quant: one GEMM with the fused epilogue, or (fused=False) the GEMM's
    bf16 [gate | up] output followed by silu_mul_quant."""
    from ..models.llama import interleave_gate_up
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    xq, xs = ops.act_quant(x)
    wq = (torch.randn(2 * f, k, device="cuda", dtype=torch.bfloat16) * 0.05).to(FP8_DTYPE)
    ws = pow2_scale(torch.rand(2 * f // 128, k // 128, device="cuda") * 4.48)
    if fused:
        wi, si = interleave_gate_up(wq, ws)
        fn = lambda: ops.gemm_fp8_swiglu(xq, xs, wi, si)
    else:
        fn = lambda: ops.silu_mul_quant(ops.gemm_fp8_block(xq, xs, wq, ws), quant=True, out_bf16=False)
    return fn, 2.0 * m * 2 * f * k, "fp8"


def case_gemm_bf16(m, n, k):
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(n, k, device="cuda", dtype=torch.bfloat16) * 0.05
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    return (lambda: ops.gemm_bf16(x, w, out=out)), 2.0 * m * n * k, "bf16"


def _verify_case(reqs=64, nodes=64, prefix=4096, suffix=600, hq=64, hkv=8):
    """The verify attention of the headline workload: `reqs` requests sharing `prefix` keys, each with
    `suffix` private committed keys and a `nodes`-node tree."""
    ps = 64
    shared = prefix // ps
    own = (suffix + nodes + ps - 1) // ps + 1
    npages = shared + reqs * own + 1
    kc = torch.randn(npages, hkv, ps, 128, device="cuda", dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    page_lists, nxt = [], shared
    for _ in range(reqs):
        page_lists.append(list(range(shared)) + list(range(nxt, nxt + own)))
        nxt += own
    par = [-1] + [(i - 1) // 8 if i > 8 else 0 for i in range(1, nodes)]
    bits = []
    for i in range(nodes):
        b, j = 0, i
        while j >= 0:
            b |= 1 << j
            j = par[j]
        bits.append(b - (1 << 64) if b >= (1 << 63) else b)
    tree = torch.tensor(bits * reqs, dtype=torch.int64)
    meta = make_meta(page_lists, [prefix + suffix] * reqs, [nodes] * reqs, tree, False, "cuda")
    q = torch.randn(reqs * nodes, hq, 128, device="cuda", dtype=torch.bfloat16)
    return q, kc, vc, meta


def case_silu_quant(m, f):
    gu = torch.randn(m, 2 * f, device="cuda", dtype=torch.bfloat16)
    fn = lambda: ops.silu_mul_quant(gu, quant=True, out_bf16=False)
    return fn, m * (2 * f * 2 + f + 4 * f // 128), "bytes"


def case_rmsnorm_quant(m, h):
    hx = torch.randn(m, h, device="cuda", dtype=torch.bfloat16)
    dx = torch.randn(m, h, device="cuda", dtype=torch.bfloat16)
    w = torch.ones(h, device="cuda", dtype=torch.bfloat16)
    # read h, delta; write h, fp8 q, scales
    return (lambda: ops.add_rmsnorm_quant(hx, dx, w, 1e-5, quant=True)), m * h * (2 + 2 + 2 + 1) + m * h // 32, "bytes"


def case_rope_kv(m, hq, hkv):
    d, ps = 128, 64
    qkv = torch.randn(m, (hq + 2 * hkv) * d, device="cuda", dtype=torch.bfloat16)
    pos = torch.randint(0, 8000, (m,), device="cuda", dtype=torch.int32)
    slots = torch.randperm(m, device="cuda").to(torch.int64)
    cs = ops.rope_table(8192, d, 5e5, "cuda")
    kc = torch.zeros((m + ps - 1) // ps, hkv, ps, d, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    fn = lambda: ops.rope_kv_write(qkv, pos, slots, cs, kc, vc, hq, hkv, d)
    return fn, m * (hq + 2 * hkv) * d * 2 * 2, "bytes"


def case_gdn_verify(reqs, n, hk, hv):
    from ..ops import gdn as G
    t = reqs * n
    q = torch.randn(t, hk, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(t, hk, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(t, hv, 128, device="cuda", dtype=torch.bfloat16)
    g = -torch.rand(t, hv, device="cuda")
    beta = torch.rand(t, hv, device="cuda")
    state = torch.randn(reqs, hv, 128, 128, device="cuda") * 0.01
    ts = torch.arange(reqs + 1, device="cuda", dtype=torch.int32) * n
    slot = torch.arange(reqs, device="cuda", dtype=torch.int32)
    fn = lambda: G.gdn_recurrent(q, k, v, g, beta, state, ts, slot, 0.088, write_state=False, stash=True)
    # state read once per request, q/k/v read, out + stash written
    return fn, reqs * hv * 128 * 128 * 4 + t * (2 * hk + hv) * 128 * 2 + t * hv * 128 * (2 + 8), "bytes"


def case_raster(ntri, size):
    from ..render import scene as S
    g = torch.Generator().manual_seed(0)
    tris = ((torch.rand(ntri, 3, 3, generator=g) - 0.5) * 0.2 + (torch.rand(ntri, 1, 3, generator=g) - 0.5)).cuda()
    cols = torch.rand(ntri, 3, generator=g).cuda()
    vp = S.view_projection(30, 20)
    fn = lambda: S.render(tris, cols, vp, size)
    return fn, ntri * 9 * 4 + size * size * (8 + 4), "bytes"


def case_topk(rows, v, k, with_lse=True):
    x = torch.randn(rows, v, device="cuda", dtype=torch.bfloat16)
    return (lambda: ops.topk_logprobs(x, k, with_lse=with_lse)), rows * v * 2, "bytes"


def case_sample_candidates(rows, v, kc, lse=False):
    """Device sampling stage 1: top-kc of x / T per 16384-column chunk (+ chunk max / sum-exp)."""
    x = torch.randn(rows, v, device="cuda", dtype=torch.bfloat16) * 2
    nch = int(ops.ext().sample_chunks(v))
    cv = torch.empty(rows, nch, kc, device="cuda")
    ci = torch.empty(rows, nch, kc, device="cuda", dtype=torch.int32)
    cms = torch.empty(rows, nch, 2, device="cuda") if lse else None
    temp = torch.full((rows,), 0.8, device="cuda")
    return (lambda: ops.ext().sample_candidates(x, kc, temp, 1, 0, cv, ci, cms, ops.status_tensor(x.device))), rows * v * 2, "bytes"


def case_spec_accept(R=64, N=64, D=6, ranks=8, nch=1, kc=64):
    """Device sampling stage 2: the seeded accept walk of 64 requests over 64-node trees (8 candidate lists)."""
    g = torch.Generator(device="cuda").manual_seed(0)
    cv = torch.randn(ranks, R * N, nch, kc, device="cuda", generator=g)
    ci = torch.randint(0, 128256, (ranks, R * N, nch, kc), device="cuda", dtype=torch.int32, generator=g)
    parent = torch.cat([torch.full((R, 1), -1, device="cuda", dtype=torch.int64),
                        (torch.arange(1, N, device="cuda") - 1)[None].expand(R, N - 1) // 8], 1).contiguous()
    tokens = ci[0, :N * R, 0, 0].view(R, N).long().contiguous()
    temp = torch.full((R,), 0.9, device="cuda")
    topk = torch.full((R,), 50, device="cuda", dtype=torch.int32)
    topp = torch.full((R,), 0.9, device="cuda")
    seed = torch.arange(R, device="cuda", dtype=torch.int64)
    com = torch.full((R,), 4600, device="cuda", dtype=torch.int64)
    acc = torch.empty(R, D, device="cuda", dtype=torch.int64)
    bonus = torch.empty(R, device="cuda", dtype=torch.int64)
    fn = lambda: ops.ext().spec_accept(cv, ci, ranks, nch, kc, tokens, parent, temp, topk, topp, seed, com, D, acc, bonus)
    return fn, cv.numel() * 8, "bytes"


def case_attention(which, impl, hq=64, hkv=8):
    q, kc, vc, meta = _verify_case(hq=hq, hkv=hkv)
    t, hq = q.shape[0], q.shape[1]
    g = hq // kc.shape[1]
    groups = cascade_groups(meta, 64)
    p1, p2 = build_items(meta, g, groups)
    rows = ops.attn_rows(impl)
    scale = 1 / math.sqrt(128)
    op = torch.empty(t, hq, 128, device="cuda", dtype=torch.bfloat16)
    lp = torch.full((t, hq), float("-inf"), device="cuda")
    oq = torch.empty(t, hq * 128, device="cuda", dtype=FP8_DTYPE)
    osc = torch.empty(hq, t, device="cuda")
    if which == "prefix":
        it, tl = pack_work(p1, g, "cuda", rows=rows)
        fn = lambda: ops.paged_attention(q, kc, vc, meta, scale, o_part=op, lse_part=lp, items=it, tiles=tl, impl=impl)
        flops = 4.0 * t * hq * 4096 * 128
    else:
        it, tl = pack_work(p2, g, "cuda", rows=rows)
        fn = lambda: ops.paged_attention(q, kc, vc, meta, scale, o_in=op, lse_in=lp, out_q=oq, out_qs=osc, items=it,
                                         tiles=tl, impl=impl)
        keys = sum(k - 4096 for k in meta.h_kv_len) / len(meta.h_kv_len)
        flops = 4.0 * t * hq * keys * 128  # includes masked tree keys
    return fn, flops, "bf16"


CASES = {
    "gemm_fp8_qkv": lambda: case_gemm_fp8(4096, 10240, 8192),
    "gemm_fp8_o": lambda: case_gemm_fp8(4096, 8192, 8192),
    "gemm_fp8_gate_up": lambda: case_gemm_fp8(4096, 57344, 8192),
    "gemm_fp8_gate_up_bn128": lambda: case_gemm_fp8(4096, 57344, 8192, bn=128),
    "gemm_fp8_down": lambda: case_gemm_fp8(4096, 8192, 28672),
    "gemm_fp8_gate_up_tp8": lambda: case_gemm_fp8(4096, 7168, 8192),
    "gemm_fp8_draft_m512": lambda: case_gemm_fp8(512, 57344, 8192),
    "gemm_bf16_lm_head": lambda: case_gemm_bf16(4096, 128256, 8192),
    "gate_up_swiglu_fused": lambda: case_gemm_swiglu(4096, 28672, 8192),
    "gate_up_swiglu_unfused": lambda: case_gemm_swiglu(4096, 28672, 8192, fused=False),
    "gate_up_swiglu_fused_tp8": lambda: case_gemm_swiglu(4096, 3584, 8192),
    "gate_up_swiglu_unfused_tp8": lambda: case_gemm_swiglu(4096, 3584, 8192, fused=False),
    # Mixtral-shaped MoE at EP8 (8192 tokens x top-2 over 8 experts: 2048 assignments per expert)
    "moe_gate_up_gather": lambda: case_moe_gate_up_gather(8192, 2048, 28672, 4096),
    "moe_gate_up_copy": lambda: case_moe_gate_up_gather(8192, 2048, 28672, 4096, gather=False),
    "moe_gate_up_gather_small": lambda: case_moe_gate_up_gather(640, 160, 28672, 4096),
    "moe_gate_up_copy_small": lambda: case_moe_gate_up_gather(640, 160, 28672, 4096, gather=False),
    "moe_combine": lambda: case_moe_combine(8192, 2, 4096),
    "attn_prefix_tc": lambda: case_attention("prefix", "tc"),
    "attn_prefix_mma": lambda: case_attention("prefix", "mma"),
    "attn_suffix_tc": lambda: case_attention("suffix", "tc"),
    "attn_suffix_mma": lambda: case_attention("suffix", "mma"),
    # per-rank shapes of tensor parallelism over 8 GPUs (Llama-3-70B, 64 requests x 64-node verify)
    "gemm_fp8_qkv_tp8": lambda: case_gemm_fp8(4096, 1280, 8192),
    "gemm_fp8_o_tp8": lambda: case_gemm_fp8(4096, 8192, 1024),
    "gemm_fp8_o_tp8_hws": lambda: case_gemm_fp8(4096, 8192, 1024, bn=256),   # explicit BN: hardware scaling
    "gemm_fp8_o_tp8_bn128": lambda: case_gemm_fp8(4096, 8192, 1024, bn=128),
    "gemm_fp8_down_tp8_bn128": lambda: case_gemm_fp8(4096, 8192, 3584, bn=128),
    "gemm_fp8_down_tp8": lambda: case_gemm_fp8(4096, 8192, 3584),
    "gemm_bf16_lm_head_tp8": lambda: case_gemm_bf16(4096, 16032, 8192),
    "gemm_scatter_local_o_tp8": lambda: case_gemm_scatter_local(4096, 8192, 1024),
    "gemm_scatter_local_o_tp8_lane": lambda: case_gemm_scatter_local(4096, 8192, 1024, bulk=False),
    "gemm_scatter_local_down_tp8": lambda: case_gemm_scatter_local(4096, 8192, 3584),
    "attn_prefix_tc_tp8": lambda: case_attention("prefix", "tc", hq=8, hkv=1),
    "attn_suffix_tc_tp8": lambda: case_attention("suffix", "tc", hq=8, hkv=1),
    "silu_mul_quant_tp8": lambda: case_silu_quant(4096, 3584),
    "silu_mul_quant": lambda: case_silu_quant(4096, 28672),
    "add_rmsnorm_quant": lambda: case_rmsnorm_quant(4096, 8192),
    "rope_kv_write": lambda: case_rope_kv(4096, 64, 8),
    "gdn_verify_64x8": lambda: case_gdn_verify(64, 8, 16, 32),
    "raster_100k_512": lambda: case_raster(100_000, 512),
    "topk8_draft_tp8": lambda: case_topk(512, 16032, 8),
    "topk8_draft": lambda: case_topk(512, 128256, 8),
    "argmax_verify": lambda: case_topk(4096, 128256, 1, with_lse=False),
    "sample_cand_verify": lambda: case_sample_candidates(4096, 128256, 64),
    "sample_cand_verify_tp8": lambda: case_sample_candidates(4096, 16032, 64),
    "sample_cand_k16_verify": lambda: case_sample_candidates(4096, 128256, 16),
    "sample_cand_top8_lse_draft": lambda: case_sample_candidates(512, 128256, 8, lse=True),
    "sample_cand_top8_lse_draft_tp8": lambda: case_sample_candidates(512, 16032, 8, lse=True),
    "spec_accept_64x64": lambda: case_spec_accept(),
    # draft-round shapes (512 = 64 requests x top-8 frontier)
    "gemm_fp8_draft_qkv_tp8": lambda: case_gemm_fp8(512, 1280, 8192),
    "gemm_fp8_draft_gate_up_tp8": lambda: case_gemm_fp8(512, 7168, 8192),
    "gemm_fp8_draft_fc": lambda: case_gemm_fp8(512, 8192, 16384),
    "gemm_bf16_draft_lm_head_tp8": lambda: case_gemm_bf16(512, 16032, 8192),
}


# ------------------------------------------------------------------------------------------------
# reference arms: the reference's own Triton kernels, unmodified, timed at the same shapes as ours
# ------------------------------------------------------------------------------------------------

REF_ROOT = os.path.join(ROOT, "baseline", "_ref")


def _ref_module(rel: str, name: str):
    """Import one of the reference's kernel files by path from its unmodified checkout under baseline/_ref
    (the reference is not pip-installable; its Triton kernels import only torch and triton)."""
    import importlib.util
    path = os.path.join(REF_ROOT, rel)
    if not os.path.exists(path):
        raise FileNotFoundError(f"reference kernel file missing: {path}")
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def ref_pair_topk(rows, v, k):
    """top-k of bf16 logits / T per row. Ours: csrc/topk.cu (values are log-probabilities: the kernel also
    forms each row's logsumexp). Reference: docker/opt/v5/topkbf_normcfg/topkbf/kopt_topkbf.py
    topk_scaled_bf16 (two Triton stages + torch.topk on the k slots)."""
    ref = _ref_module("docker/opt/v5/topkbf_normcfg/topkbf/kopt_topkbf.py", "ref_kopt_topkbf")
    x = torch.randn(rows, v, device="cuda", dtype=torch.bfloat16) * 2
    t = torch.full((rows, 1), 0.8, device="cuda")
    ours = lambda: ops.topk_logprobs(x, k, 0.8, with_lse=True)
    theirs = lambda: ref.topk_scaled_bf16(x, t, k)
    assert ref.kernel_eligible(x, t.reshape(-1), k) is None, "reference kernel would fall back to torch"
    lp, idx, _ = ours()
    rv, ri = theirs()
    same = bool(torch.equal(idx, ri))
    return ours, theirs, rows * v * 2, {"same_indices": same}


def ref_pair_verify_candidates(rows, v, k):
    """Verify-row target candidates. Ours: sample_candidates (exact top-64 of x / T per 16384-column chunk,
    what the device accept kernel merges). Reference: topk_scaled_bf16 with k = 20 (its verify target-probs
    top-k, kopt_topkbf.py:353-399)."""
    ref = _ref_module("docker/opt/v5/topkbf_normcfg/topkbf/kopt_topkbf.py", "ref_kopt_topkbf")
    x = torch.randn(rows, v, device="cuda", dtype=torch.bfloat16) * 2
    t = torch.full((rows, 1), 0.8, device="cuda")
    nch = int(ops.ext().sample_chunks(v))
    cv = torch.empty(rows, nch, 64, device="cuda")
    ci = torch.empty(rows, nch, 64, device="cuda", dtype=torch.int32)
    ours = lambda: ops.ext().sample_candidates(x, 64, t.reshape(-1), 1, 0, cv, ci, None, ops.status_tensor(x.device))
    theirs = lambda: ref.topk_scaled_bf16(x, t, k)
    return ours, theirs, rows * v * 2, {"ours": "per-chunk top-64 lists", "theirs": f"row top-{k}"}


def ref_pair_gdn_verify(reqs, n, hk, hv):
    """GDN target verify of a draft window of n tokens per request (gates included). Ours: csrc/gdn.cu (fp32
    state [slots, HV, K, V], per-token recurrence with stash). Reference: docker/opt/kern/braw/kernels.py
    gdn_b_verify (chunked WY/UT form on tensor cores, bf16 state [slots, HV, V, K], fp32 stash)."""
    from ..ops import gdn as G
    ref = _ref_module("docker/opt/kern/braw/kernels.py", "ref_braw")
    t = reqs * n
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(t, hk, 128, device="cuda", dtype=torch.bfloat16, generator=g)
    k = torch.randn(t, hk, 128, device="cuda", dtype=torch.bfloat16, generator=g)
    v = torch.randn(t, hv, 128, device="cuda", dtype=torch.bfloat16, generator=g)
    a = torch.randn(t, hv, device="cuda", dtype=torch.bfloat16, generator=g)
    b = torch.randn(t, hv, device="cuda", dtype=torch.bfloat16, generator=g)
    A_log = torch.rand(hv, device="cuda", generator=g)
    dt_bias = torch.rand(hv, device="cuda", generator=g)
    state32 = torch.randn(reqs, hv, 128, 128, device="cuda", generator=g) * 0.01
    state16 = state32.transpose(-1, -2).contiguous().to(torch.bfloat16)   # [slots, HV, V, K]
    ts = torch.arange(reqs + 1, device="cuda", dtype=torch.int32) * n
    slot = torch.arange(reqs, device="cuda", dtype=torch.int32)
    per_row = ref.stash_floats(hk, hv, 128, 128, n)
    stash = torch.empty(reqs, n, 1, 1, (per_row + n - 1) // n, device="cuda")
    scale = 128 ** -0.5

    def ours():
        gg, beta = G.gdn_gates(a, b, A_log, dt_bias)
        G.gdn_recurrent(q, k, v, gg, beta, state32, ts, slot, scale, write_state=False, stash=True)
    theirs = lambda: ref.gdn_b_verify(A_log, dt_bias, q, k, v, a, b, state16, slot, ts, stash, slot, scale=scale)
    byts = reqs * hv * 128 * 128 * 2 + t * (2 * hk + hv) * 128 * 2 + t * hv * 128 * 2
    return ours, theirs, byts, {"ours_state": "fp32", "theirs_state": "bf16"}


REF_CASES = {
    "ref_topk8_draft": lambda: ref_pair_topk(512, 128256, 8),
    "ref_topk16_verify": lambda: ref_pair_topk(4096, 128256, 16),
    "ref_verify_candidates_k20": lambda: ref_pair_verify_candidates(4096, 128256, 20),
    "ref_gdn_verify_64x8": lambda: ref_pair_gdn_verify(64, 8, 16, 32),
}


def run_reference(names, iters):
    """Time each (ours, reference) pair at the same shape: ms of both and reference / ours (> 1: ours faster).
    The byte count is the minimal HBM traffic of the op (bf16 state for the GDN row)."""
    pk = peaks()
    for name in names:
        ours, theirs, byts, extra = REF_CASES[name]()
        o_ms = time_it(ours, iters)
        r_ms = time_it(theirs, iters)
        ops.check_status()
        print(json.dumps({"kernel": name, "ours_ms": round(o_ms, 4), "reference_ms": round(r_ms, 4),
                          "reference_over_ours": round(r_ms / o_ms, 2),
                          "ours_frac_of_" + pk["src"] + "_hbm": round(byts / o_ms / 1e6 / pk["hbm_gbs"], 3),
                          "reference_frac_of_" + pk["src"] + "_hbm": round(byts / r_ms / 1e6 / pk["hbm_gbs"], 3),
                          **extra}))
        torch.cuda.empty_cache()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", nargs="*", default=None)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"],
                    help="reference: time the reference's own kernels against ours at the same shapes")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args.kernel or list(REF_CASES), args.iters)
        return
    args.kernel = args.kernel or list(CASES)
    pk = peaks()
    for name in args.kernel:
        fn, flops, kind = CASES[name]()
        ms = time_it(fn, args.iters)
        ops.check_status()
        if kind == "bytes":
            gbs = flops / ms / 1e6
            print(json.dumps({"kernel": name, "ms": round(ms, 4), "gb_s": round(gbs, 1),
                              "frac_of_" + pk["src"]: round(gbs / pk["hbm_gbs"], 3), "denominator_gbs": pk["hbm_gbs"]}))
        else:
            tf = flops / ms / 1e9
            denom = pk["bf16_tflops"] * (2 if kind == "fp8" else 1)
            print(json.dumps({"kernel": name, "ms": round(ms, 4), "tflops": round(tf, 1),
                              "frac_of_" + pk["src"]: round(tf / denom, 3),
                              "denominator_tflops": denom, "kind": kind}))
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
