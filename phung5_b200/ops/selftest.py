"""Kernel self-test: every sm_100a kernel against its plain-torch definition on small shapes.

The reference's patch kits each carry a `--check` (compile, import probe, GPU bitwise self-test) with
distinct exit codes (e.g. docker/opt/v5/topkbf_normcfg/topkbf/apply_topkbf.py). Here the kernels are part
of the package, so one command checks them all on the current GPU:

    python -m phung5_b200.ops.selftest [--json out.json] [--check-bounds]
exit 0: all pass; 7: a kernel disagrees with its definition; 8: the extension is missing or no GPU.
--check-bounds runs every op with the bounds-check debug mode on (ops/check.py: index data validated
against its buffers, write-conflict and TMA-alignment rules) -- the small-shape bounds-checked run.
Each check uses the same tolerance as the test suite and reports its error metric.
"""
from __future__ import annotations

import argparse
import json
import math
import sys
import time
from typing import Callable, Dict, List, Tuple

import torch


def _rel(a, b) -> float:
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm().clamp(min=1e-12)).item()


def _checks() -> List[Tuple[str, Callable[[], Tuple[bool, float]]]]:
    from .. import ops
    from ..weights.quant import dequant_act_block, gemm_fp8_block_ref, quant_act_block, quant_weight_block
    dev = "cuda"

    def gemm_fp8():
        x = torch.randn(200, 512, device=dev)
        w = torch.randn(384, 512, device=dev) * 0.05
        xq, xs = quant_act_block(x)
        wq, ws = quant_weight_block(w)
        e = _rel(ops.gemm_fp8_block(xq, xs, wq, ws), gemm_fp8_block_ref(xq, xs, wq, ws))
        return e < 5e-3, e

    def gemm_bf16():
        x = torch.randn(300, 1024, device=dev).bfloat16()
        w = (torch.randn(640, 1024, device=dev) * 0.05).bfloat16()
        e = _rel(ops.gemm_bf16(x, w), x.float() @ w.float().t())
        return e < 5e-3, e

    def gemm_grouped():
        sizes = [100, 0, 37]
        x = torch.randn(sum(sizes), 256, device=dev)
        xq, xs = quant_act_block(x)
        ws_, ss_ = zip(*[quant_weight_block(torch.randn(256, 256, device=dev) * 0.05) for _ in sizes])
        off = torch.tensor([0, 100, 100, 137], dtype=torch.int32, device=dev)
        out = ops.gemm_grouped((xq, xs), torch.cat(ws_), torch.cat(ss_), off, 256)
        errs = [_rel(out[a:b], gemm_fp8_block_ref(xq[a:b], xs[:, a:b].contiguous(), ws_[g], ss_[g]))
                for g, (a, b) in enumerate([(0, 100), (100, 100), (100, 137)]) if b > a]
        return max(errs) < 5e-3, max(errs)

    def norm_quant():
        h = torch.randn(33, 1024, device=dev).bfloat16()
        d = torch.randn(33, 1024, device=dev).bfloat16()
        w = (1 + 0.1 * torch.randn(1024, device=dev)).bfloat16()
        hf = (h.float() + d.float()).bfloat16().float()
        q, s, y = ops.add_rmsnorm_quant(h, d, w, 1e-5, quant=True, out_bf16=True)
        ref = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-5) * w.float()
        e = max(_rel(y, ref), _rel(dequant_act_block(q, s), ref))
        return e < 4e-2, e

    def silu_quant():
        gu = torch.randn(37, 2 * 512, device=dev).bfloat16()
        q, s, y = ops.silu_mul_quant(gu, quant=True, out_bf16=True)
        ref = torch.nn.functional.silu(gu[:, :512].float()) * gu[:, 512:].float()
        e = max(_rel(y, ref), _rel(dequant_act_block(q, s), ref))
        return e < 4e-2, e

    def gemm_swiglu():
        from ..models.llama import interleave_gate_up
        x = torch.randn(150, 512, device=dev)
        w = torch.randn(512, 512, device=dev) * 0.05          # [gate; up], F = 256
        xq, xs = quant_act_block(x)
        wq, ws = quant_weight_block(w)
        gu = ops.gemm_fp8_block(xq, xs, wq, ws, bn=256, hw_scale=True)
        q_ref, s_ref, _ = ops.silu_mul_quant(gu, quant=True, out_bf16=False)
        q, s = ops.gemm_fp8_swiglu(xq, xs, *interleave_gate_up(wq, ws))
        e = (dequant_act_block(q, s) - dequant_act_block(q_ref, s_ref)).abs().max().item()
        return e == 0.0, e

    def moe_combine():
        y = torch.randn(40, 256, device=dev).bfloat16()
        pos = torch.randperm(40, device=dev).view(20, 2)
        w = torch.rand(20, 2, device=dev)
        local = torch.rand(20, 2, device=dev) > 0.3
        out = torch.empty(20, 256, device=dev, dtype=torch.bfloat16)
        ops.moe_combine(y, pos, w, local, out)
        ref = torch.where(local[..., None], y.float()[pos] * w[..., None], torch.zeros((), device=dev)).sum(1)
        e = _rel(out, ref) if ref.norm() > 0 else 0.0
        return e < 1e-2, e

    def topk():
        x = (torch.randn(64, 32000, device=dev) * 2).bfloat16()
        lp, idx, lse = ops.topk_logprobs(x, 8, temperature=0.7)
        xf = x.float() / 0.7
        rl = torch.logsumexp(xf, -1)
        rv, _ = torch.topk(xf, 8, dim=-1)
        e = max((lse - rl).abs().max().item(), (lp - (rv - rl[:, None])).abs().max().item())
        ok = e < 1e-3 and torch.equal(xf.gather(1, idx), rv)
        return ok, e

    def attention():
        from ..engine.attn_meta import build_items, make_meta, pack_work
        g = torch.Generator().manual_seed(0)
        hq, hkv, d, ps = 8, 2, 128, 64
        q_lens, prefix = [40, 9], [150, 64]
        need = [(p + n + ps - 1) // ps for p, n in zip(prefix, q_lens)]
        perm = torch.randperm(sum(need) + 1, generator=g).tolist()
        pages, k0 = [], 0
        for n in need:
            pages.append(perm[k0:k0 + n])
            k0 += n
        kc = torch.randn(len(perm), hkv, ps, d, generator=g).bfloat16()
        vc = torch.randn(len(perm), hkv, ps, d, generator=g).bfloat16()
        q = torch.randn(sum(q_lens), hq, d, generator=g).bfloat16()
        scale = 1 / math.sqrt(d)
        meta = make_meta(pages, prefix, q_lens, None, True, "cpu")
        _, p2 = build_items(meta, hq // hkv)
        ref = torch.zeros(q.shape[0], hq * d)
        ops.paged_attention(q, kc, vc, meta, scale, out=ref, items=p2)
        gm = make_meta(pages, prefix, q_lens, None, True, dev)
        out = torch.zeros(q.shape[0], hq * d, device=dev, dtype=torch.bfloat16)
        it, tl = pack_work(p2, hq // hkv, dev, rows=ops.attn_rows())
        ops.paged_attention(q.to(dev), kc.to(dev), vc.to(dev), gm, scale, out=out, items=it, tiles=tl)
        e = _rel(out, ref)
        return e < 1e-2, e

    def raster():
        from ..render import scene as S
        sc = {"geometries": [{"uuid": "g", "type": "BoxGeometry", "width": 1, "height": 0.6, "depth": 0.4}],
              "materials": [{"uuid": "m", "color": 0x3366CC}],
              "object": {"children": [{"geometry": "g", "material": "m"}]}}
        tris, cols = S.scene_triangles(sc)
        vp = S.view_projection(30, 20)
        a = S.render(tris, cols, vp, 96)
        b = S.render(tris.to(dev), cols.to(dev), vp, 96).cpu()
        diff = (a.int() - b.int()).abs()
        frac = (diff.amax(-1) > 1).float().mean().item()
        return frac < 0.01, frac

    def gemm_split():
        x = torch.randn(512, 4096, device=dev)
        w = torch.randn(1280, 4096, device=dev) * 0.05
        xq, xs = quant_act_block(x)
        wq, ws = quant_weight_block(w)
        ref = gemm_fp8_block_ref(xq, xs, wq, ws)
        e = max(_rel(ops.gemm_fp8_block(xq, xs, wq, ws, bn=256, hw_scale=True, split=s), ref) for s in (0, 5))
        return e < 5e-3, e

    def argmax():
        x = (torch.randn(300, 128256, device=dev) * 2).bfloat16()
        v, idx, _ = ops.topk_logprobs(x, 1, with_lse=False)
        ok = torch.equal(v[:, 0], x.float().max(-1).values) and torch.equal(x.float().gather(1, idx)[:, 0], v[:, 0])
        return ok, 0.0 if ok else 1.0

    def rope_kv():
        hq, hkv, d, ps = 8, 2, 128, 64
        qkv = torch.randn(37, (hq + 2 * hkv) * d, device=dev).bfloat16()
        pos = torch.randint(0, 4000, (37,), device=dev, dtype=torch.int32)
        slots = torch.randperm(10 * ps, device=dev)[:37].to(torch.int64)
        cs = ops.rope_table(4096, d, 5e5, dev)
        kc = torch.zeros(10, hkv, ps, d, device=dev, dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        qo = ops.rope_kv_write(qkv, pos, slots, cs, kc, vc, hq, hkv, d)
        kc2, vc2 = kc.cpu().zero_(), vc.cpu().zero_()
        qo2 = ops.rope_kv_write(qkv.cpu(), pos.cpu(), slots.cpu(), cs.cpu(), kc2, vc2, hq, hkv, d)
        e = max(_rel(qo, qo2), _rel(kc, kc2))
        return e < 1e-2 and torch.equal(vc.cpu(), vc2), e

    def gdn_verify():
        from . import gdn as G
        lens = [5, 0, 19, 1]
        ts = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
        t = int(ts[-1])
        q = torch.randn(t, 2, 128).bfloat16()
        k = torch.randn(t, 2, 128).bfloat16()
        v = torch.randn(t, 4, 128).bfloat16()
        gg, beta = -torch.rand(t, 4) * 0.5, torch.rand(t, 4)
        slot = torch.tensor([3, 0, 1, 2], dtype=torch.int32)
        st = torch.randn(4, 4, 128, 128) * 0.02
        st_c, st_g = st.clone(), st.to(dev)
        o_c, _ = G.gdn_recurrent(q.float(), k.float(), v.float(), gg, beta, st_c, ts, slot, 0.088, True)
        o_g, _ = G.gdn_recurrent(q.to(dev), k.to(dev), v.to(dev), gg.to(dev), beta.to(dev), st_g, ts.to(dev),
                                 slot.to(dev), 0.088, True)
        e = max(_rel(o_g, o_c), _rel(st_g, st_c))
        return e < 2e-2, e

    def sample_candidates():
        rows, V, kc = 6, 40000, 16
        x = (torch.randn(rows, V, device=dev) * 2).bfloat16()
        temp = torch.full((rows,), 0.8, device=dev)
        nch = int(ops.ext().sample_chunks(V))
        cv = torch.empty(rows, nch, kc, device=dev)
        ci = torch.empty(rows, nch, kc, device=dev, dtype=torch.int32)
        ops.ext().sample_candidates(x, kc, temp, 1, 0, cv, ci, None, ops.status_tensor(x.device))
        xf = x.float() / 0.8
        ok = True
        for c in range(nch):
            a, b = c * 16384, min(V, (c + 1) * 16384)
            want = sorted(torch.topk(xf[:, a:b], kc, dim=-1).values.flatten().tolist())
            got = sorted(cv[:, c].flatten().tolist())
            ok &= want == got
        return ok, 0.0 if ok else 1.0

    return [("gemm_fp8_block", gemm_fp8), ("gemm_bf16", gemm_bf16), ("gemm_grouped", gemm_grouped),
            ("gemm_split_k", gemm_split), ("add_rmsnorm_quant", norm_quant), ("silu_mul_quant", silu_quant),
            ("topk_logprobs", topk), ("argmax", argmax), ("paged_attention", attention), ("raster", raster),
            ("gemm_fp8_swiglu", gemm_swiglu), ("moe_combine", moe_combine), ("rope_kv_write", rope_kv),
            ("gdn_recurrent", gdn_verify), ("sample_candidates", sample_candidates)]


def run() -> Dict[str, dict]:
    from .. import ops
    out = {}
    for name, fn in _checks():
        t0 = time.perf_counter()
        try:
            ok, metric = fn()
            torch.cuda.synchronize()
            ops.check_status()
            out[name] = {"ok": bool(ok), "metric": float(metric), "ms": round(1e3 * (time.perf_counter() - t0), 1)}
        except Exception as e:  # noqa: BLE001 - reported per kernel
            out[name] = {"ok": False, "error": f"{type(e).__name__}: {str(e)[:200]}"}
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--json")
    ap.add_argument("--check-bounds", action="store_true")
    args = ap.parse_args(argv)
    if args.check_bounds:
        from . import check
        check.ON[0] = True
    if not torch.cuda.is_available():
        print("selftest: no CUDA device", file=sys.stderr)
        return 8
    try:
        from .. import ops
        ops.ext()
    except Exception as e:  # noqa: BLE001
        print(f"selftest: extension unavailable: {e}", file=sys.stderr)
        return 8
    res = run()
    for k, v in res.items():
        print(f"{k:20s} {'PASS' if v['ok'] else 'FAIL'} {v.get('metric', v.get('error'))}")
    if args.json:
        with open(args.json, "w") as f:
            json.dump(res, f, indent=1)
    return 0 if all(v["ok"] for v in res.values()) else 7


if __name__ == "__main__":
    sys.exit(main())
