"""CPU checks of the op definitions (the oracles the GPU kernels are tested against)."""
import math

import torch

from phung5_b200 import ops
from phung5_b200.engine.attn_meta import build_items, cascade_groups
from phung5_b200.weights.quant import gemm_fp8_block_ref, quant_act_block, quant_weight_block
from tests.test_kernels_gpu import _paged_case


def _run(q, kc, vc, meta, groups):
    hq, hkv = q.shape[1], kc.shape[1]
    t = q.shape[0]
    p1, p2 = build_items(meta, hq // hkv, groups)
    out = torch.zeros(t, hq * 128)
    op = torch.zeros(t, hq, 128)
    lp = torch.full((t, hq), float("-inf"))
    if p1:
        ops.paged_attention(q, kc, vc, meta, 1 / math.sqrt(128), o_part=op, lse_part=lp, items=p1)
    ops.paged_attention(q, kc, vc, meta, 1 / math.sqrt(128), o_in=op if p1 else None, lse_in=lp if p1 else None,
                        out=out, items=p2)
    return out


def test_cascade_equals_single_pass():
    q, kc, vc, meta = _paged_case(4, [64, 64, 9], [640, 700, 520], tree=True, shared_pages=8)
    groups = cascade_groups(meta, 64)
    assert groups == [(0, 2, 512)]
    a = _run(q, kc, vc, meta, None)
    b = _run(q, kc, vc, meta, groups)
    assert (a - b).abs().max() < 1e-4


def test_tree_mask_matches_dense_reference():
    # a token whose mask is only itself + root sees the committed prefix, the root and itself
    from phung5_b200.models.reference import attention
    q, kc, vc, meta = _paged_case(3, [64, 17], [300, 1024], tree=True)
    out = _run(q, kc, vc, meta, None)
    r = 1
    q0, n, plen = meta.h_q_start[r], 17, meta.h_prefix_len[r]
    pages = meta.h_pages[meta.h_page_indptr[r]:meta.h_page_indptr[r + 1]]
    keys = torch.arange(plen + n)
    k = kc[torch.tensor(pages)[keys // 64], :, keys % 64].float()
    v = vc[torch.tensor(pages)[keys // 64], :, keys % 64].float()
    bits = meta.tree[q0:q0 + n]
    mask = torch.ones(n, plen + n, dtype=torch.bool)
    for i in range(n):
        for j in range(n):
            mask[i, plen + j] = bool((int(bits[i]) >> j) & 1)
    ref = attention(q[q0:q0 + n].float(), k, v, mask, 1 / math.sqrt(128)).reshape(n, -1)
    assert (out[q0:q0 + n] - ref).abs().max() < 1e-4


def test_gemm_fp8_ref_close_to_dense():
    x = torch.randn(64, 512)
    w = torch.randn(256, 512) * 0.05
    xq, xs = quant_act_block(x)
    wq, ws = quant_weight_block(w)
    out = ops.gemm_fp8_block(xq, xs, wq, ws)
    dense = x @ w.t()
    assert ((out.float() - dense).norm() / dense.norm()) < 0.08


def test_pow2_block_scales_and_checkpoint_requant():
    """Block scales are the smallest power of two >= amax / 448 (exact UE8M0 values); a checkpoint with arbitrary
    fp32 scales is requantized once to power-of-two scales, within one e4m3 rounding of the original weight."""
    from phung5_b200.weights.quant import FP8_MAX, ensure_pow2, is_pow2, pow2_scale
    amax = torch.tensor([0.0, 448.0, 449.0, 1.0, 3e-30, 224.0 * 2 ** -20])
    s = pow2_scale(amax)
    assert is_pow2(s) and s[0] == 1 and s[1] == 1 and s[2] == 2 and s[5] == 2 ** -21
    assert ((amax / s) <= FP8_MAX).all() and ((amax / s)[1:] > FP8_MAX / 2).all()
    w = torch.randn(256, 384) * 0.03
    xq, xs = quant_act_block(torch.randn(8, 384))
    wq, ws = quant_weight_block(w)
    assert is_pow2(xs) and is_pow2(ws)
    assert ensure_pow2(wq, ws)[0] is wq                                     # already powers of two: unchanged
    ws_odd = ws * 0.77                                                      # a checkpoint's own scales
    q2, s2 = ensure_pow2(wq, ws_odd)
    assert is_pow2(s2)
    deq = lambda q, sc: q.float() * sc.repeat_interleave(128, 0).repeat_interleave(128, 1)
    orig = deq(wq, ws_odd)
    blk = orig.abs().view(2, 128, 3, 128).amax((1, 3)).repeat_interleave(128, 0).repeat_interleave(128, 1)
    assert ((deq(q2, s2) - orig).abs() / blk).max() <= 1 / 16 + 1e-6


def test_gate_up_interleave_layout():
    """128-row blocks of [gate; up] interleave as gate 0, up 0, gate 1, up 1, ... with their block scales."""
    from phung5_b200.models.llama import interleave_gate_up
    f, k = 384, 256
    w = torch.arange(2 * f, dtype=torch.float32)[:, None].expand(2 * f, k).contiguous()
    ws = torch.arange(2 * f // 128, dtype=torch.float32)[:, None].expand(2 * f // 128, k // 128).contiguous()
    w2, s2 = interleave_gate_up(w, ws)
    order = [r for j in range(f // 128) for r in list(range(128 * j, 128 * j + 128)) + list(range(f + 128 * j, f + 128 * j + 128))]
    assert torch.equal(w2[:, 0], torch.tensor(order, dtype=torch.float32))
    assert s2[:, 0].tolist() == [0, 3, 1, 4, 2, 5]


def test_loader_requantizes_non_pow2_checkpoint_scales():
    """An FP8 checkpoint whose weight_scale_inv values are not powers of two goes through the loader with every
    packed scale a power of two, and each packed weight stays within one e4m3 step of the checkpoint's."""
    from phung5_b200.config import preset
    from phung5_b200.models.llama import pack_weights
    from phung5_b200.models.reference import dequant_block_fp8
    from phung5_b200.weights.init import random_weights
    from phung5_b200.weights.quant import is_pow2
    cfg = preset("small-fp8")
    wd = random_weights(cfg, seed=1, std=0.02)
    for name in [n for n in wd if n.endswith("_scale_inv")]:
        wd[name] = wd[name] * 0.77                                # a checkpoint's own (non-power-of-two) scales
    pw = pack_weights(cfg, wd, "cpu")
    lw = pw.layers[0]
    for lin in (lw.qkv, lw.o, lw.gu, lw.down):
        assert is_pow2(lin.ws)
    p = "model.layers.0.self_attn.o_proj.weight"
    orig = dequant_block_fp8(wd[p], wd[p + "_scale_inv"])
    got = dequant_block_fp8(lw.o.w, lw.o.ws)
    n, k = orig.shape
    blk = orig.abs().view(n // 128, 128, k // 128, 128).amax((1, 3)).repeat_interleave(128, 0).repeat_interleave(128, 1)
    assert ((got - orig).abs() / blk).max() <= 1 / 16 + 1e-6


def test_gemm_table_lookup_and_switches(monkeypatch, tmp_path):
    """The per-shape GEMM table: M is bucketed to the nearest measured size at or above it (the largest bucket
    beyond), entries without a tile choice keep the kernel's heuristic, a caller's explicit choice wins, and
    PHX_GEMM_SPLIT=0 turns the automatic split-K tail off unless a caller asks for a split."""
    import json

    from phung5_b200 import ops
    from phung5_b200.ops import gemm_table as T
    table = {"m_buckets": [128, 512, 4096],
             "entries": {"fp8:1280:8192:512": {"bn": 256, "hws": True, "pair": False, "split": 0, "ms": 0.03},
                         "fp8:1280:8192:4096": {"ms": 0.07, "default_ms": 0.07},
                         "bf16:16032:8192:4096": {"bn": 256, "split": 1, "ms": 0.8}}}
    path = tmp_path / "table.json"
    path.write_text(json.dumps(table))
    monkeypatch.setattr(T, "PATH", str(path))
    monkeypatch.setattr(T, "_TABLE", {"loaded": False, "entries": {}, "buckets": []})
    assert T.lookup("fp8", 1280, 8192, 300)["bn"] == 256          # 300 -> bucket 512
    assert T.lookup("fp8", 1280, 8192, 2000) is None               # 2000 -> 4096: default kept
    assert T.lookup("fp8", 1280, 8192, 9000) is None               # beyond the last bucket -> 4096
    assert T.lookup("bf16", 16032, 8192, 9000)["split"] == 1
    assert ops._table_choice("fp8", 1280, 8192, 300, 0, None, None, True) == (256, True, False, 0)
    assert ops._table_choice("fp8", 1280, 8192, 300, 128, None, None, True)[0] == 128     # caller's BN wins
    assert ops._table_choice("bf16", 16032, 8192, 4096, 0, None, None, True)[3] == 1
    monkeypatch.setattr(ops, "GEMM_SPLIT", False)
    assert ops._table_choice("fp8", 1280, 8192, 2000, 0, None, None, True)[3] == 1         # no entry: split off
    assert ops._table_choice("fp8", 1280, 8192, 2000, 0, None, None, True, split=4)[3] == 4
