"""Bounds-check debug mode (ops/check.py): each rule rejects a seeded bad index before the op runs, and a whole
engine run with the checks on raises nothing and emits the same tokens as without them."""
import pytest
import torch

from phung5_b200 import ops
from phung5_b200.config import CacheConfig, DraftConfig, EngineConfig, SpecConfig, preset
from phung5_b200.engine.attn_meta import build_items, make_meta, pack_work
from phung5_b200.engine.engine import LLMEngine
from phung5_b200.engine.oracle import SamplingParams
from phung5_b200.models.llama import pack_weights
from phung5_b200.ops import check
from phung5_b200.ops.check import BoundsError, bounds_checks
from phung5_b200.weights.init import random_weights
from phung5_b200.weights.quant import quant_act_block


def _rope_args(m=4, hq=2, hkv=1, d=8, pages=3, ps=4):
    qkv = torch.randn(m, (hq + 2 * hkv) * d)
    pos = torch.arange(m, dtype=torch.int32)
    cs = ops.rope_table(16, d, 10000.0, "cpu")
    kc = torch.zeros(pages, hkv, ps, d)
    vc = torch.zeros_like(kc)
    return qkv, pos, cs, kc, vc, hq, hkv, d


def test_rope_kv_write_rejects_bad_slots_and_positions():
    qkv, pos, cs, kc, vc, hq, hkv, d = _rope_args()
    with bounds_checks():
        ops.rope_kv_write(qkv, pos, torch.tensor([0, 5, -1, 11]), cs, kc, vc, hq, hkv, d)      # fine
        with pytest.raises(BoundsError, match=r"slots\[1\] = 12 outside \[0, 12\)"):
            ops.rope_kv_write(qkv, pos, torch.tensor([0, 12, 1, 2]), cs, kc, vc, hq, hkv, d)
        with pytest.raises(BoundsError, match="appears more than once"):
            ops.rope_kv_write(qkv, pos, torch.tensor([3, 4, 3, -1]), cs, kc, vc, hq, hkv, d)
        with pytest.raises(BoundsError, match=r"pos\[2\] = 16"):
            ops.rope_kv_write(qkv, torch.tensor([0, 1, 16, 2], dtype=torch.int32), None, cs, kc, vc, hq, hkv, d)
    # off: the same bad slot reaches the op (its CPU definition raises an indexing error of its own)
    with pytest.raises(IndexError):
        ops.rope_kv_write(qkv, pos, torch.tensor([0, 12, 1, 2]), cs, kc, vc, hq, hkv, d)


def _attn_case(ps=4):
    # two requests: 6 and 5 committed keys, 2 new tokens each; request 1's pages are 3 and 4
    meta = make_meta([[0, 1, 2], [3, 4]], [6, 5], [2, 2], None, True, "cpu")
    _, p2 = build_items(meta, 2)
    it, tl = pack_work(p2, 2, "cpu", rows=64)
    q = torch.randn(4, 4, 8)
    kc = torch.randn(5, 2, ps, 8)
    return q, kc, meta, it, tl


def test_attention_checks_pages_keys_items_and_tiles():
    q, kc, meta, it, tl = _attn_case()
    vc = torch.randn_like(kc)
    out = torch.zeros(4, 4 * 8)
    with bounds_checks():
        ops.paged_attention(q, kc, vc, meta, 0.3, out=out, items=it, tiles=tl)                 # fine
        bad = make_meta([[0, 1, 2], [3, 7]], [6, 5], [2, 2], None, True, "cpu")
        with pytest.raises(BoundsError, match=r"pages\[4\] = 7 outside \[0, 5\)"):
            ops.paged_attention(q, kc, vc, bad, 0.3, out=out, items=it, tiles=tl)
        it2 = it.clone()
        it2[1, 4] = 9                       # request 1 holds 2 pages of 4 keys
        with pytest.raises(BoundsError, match=r"keys \[0, 9\) outside request 1's 2 pages"):
            ops.paged_attention(q, kc, vc, meta, 0.3, out=out, items=it2, tiles=tl)
        it3 = it.clone()
        it3[1, 0] = 1                       # item 1 now starts inside item 0's rows
        with pytest.raises(BoundsError, match="rows"):
            ops.paged_attention(q, kc, vc, meta, 0.3, out=out, items=it3, tiles=tl)
        ti, tr, nt = tl
        with pytest.raises(BoundsError, match="repeats item 0"):
            ops.paged_attention(q, kc, vc, meta, 0.3, out=out, items=it, tiles=(ti.clone().fill_(0), tr, nt))
        with pytest.raises(BoundsError, match="tile_item"):
            ops.paged_attention(q, kc, vc, meta, 0.3, out=out, items=it, tiles=(ti + 5, tr, nt))


def test_overlapping_work_items_are_a_race():
    q, kc, meta, it, tl = _attn_case()
    both = torch.cat([it, it[:1]])         # item 0 twice: two CTAs would write the same output rows
    with bounds_checks(), pytest.raises(BoundsError, match="both write query rows"):
        check.attention(q, kc, meta, both, None, 2, 64)


def test_grouped_gemm_offsets_and_rows():
    x = torch.randn(10, 16)
    w = torch.randn(3 * 8, 16)
    with bounds_checks():
        ops.gemm_grouped(x, w, None, torch.tensor([0, 4, 4, 10], dtype=torch.int32), 8)
        with pytest.raises(BoundsError, match="decreases"):
            ops.gemm_grouped(x, w, None, torch.tensor([0, 6, 4, 10], dtype=torch.int32), 8)
        with pytest.raises(BoundsError, match=r"offsets\[3\] = 11"):
            ops.gemm_grouped(x, w, None, torch.tensor([0, 4, 4, 11], dtype=torch.int32), 8)
        with pytest.raises(BoundsError, match="for 3 groups"):
            ops.gemm_grouped(x, w, None, torch.tensor([0, 4, 10], dtype=torch.int32), 8)
        with pytest.raises(BoundsError, match=r"rows\[1\] = 10"):
            check.gemm_grouped(10, w, 8, torch.tensor([0, 1, 2, 3]), torch.tensor([0, 10, 2]))


def test_moe_combine_positions():
    y = torch.randn(6, 8)
    pos = torch.tensor([[0, 5], [2, 6]])
    w = torch.ones(2, 2)
    out = torch.zeros(2, 8)
    with bounds_checks():
        ops.moe_combine(y, pos, w, torch.tensor([[True, True], [True, False]]), out)   # pos 6 is not local
        with pytest.raises(BoundsError, match=r"= 6 outside \[0, 6\)"):
            ops.moe_combine(y, pos, w, torch.ones(2, 2, dtype=torch.bool), out)


def test_spec_accept_tree_order_and_topk_checked_before_launch():
    R, N, V = 2, 4, 32
    logits = torch.randn(R * N, V)
    tokens = torch.randint(0, V, (R, N))
    temp = torch.tensor([1.0, 0.0])
    topk = torch.tensor([4, 0], dtype=torch.int32)
    topp = torch.ones(R)
    seed = torch.zeros(R, dtype=torch.int64)
    com = torch.zeros(R, dtype=torch.int64)
    good = torch.tensor([[-1, 0, 0, 1], [-1, 0, 1, 2]])
    check.spec_sample_accept(logits, tokens, good, topk, temp, 3, 16, 0)
    with bounds_checks():
        with pytest.raises(BoundsError, match=r"parent\[1, 2\] = 3 is not an earlier node"):
            ops.spec_sample_accept(logits, tokens, torch.tensor([[-1, 0, 0, 1], [-1, 0, 3, 2]]), temp, topk, topp,
                                   seed, com, 3, 16)
        with pytest.raises(BoundsError, match="root"):
            ops.spec_sample_accept(logits, tokens, torch.tensor([[0, 0, 0, 1], [-1, 0, 1, 2]]), temp, topk, topp,
                                   seed, com, 3, 16)
        with pytest.raises(BoundsError, match=r"top_k \(sampled requests\)\[0\] = 17"):
            ops.spec_sample_accept(logits, tokens, good, temp, torch.tensor([17, 0], dtype=torch.int32), topp,
                                   seed, com, 3, 16)


def test_gemm_shapes_and_power_of_two_scales():
    x = torch.randn(8, 256)
    w = torch.randn(128, 256)
    xq, xs = quant_act_block(x)
    wq, _ = quant_act_block(w)
    wsb = torch.ones(1, 2)                 # weight scales: one per 128 x 128 block
    check.gemm_fp8_block(xq, xs, wq, wsb, torch.empty(8, 128), True)
    with pytest.raises(BoundsError, match="not a positive power of two"):
        check.gemm_fp8_block(xq, xs * 1.5, wq, wsb, torch.empty(8, 128), True)
    with pytest.raises(BoundsError, match=r"ws has shape \(2, 2\)"):
        check.gemm_fp8_block(xq, xs, wq, torch.ones(2, 2), torch.empty(8, 128), False)
    with pytest.raises(BoundsError, match="K = 200"):
        check.gemm_fp8_block(xq[:, :200], xs, wq[:, :200], wsb, torch.empty(8, 128), False)
    with bounds_checks(), pytest.raises(BoundsError, match="hidden 200"):
        ops.add_rmsnorm_quant(torch.randn(2, 200), None, torch.ones(200), 1e-6)
    with bounds_checks(), pytest.raises(BoundsError, match="width 300"):
        ops.silu_mul_quant(torch.randn(2, 300))


def test_engine_run_with_checks_matches_run_without():
    tcfg, dcfg = preset("tiny"), preset("tiny-draft")
    tw, dw = random_weights(tcfg, seed=0, std=0.05), random_weights(dcfg, seed=1, std=0.05)

    def run():
        ecfg = EngineConfig(model=tcfg, spec=SpecConfig(mode="tree", tree_nodes=12, topk=3, depth=3),
                            draft=DraftConfig(kind="model"),
                            cache=CacheConfig(page_size=16, num_pages=200, enable_cascade=True))
        eng = LLMEngine(ecfg, device="cpu", target=pack_weights(tcfg, tw, "cpu", dtype=torch.float32),
                        drafter=pack_weights(dcfg, dw, "cpu", dtype=torch.float32), dtype=torch.float32,
                        max_context=1024)
        g = torch.Generator().manual_seed(5)
        pre = torch.randint(0, 4096, (40,), generator=g).tolist()
        prompts = [pre + torch.randint(0, 4096, (8,), generator=g).tolist() for _ in range(3)]
        return eng.generate(prompts, SamplingParams(max_new_tokens=12))

    plain = run()
    n0 = check.CHECKS[0]
    with bounds_checks():
        checked = run()
    assert check.CHECKS[0] - n0 > 50          # every op of every forward went through the checks
    assert checked == plain
