"""The engine on the GPU kernels against the fp32 oracle (small shapes)."""
import pytest
import torch

from phung5_b200 import ops
from phung5_b200.config import CacheConfig, DraftConfig, EngineConfig, SpecConfig, preset
from phung5_b200.engine.engine import LLMEngine
from phung5_b200.engine.oracle import SamplingParams, greedy_generate
from phung5_b200.models.llama import pack_weights
from phung5_b200.models.reference import RefModel
from phung5_b200.weights.init import random_weights

pytestmark = pytest.mark.gpu


def _prompts(b, n, vocab, seed=0, shared=0):
    g = torch.Generator().manual_seed(seed)
    pre = torch.randint(0, vocab, (shared,), generator=g).tolist()
    return [pre + torch.randint(0, vocab, (n - shared,), generator=g).tolist() for _ in range(b)]


@pytest.mark.parametrize("name,tol", [("small-bf16", 0.03), ("small-fp8", 0.12), ("small-moe-fp8", 0.15)])
def test_engine_prefill_logits_close_to_oracle(name, tol):
    from phung5_b200.engine.attn_meta import build_items, make_meta, pack_work
    from phung5_b200.models.llama import ForwardBatch
    cfg = preset(name)
    hf = random_weights(cfg, seed=0, std=0.02)
    ref = RefModel(cfg, hf)
    ecfg = EngineConfig(model=cfg, spec=SpecConfig(enabled=False), cache=CacheConfig(num_pages=256))
    eng = LLMEngine(ecfg, device="cuda", target=pack_weights(cfg, hf, "cuda"), max_context=4096)
    prompt = _prompts(1, 200, cfg.vocab, seed=1)[0]
    pages = eng.pool.prefix.alloc_pages(4)
    meta = make_meta([pages], [0], [200], None, True, "cuda")
    g = cfg.num_heads // cfg.num_kv_heads
    _, p2 = build_items(meta, g)
    slots = torch.tensor([pages[i // 64] * 64 + i % 64 for i in range(200)], device="cuda")
    fb = ForwardBatch(tokens=torch.tensor(prompt, device="cuda"), positions=torch.arange(200, device="cuda",
                      dtype=torch.int32), slots=slots, meta=meta, work2=pack_work(p2, g, "cuda"))
    logits, _ = eng.target.forward(fb)
    ops.check_status()
    rl, _ = ref.forward(torch.tensor(prompt), torch.arange(200), ref.new_cache())
    rows = (logits.float().cpu() - rl).norm(dim=-1) / rl.norm(dim=-1)
    if cfg.is_moe:
        # random-init routers have small logit gaps: the fp8 error of the attention output flips the
        # expert choice of a minority of tokens (whose rows then differ entirely); judge the typical row.
        # The MoE block itself matches the oracle on identical inputs (tests/test_kernels_gpu.py).
        err = rows.median().item()
    else:
        err = rows.max().item()
    assert err < tol, err
    # argmax agreement per position (a single greedy trajectory is fragile: near-tied random logits)
    agree = (logits.float().cpu().argmax(-1) == rl.argmax(-1)).float().mean().item()
    # MoE: a token whose routing flipped gets an unrelated row, which lowers its argmax agreement
    assert agree >= (0.95 if name == "small-bf16" else (0.7 if cfg.is_moe else 0.8)), agree


def _teacher_forced_argmax(eng, seq):
    """Target argmax after every position of `seq`, from one causal forward over fresh pages."""
    from phung5_b200.engine.attn_meta import build_items, make_meta, pack_work
    from phung5_b200.models.llama import ForwardBatch
    n = len(seq)
    pages = eng.pool.prefix.alloc_pages((n + 63) // 64)
    meta = make_meta([pages], [0], [n], None, True, "cuda")
    g = eng.target.hq // eng.target.hkv
    _, p2 = build_items(meta, g)
    slots = torch.tensor([pages[i // 64] * 64 + i % 64 for i in range(n)], device="cuda")
    fb = ForwardBatch(tokens=torch.tensor(seq, device="cuda"), positions=torch.arange(n, device="cuda",
                      dtype=torch.int32), slots=slots, meta=meta, work2=pack_work(p2, g, "cuda"))
    logits, _ = eng.target.forward(fb)
    eng.pool.alloc.release(pages)
    return logits.argmax(-1).tolist()


@pytest.mark.parametrize("name,mode", [("small-bf16", "tree"), ("small-fp8", "tree"), ("small-bf16", "chain")])
def test_engine_spec_tokens_are_target_greedy(name, mode):
    cfg = preset(name)
    hf = random_weights(cfg, seed=0, std=0.05)
    prompts = _prompts(4, 300, cfg.vocab, seed=2, shared=128)
    spec = SpecConfig(mode=mode, tree_nodes=32, topk=4, depth=4, num_draft=4)
    eng = LLMEngine(EngineConfig(model=cfg, spec=spec, draft=DraftConfig(kind="eagle"),
                                 cache=CacheConfig(num_pages=256)),
                    device="cuda", target=pack_weights(cfg, hf, "cuda"), max_context=4096)
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=32))
    ops.check_status()
    assert eng.stats["spec_steps"] > 0
    agree = total = 0
    for p, o in zip(prompts, outs):
        am = _teacher_forced_argmax(eng, p + o[:-1])
        pred = am[len(p) - 1:]
        agree += sum(a == b for a, b in zip(pred, o))
        total += len(o)
    # fp8 re-rounds every activation: a last-bit difference in one attention output (different key
    # tiling between verify and the teacher-forced pass) can move an fp8 value by 1/16, which flips
    # near-tied random-weight argmaxes; a wrong KV position or mask gives near-zero agreement instead.
    assert agree >= (0.95 if name == "small-bf16" else 0.75) * total, (agree, total)


def test_engine_geometric_synthetic_acceptance():
    cfg = preset("small-fp8")
    spec = SpecConfig(mode="tree", tree_nodes=64, topk=8, depth=6, accept="geometric")
    eng = LLMEngine(EngineConfig(model=cfg, spec=spec, draft=DraftConfig(kind="eagle"),
                                 cache=CacheConfig(num_pages=512)), device="cuda", max_context=4096)
    prompts = _prompts(16, 256, cfg.vocab, seed=3, shared=128)
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=40))
    ops.check_status()
    assert all(len(o) == 40 for o in outs)
    mean_acc = eng.stats["accepted"] / max(1, sum(len(r.accepted) for r in eng.reqs.values()))
    assert 1.2 < mean_acc < 3.0, mean_acc   # E[min(Geom(0.3), 6)] ~= 2.06


@pytest.mark.parametrize("accept,model,mode", [("greedy", "small-fp8", "tree"), ("geometric", "small-fp8", "tree"),
                                               ("greedy", "small-fp8", "chain"), ("geometric", "small-moe-fp8", "chain"),
                                               ("greedy", "small-moe-fp8", "tree")])
def test_graph_replayed_step_equals_eager_step(accept, model, mode, monkeypatch):
    """The CUDA-graph speculative step (static buffers, device-built metadata) must emit exactly the tokens
    of the eager step: same kernels on the same inputs. 16 requests sharing a 128-token prefix (cascade
    groups); tree and chain speculation, dense and MoE models (routing on the device inside the graph)."""
    cfg = preset(model)
    kw = dict(mode="tree", tree_nodes=64, topk=8, depth=6) if mode == "tree" else dict(mode="chain", num_draft=4)
    if accept == "geometric":
        kw["accept"] = "geometric"
    prompts = _prompts(16, 256, cfg.vocab, seed=4, shared=128)
    outs = {}
    for graphs in ("1", "0"):
        monkeypatch.setenv("PHX_GRAPHS", graphs)
        eng = LLMEngine(EngineConfig(model=cfg, spec=SpecConfig(**kw), draft=DraftConfig(kind="eagle"),
                                     cache=CacheConfig(num_pages=512)), device="cuda", max_context=4096)
        outs[graphs] = eng.generate(prompts, SamplingParams(max_new_tokens=48))
        ops.check_status()
        if graphs == "1":       # requests finish at different steps: one graph per live batch size
            assert eng.stats["graph_replays"] >= 5
        del eng
        torch.cuda.empty_cache()
    assert outs["1"] == outs["0"]


def test_hybrid_gdn_engine_chain_speculation_on_gpu():
    """Hybrid GDN + attention model on the GDN kernels: chain speculation with a drafter that proposes the
    target's own greedy continuation accepts whole chains (verify + fold of 1 + num_draft tokens per step)
    and reproduces plain decoding; bf16 near-ties may flip an occasional token."""
    cfg = preset("hybrid-gdn-small")
    g = torch.Generator().manual_seed(13)
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (200, 130, 257, 64)]

    def make(spec_on):
        spec = SpecConfig(enabled=spec_on, mode="chain", num_draft=4)
        return LLMEngine(EngineConfig(model=cfg, spec=spec, draft=DraftConfig(kind="model", num_layers=1),
                                      cache=CacheConfig(num_pages=128, max_seqs=8)), device="cuda", max_context=2048)
    base_eng = make(False)
    base = base_eng.generate(prompts, SamplingParams(max_new_tokens=24))
    ops.check_status()
    del base_eng
    seqs = [p + o for p, o in zip(prompts, base)]
    eng = make(True)

    def oracle_draft(fb, hidden_in):
        rows = fb.logits_rows if fb.logits_rows is not None else torch.arange(fb.tokens.shape[0], device="cuda")
        pos, tok = fb.positions.tolist(), fb.tokens.tolist()
        logits = torch.zeros(rows.shape[0], cfg.vocab, device="cuda", dtype=torch.bfloat16)
        for j, i in enumerate(rows.tolist()):
            nxt = next((s[pos[i] + 1] for s in seqs if pos[i] + 1 < len(s) and s[pos[i]] == tok[i]), 0)
            logits[j, nxt] = 10.0
        return logits, None
    eng._draft_forward = oracle_draft
    out = eng.generate(prompts, SamplingParams(max_new_tokens=24))
    ops.check_status()
    same = sum(a == b for o, b0 in zip(out, base) for a, b in zip(o, b0))
    assert same >= 0.9 * sum(len(b) for b in base), (out, base)
    acc = [a for r in eng.reqs.values() for a in r.accepted]
    assert sum(acc) >= 2 * len(acc)
