"""Engine admission control and preemption: with a KV pool too small for every request at once, requests are
admitted while their pages fit, the most recently admitted ones are preempted when a step's pages do not fit,
and they resume after recomputing their committed tokens -- emitting exactly the tokens of an unconstrained run
(greedy: the target's greedy continuation; seeded sampling: the same draws)."""
import dataclasses

import torch

from phung5_b200.config import CacheConfig, DraftConfig, EngineConfig, SpecConfig, preset
from phung5_b200.engine.engine import LLMEngine
from phung5_b200.engine.oracle import SamplingParams, greedy_generate
from phung5_b200.models.llama import pack_weights
from phung5_b200.models.reference import RefModel
from phung5_b200.weights.init import random_weights

F32 = torch.float32


def _engine(spec, num_pages, max_running=256, cascade=True):
    tcfg, dcfg = preset("tiny"), preset("tiny-draft")
    tw, dw = random_weights(tcfg, seed=0, std=0.05), random_weights(dcfg, seed=1, std=0.05)
    ecfg = EngineConfig(model=tcfg, spec=spec, draft=DraftConfig(kind="model"),
                        cache=CacheConfig(page_size=16, num_pages=num_pages, enable_cascade=cascade),
                        max_running=max_running)
    eng = LLMEngine(ecfg, device="cpu", target=pack_weights(tcfg, tw, "cpu", dtype=F32),
                    drafter=pack_weights(dcfg, dw, "cpu", dtype=F32), dtype=F32, max_context=2048)
    return eng, RefModel(tcfg, tw)


def _prompts(b, n, shared=0, seed=0):
    g = torch.Generator().manual_seed(seed)
    pre = torch.randint(0, 4096, (shared,), generator=g).tolist()
    return [pre + torch.randint(0, 4096, (n - shared,), generator=g).tolist() for _ in range(b)]


def test_small_pool_preempts_and_resumes_with_identical_greedy_output():
    eng, ref = _engine(SpecConfig(mode="chain", num_draft=4), num_pages=22)
    prompts = _prompts(4, 60)
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=80))
    assert eng.stats["preempted"] > 0
    for p, o in zip(prompts, outs):
        assert o == greedy_generate(ref, p, 80)
    assert eng.pool.alloc.available() + len(eng.pool.prefix.lru) == eng.pool.num_pages - 1   # nothing leaked


def test_tree_speculation_with_shared_prefix_under_pressure():
    eng, ref = _engine(SpecConfig(mode="tree", tree_nodes=12, topk=3, depth=3), num_pages=24)
    prompts = _prompts(4, 56, shared=32, seed=3)
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=60))
    assert eng.stats["preempted"] > 0
    for p, o in zip(prompts, outs):
        assert o == greedy_generate(ref, p, 60)


def test_seeded_sampling_is_unchanged_by_preemption():
    params = [SamplingParams(max_new_tokens=48, temperature=0.8, top_k=20, top_p=0.9, seed=100 + i) for i in range(3)]
    prompts = _prompts(3, 40, seed=5)

    def run(pages):
        eng, _ = _engine(SpecConfig(mode="chain", num_draft=3), num_pages=pages)
        rids = [eng.add_request(p, sp) for p, sp in zip(prompts, params)]
        while eng.has_work():
            eng.step()
        return [eng.reqs[r].out for r in rids], eng.stats["preempted"]
    big, n0 = run(200)
    small, n1 = run(14)
    assert n0 == 0 and n1 > 0
    assert small == big


def test_max_running_caps_the_batch():
    eng, ref = _engine(SpecConfig(mode="chain", num_draft=2), num_pages=200, max_running=2)
    prompts = _prompts(5, 24, seed=9)
    rids = [eng.add_request(p, SamplingParams(max_new_tokens=20)) for p in prompts]
    peak = 0
    while eng.has_work():
        eng.step()
        peak = max(peak, len([r for r in eng.running if not r.finished]))
    assert peak == 2
    for p, r in zip(prompts, rids):
        assert eng.reqs[r].out == greedy_generate(ref, p, 20)
