"""The batched engine (paged KV, prefix cache, cascade attention, chain/tree speculation) against the
unbatched fp32 oracle, on CPU in fp32."""
import dataclasses

import pytest
import torch

from phung5_b200.config import CacheConfig, DraftConfig, EngineConfig, SpecConfig, preset
from phung5_b200.engine.engine import LLMEngine
from phung5_b200.engine.oracle import OracleSpecDecoder, SamplingParams, greedy_generate
from phung5_b200.models.eagle import pack_eagle
from phung5_b200.models.llama import pack_weights
from phung5_b200.models.reference import RefEagleHead, RefModel
from phung5_b200.weights.init import random_eagle_weights, random_weights

F32 = torch.float32


def _prompts(b, n, vocab=4096, seed=0, shared=0):
    g = torch.Generator().manual_seed(seed)
    pre = torch.randint(0, vocab, (shared,), generator=g).tolist()
    return [pre + torch.randint(0, vocab, (n - shared,), generator=g).tolist() for _ in range(b)]


def _engine(spec: SpecConfig, draft_kind="model", page_size=16, cascade=True):
    tcfg, dcfg = preset("tiny"), preset("tiny-draft")
    tw = random_weights(tcfg, seed=0, std=0.05)
    dw = random_weights(dcfg, seed=1, std=0.05)
    ecfg = EngineConfig(model=tcfg, spec=spec, draft=DraftConfig(kind=draft_kind),
                        cache=CacheConfig(page_size=page_size, num_pages=400, enable_cascade=cascade))
    target = pack_weights(tcfg, tw, "cpu", dtype=F32)
    if draft_kind == "eagle":
        ew = random_eagle_weights(tcfg, seed=3, std=0.05)
        drafter = pack_eagle(tcfg, ew, "cpu")
        drafter = dataclasses.replace(drafter, fc=dataclasses.replace(drafter.fc, w=drafter.fc.w.float()))
        drafter.layer.qkv.w = drafter.layer.qkv.w.float()
        for nm in ("o", "gu", "down"):
            getattr(drafter.layer, nm).w = getattr(drafter.layer, nm).w.float()
        drafter.layer.in_norm = drafter.layer.in_norm.float()
        drafter.layer.post_norm = drafter.layer.post_norm.float()
        drafter.norm = drafter.norm.float()
        ref_d = RefEagleHead(tcfg, ew, tw)
    else:
        drafter = pack_weights(dcfg, dw, "cpu", dtype=F32)
        ref_d = RefModel(dcfg, dw)
    eng = LLMEngine(ecfg, device="cpu", target=target, drafter=drafter, dtype=F32, max_context=2048)
    return eng, RefModel(tcfg, tw), ref_d


def test_config1_engine_chain_matches_target_greedy():
    eng, ref, _ = _engine(SpecConfig(mode="chain", num_draft=4))
    prompts = _prompts(2, 64)
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=64))
    for p, o in zip(prompts, outs):
        assert o == greedy_generate(ref, p, 64)


def test_engine_tree_shared_prefix_cascade():
    # 3 requests sharing 48 prompt tokens (3 pages of 16): prefix cache + cascade attention engaged
    eng, ref, _ = _engine(SpecConfig(mode="tree", tree_nodes=12, topk=3, depth=3))
    prompts = _prompts(3, 60, shared=48, seed=5)
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=20))
    for p, o in zip(prompts, outs):
        assert o == greedy_generate(ref, p, 20)
    assert eng.stats["prefill_tokens"] < 3 * 60  # shared pages were reused


def test_engine_eagle_tree_matches_oracle_decoder():
    spec = SpecConfig(mode="tree", tree_nodes=10, topk=3, depth=3)
    eng, ref, ref_d = _engine(spec, draft_kind="eagle")
    prompts = _prompts(2, 40, seed=7)
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=16))
    dec = OracleSpecDecoder(ref, ref_d, spec)
    for i, (p, o) in enumerate(zip(prompts, outs)):
        assert o == greedy_generate(ref, p, 16)
        st = dec.generate(p, SamplingParams(max_new_tokens=16), rid=i)
        assert o == st.out


def test_engine_geometric_accept_and_sampling_runs():
    eng, ref, _ = _engine(SpecConfig(mode="tree", tree_nodes=12, topk=3, depth=3, accept="geometric"))
    outs = eng.generate(_prompts(2, 40, seed=9), SamplingParams(max_new_tokens=12))
    assert all(len(o) == 12 for o in outs)
    eng2, _, _ = _engine(SpecConfig(mode="chain", num_draft=3))
    sp = SamplingParams(temperature=0.8, top_k=50, top_p=0.9, seed=123, max_new_tokens=12)
    a = eng2.generate(_prompts(2, 40, seed=11), sp)
    eng3, _, _ = _engine(SpecConfig(mode="chain", num_draft=3))
    b = eng3.generate(_prompts(2, 40, seed=11), sp)
    assert a == b  # seeded sampling is reproducible
