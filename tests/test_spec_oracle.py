"""CPU fp32 check: CPU fp32 greedy speculative decode equals target-only greedy decode."""
import torch

from phung5_b200.config import SpecConfig, preset
from phung5_b200.engine.oracle import OracleSpecDecoder, SamplingParams, greedy_generate
from phung5_b200.models.reference import RefEagleHead, RefModel
from phung5_b200.weights.init import random_eagle_weights, random_weights


def _models(std=0.05):
    tcfg, dcfg = preset("tiny"), preset("tiny-draft")
    tw = random_weights(tcfg, seed=0, std=std)
    dw = random_weights(dcfg, seed=1, std=std)
    return RefModel(tcfg, tw), RefModel(dcfg, dw)


def _prompts(b=2, n=64, vocab=4096, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (n,), generator=g).tolist() for _ in range(b)]


def test_config1_chain_greedy_equals_target_greedy():
    target, draft = _models()
    dec = OracleSpecDecoder(target, draft, SpecConfig(mode="chain", num_draft=4))
    for i, p in enumerate(_prompts()):
        ref = greedy_generate(target, p, 64)
        st = dec.generate(p, SamplingParams(max_new_tokens=64), rid=i)
        assert st.out == ref


def test_self_draft_accepts_everything():
    # the target drafting for itself must accept all k drafts every step
    target, _ = _models()
    dec = OracleSpecDecoder(target, target, SpecConfig(mode="chain", num_draft=4))
    p = _prompts(1)[0]
    st = dec.generate(p, SamplingParams(max_new_tokens=20))
    assert st.out == greedy_generate(target, p, 20)
    assert all(a == 4 for a in st.accepted[:-1])


def test_tree_greedy_equals_target_greedy():
    target, draft = _models()
    dec = OracleSpecDecoder(target, draft, SpecConfig(mode="tree", tree_nodes=16, topk=4, depth=3))
    p = _prompts(1, n=32)[0]
    st = dec.generate(p, SamplingParams(max_new_tokens=24))
    assert st.out == greedy_generate(target, p, 24)


def test_tree_self_draft_accepts_full_depth():
    target, _ = _models()
    dec = OracleSpecDecoder(target, target, SpecConfig(mode="tree", tree_nodes=37, topk=4, depth=3))
    p = _prompts(1, n=32)[0]
    st = dec.generate(p, SamplingParams(max_new_tokens=20))
    assert st.out == greedy_generate(target, p, 20)
    assert max(st.accepted) == 3


def test_eagle_head_greedy_equals_target_greedy():
    tcfg = preset("tiny")
    tw = random_weights(tcfg, seed=0, std=0.05)
    ew = random_eagle_weights(tcfg, seed=3, std=0.05)
    target = RefModel(tcfg, tw)
    head = RefEagleHead(tcfg, ew, tw)
    for mode in ("chain", "tree"):
        dec = OracleSpecDecoder(target, head, SpecConfig(mode=mode, num_draft=3, tree_nodes=12, topk=3, depth=3))
        p = _prompts(1, n=16)[0]
        st = dec.generate(p, SamplingParams(max_new_tokens=16))
        assert st.out == greedy_generate(target, p, 16)
