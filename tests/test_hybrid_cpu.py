"""Hybrid GDN + attention model in the engine (CPU, fp32): chain speculation (GDN verify, then fold of the
accepted prefix) emits exactly the tokens of plain greedy decoding, across ragged batches, and state slots
are recycled."""
import torch

from phung5_b200.config import CacheConfig, DraftConfig, EngineConfig, SpecConfig, preset
from phung5_b200.engine.engine import LLMEngine
from phung5_b200.engine.oracle import SamplingParams


def _engine(spec_on: bool, num_draft: int = 3):
    cfg = preset("tiny-hybrid")
    spec = SpecConfig(enabled=spec_on, mode="chain", num_draft=num_draft)
    ecfg = EngineConfig(model=cfg, spec=spec, draft=DraftConfig(kind="model", num_layers=1),
                        cache=CacheConfig(page_size=16, num_pages=256, max_seqs=4))
    return LLMEngine(ecfg, device="cpu", dtype=torch.float32, max_context=1024)


def test_hybrid_chain_speculation_equals_greedy_decode():
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, 4096, (n,), generator=g).tolist() for n in (37, 20, 53)]
    base = _engine(False).generate(prompts, SamplingParams(max_new_tokens=14))
    eng = _engine(True)
    spec = eng.generate(prompts, SamplingParams(max_new_tokens=14))
    assert eng.stats["spec_steps"] > 0
    assert spec == base
    assert sorted(eng.gdn_pool.free) == [0, 1, 2, 3]           # every slot returned


def test_hybrid_rejects_tree_and_tensor_parallel():
    import pytest
    cfg = preset("tiny-hybrid")
    with pytest.raises(ValueError):
        LLMEngine(EngineConfig(model=cfg, spec=SpecConfig(mode="tree"), draft=DraftConfig(kind="model"),
                               cache=CacheConfig(page_size=16, num_pages=64, max_seqs=2)), device="cpu",
                  dtype=torch.float32)


def test_hybrid_full_acceptance_folds_accepted_chains():
    """A drafter that always proposes the target's own continuation: every step accepts the whole chain, so the
    GDN fold commits 1 + num_draft tokens per step; the output must still equal plain greedy decoding."""
    g = torch.Generator().manual_seed(12)
    prompts = [torch.randint(0, 4096, (n,), generator=g).tolist() for n in (29, 41)]
    base = _engine(False).generate(prompts, SamplingParams(max_new_tokens=16))
    seqs = [p + o for p, o in zip(prompts, base)]
    eng = _engine(True, num_draft=3)
    V = eng.cfg.model.vocab

    def oracle_draft(fb, hidden_in):
        rows = fb.logits_rows if fb.logits_rows is not None else torch.arange(fb.tokens.shape[0])
        logits = torch.zeros(rows.shape[0], V)
        for j, i in enumerate(rows.tolist()):
            p, t = int(fb.positions[i]), int(fb.tokens[i])
            nxt = next((s[p + 1] for s in seqs if p + 1 < len(s) and s[p] == t), 0)
            logits[j, nxt] = 10.0
        return logits, None
    eng._draft_forward = oracle_draft
    out = eng.generate(prompts, SamplingParams(max_new_tokens=16))
    assert out == base
    acc = [a for r in eng.reqs.values() for a in r.accepted]
    assert max(acc) == 3 and sum(acc) >= 2 * len(acc)         # long chains were accepted and folded
