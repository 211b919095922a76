"""Negative controls: deliberately wrong variants of the exact parts must be caught by the same checks the suite
relies on, so a passing check means something (CPU, fp32).

- speculative decoding accepting drafts without checking the target -> output differs from target greedy;
- a verify KV move that skips the accepted nodes -> output differs;
- tree attention run with a causal mask instead of the ancestor mask -> differs from the dense reference;
- the cascade's second pass without its pass-1 seed -> differs from the single-pass result.
"""
import math

import torch

from phung5_b200.config import SpecConfig
from phung5_b200.engine.oracle import SamplingParams, greedy_generate
from tests.test_engine_cpu import _engine, _prompts
from tests.test_ops_cpu import _run
from tests.test_kernels_gpu import _paged_case


def _accept_without_checking(self, logits, tokens, parent, ngeo):
    """Wrong: the first child at every depth is accepted, whatever the target predicts."""
    R, N, D = tokens.shape[0], self.N, self.D
    cur = torch.zeros(R, dtype=torch.int64)
    acc = torch.full((R, D), -1, dtype=torch.int64)
    nidx = torch.arange(N)[None, :]
    tgt = self.vocab.argmax(logits.reshape(R * N, -1)).reshape(R, N)
    for d in range(1, D + 1):
        kids = parent == cur[:, None]
        has = kids.any(1)
        first = torch.where(kids, nidx.expand(R, N), torch.full_like(tokens, N)).min(1).values
        acc[:, d - 1] = torch.where(has, first, torch.full_like(first, -1))
        cur = torch.where(has, first, cur)
    return acc, tgt.gather(1, cur[:, None])[:, 0]


def test_wrong_acceptance_is_caught(monkeypatch):
    eng, ref, _ = _engine(SpecConfig(mode="chain", num_draft=4))
    monkeypatch.setattr(type(eng), "_accept_static", _accept_without_checking)
    prompts = _prompts(2, 64)
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=32))
    assert any(o != greedy_generate(ref, p, 32) for p, o in zip(prompts, outs))


def _oracle_drafter(eng, seqs):
    """A drafter that proposes each sequence's own greedy continuation (writes no target KV)."""
    V = eng.cfg.model.vocab

    def draft(fb, hidden_in):
        rows = fb.logits_rows if fb.logits_rows is not None else torch.arange(fb.tokens.shape[0])
        logits = torch.full((rows.shape[0], V), -10.0)
        for j, i in enumerate(rows.tolist()):
            p, t = int(fb.positions[i]), int(fb.tokens[i])
            logits[j, next((s[p + 1] for s in seqs if p + 1 < len(s) and s[p] == t), 0)] = 10.0
        return logits, None
    return draft


def test_skipped_kv_move_is_caught(monkeypatch):
    """With a drafter that is always right, the accepted top-1 chain sits at tree nodes 1, K+1, ... and its KV
    must be moved to the committed positions; a step that skips the move leaves other nodes' KV there."""
    prompts = _prompts(2, 48, seed=5)
    outs = {}
    for broken in (False, True):
        eng, ref, _ = _engine(SpecConfig(mode="tree", tree_nodes=12, topk=3, depth=3), draft_kind="model")
        seqs = [p + greedy_generate(ref, p, 40) for p in prompts]
        eng._draft_forward = _oracle_drafter(eng, seqs)
        if broken:
            monkeypatch.setattr(eng.pool, "move_slots", lambda src, dst: None)
        outs[broken] = eng.generate(prompts, SamplingParams(max_new_tokens=40))
        assert max(a for r in eng.reqs.values() for a in r.accepted) == 3
    assert outs[False] == [s[len(p):] for s, p in zip(seqs, prompts)]      # the correct step passes the check
    assert outs[True] != outs[False]                                        # the broken one is caught


def test_causal_mask_in_place_of_tree_mask_is_caught():
    import dataclasses
    q, kc, vc, meta = _paged_case(3, [64, 17], [300, 1024], tree=True)
    good = _run(q, kc, vc, meta, None)
    bad = _run(q, kc, vc, dataclasses.replace(meta, causal=True, tree=None), None)
    assert (good - bad).abs().max() > 1e-2


def test_cascade_without_seed_is_caught():
    from phung5_b200 import ops
    from phung5_b200.engine.attn_meta import build_items, cascade_groups
    q, kc, vc, meta = _paged_case(4, [64, 64, 9], [640, 700, 520], tree=True, shared_pages=8)
    single = _run(q, kc, vc, meta, None)
    groups = cascade_groups(meta, 64)
    hq, hkv, t = q.shape[1], kc.shape[1], q.shape[0]
    _, p2 = build_items(meta, hq // hkv, groups)
    out = torch.zeros(t, hq * 128)
    ops.paged_attention(q, kc, vc, meta, 1 / math.sqrt(128), out=out, items=p2)   # pass 2 alone, no seed
    assert (single - out).abs().max() > 1e-2
