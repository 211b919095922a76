"""Unbatched CPU speculative decoder over the fp32 oracle models.

This is the reference path of the CPU fp32 speculative-decode check (target-only greedy vs speculative greedy must produce the
same tokens) and the behavioural oracle for the batched engine: the engine's per-request outputs are
checked token-for-token against `OracleSpecDecoder`.

Step structure (one speculative step of one request):
  1. draft: catch the drafter up on committed tokens, then propose a chain of k tokens or build an
     EAGLE-2 tree (engine/tree.py);
  2. verify: one target forward over all tree nodes (root = pending token) with the ancestor mask;
  3. accept: walk the tree with the accept rule (engine/sampling.py), keep the KV rows of the root
     and accepted nodes, emit accepted tokens + the bonus token, which becomes the next root.
This mirrors the reference's DFlash verify step (draft -> target verify -> target
probs -> accept -> commit), done per request in plain torch.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import torch

from ..config import SpecConfig
from ..models.reference import RefEagleHead, RefKV, RefModel, causal_mask
from .sampling import accept_tree, geometric_accept_len, seeded_coins, target_probs
from .tree import Tree, chain_tree, select_tree


@dataclass
class SamplingParams:
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    seed: int = 42
    max_new_tokens: int = 64
    stop_token_ids: tuple = ()      # generation ends at the first of these (not emitted); e.g. the EOS id


def _probs(logits: torch.Tensor, sp: SamplingParams) -> torch.Tensor:
    r = logits.shape[0]
    return target_probs(logits, torch.full((r,), sp.temperature), torch.full((r,), sp.top_k, dtype=torch.int64),
                        torch.full((r,), sp.top_p))


def greedy_generate(model: RefModel, prompt: List[int], n: int, embeds=None) -> List[int]:
    """Target-only greedy decode: prefill the prompt, then one token per forward. embeds: (rows, features)
    replacing those prompt rows' token embeddings (image inputs)."""
    kv = model.new_cache()
    toks = torch.tensor(prompt, dtype=torch.int64)
    logits, _ = model.forward(toks, torch.arange(len(prompt)), kv, embeds=embeds)
    out = [int(logits[-1].argmax())]
    while len(out) < n:
        pos = torch.tensor([kv.length()])
        logits, _ = model.forward(torch.tensor([out[-1]]), pos, kv)
        out.append(int(logits[-1].argmax()))
    return out


@dataclass
class _ReqState:
    committed: List[int]                 # prompt + emitted tokens that are in the target KV
    root: int                            # pending token (emitted, not yet in target KV)
    kv: RefKV
    dkv: RefKV
    last_hidden: Optional[torch.Tensor] = None   # target hidden at the last committed position
    out: List[int] = field(default_factory=list)
    steps: int = 0
    accepted: List[int] = field(default_factory=list)


class OracleSpecDecoder:
    """Speculative decoding with a standalone draft LM (chain or tree) or an EAGLE head."""

    def __init__(self, target: RefModel, drafter, spec: SpecConfig):
        self.target = target
        self.drafter = drafter
        self.spec = spec
        self.eagle = isinstance(drafter, RefEagleHead)

    # -- drafter helpers ---------------------------------------------------------------------
    def _draft_catch_up(self, st: _ReqState, hidden_seq: Optional[torch.Tensor]) -> torch.Tensor:
        """Feed the drafter every committed token it has not seen plus the root; return the logits
        after the root and (for EAGLE) the head's feature there."""
        seq = st.committed + [st.root]
        start = st.dkv.length()
        toks = torch.tensor(seq[start:], dtype=torch.int64)
        pos = torch.arange(start, len(seq))
        if self.eagle:
            # EAGLE input at position t pairs token x_t with the target feature of position t-1
            # (position 0 has no predecessor and gets a zero feature)
            h = hidden_seq
            if start == 0:
                h = torch.cat([torch.zeros_like(h[:1]), h], 0)
                hid = h[0: len(seq)]
            else:
                hid = h[start - 1: len(seq) - 1]
            logits, feat = self.drafter.forward(toks, hid, pos, st.dkv)
            return logits[-1], feat[-1]
        logits, _ = self.drafter.forward(toks, pos, st.dkv)
        return logits[-1], None

    def _draft_chain(self, st: _ReqState, hidden_seq) -> Tree:
        logits, feat = self._draft_catch_up(st, hidden_seq)
        drafts = []
        base = st.dkv.length()
        for i in range(self.spec.num_draft):
            tok = int(logits.argmax())
            drafts.append(tok)
            if i == self.spec.num_draft - 1:
                break
            pos = torch.tensor([base + i])
            if self.eagle:
                lg, f = self.drafter.forward(torch.tensor([tok]), feat[None], pos, st.dkv)
                logits, feat = lg[-1], f[-1]
            else:
                lg, _ = self.drafter.forward(torch.tensor([tok]), pos, st.dkv)
                logits = lg[-1]
        # drop the drafted tokens from the draft KV: only committed context stays
        st.dkv.truncate(base)
        return chain_tree(st.root, drafts)

    def _draft_tree(self, st: _ReqState, hidden_seq) -> Tree:
        sp = self.spec
        logits, feat = self._draft_catch_up(st, hidden_seq)
        base = st.dkv.length()
        lp = torch.log_softmax(logits.float(), -1)
        top = torch.topk(lp, sp.topk)
        c_tok, c_par, c_score, c_depth = [], [], [], []
        c_feat = []
        for j in range(sp.topk):
            c_tok.append(int(top.indices[j])); c_par.append(-1); c_score.append(float(top.values[j]))
            c_depth.append(1); c_feat.append(feat)
        frontier = list(range(sp.topk))
        for d in range(1, sp.depth):
            # run the drafter on the frontier nodes; each sees the committed context + its ancestors
            nodes = frontier
            def _anc(c):
                path, j = [], c
                while j >= 0:
                    path.append(j)
                    j = c_par[j]
                return path[::-1]
            anc = {}
            for c in nodes:
                for x in _anc(c):
                    anc[x] = _anc(x)
            # process every node on the frontier's paths in one masked forward
            allnodes = sorted(anc, key=lambda x: (c_depth[x], x))
            idx = {x: i for i, x in enumerate(allnodes)}
            n = len(allnodes)
            mask = torch.zeros(n, base + n, dtype=torch.bool)
            mask[:, :base] = True
            for x in allnodes:
                for a in anc[x]:
                    mask[idx[x], base + idx[a]] = True
            toks = torch.tensor([c_tok[x] for x in allnodes])
            pos = torch.tensor([base + c_depth[x] - 1 for x in allnodes])
            if self.eagle:
                hid = torch.stack([c_feat[x] for x in allnodes])
                lg, fe = self.drafter.forward(toks, hid, pos, st.dkv, mask)
            else:
                lg, fe = self.drafter.forward(toks, pos, st.dkv, mask)
            st.dkv.truncate(base)
            cands = []
            for c in nodes:
                lpc = torch.log_softmax(lg[idx[c]].float(), -1)
                tk = torch.topk(lpc, sp.topk)
                for j in range(sp.topk):
                    cands.append((c_score[c] + float(tk.values[j]), c, int(tk.indices[j]), fe[idx[c]]))
            cands.sort(key=lambda t: -t[0])
            new_front = []
            for score, par, tok, f in cands:
                c_tok.append(tok); c_par.append(par); c_score.append(score); c_depth.append(d + 1)
                c_feat.append(f)
                if len(new_front) < sp.topk:
                    new_front.append(len(c_tok) - 1)
            frontier = new_front
        return select_tree(st.root, c_tok, c_par, c_score, c_depth, sp.tree_nodes)

    # -- main loop -------------------------------------------------------------------------------
    def generate(self, prompt: List[int], sp: SamplingParams, rid: int = 0) -> _ReqState:
        tgt = self.target
        st = _ReqState(committed=list(prompt), root=-1, kv=tgt.new_cache(), dkv=self.drafter.new_cache())
        logits, hid = tgt.forward(torch.tensor(prompt), torch.arange(len(prompt)), st.kv)
        hidden_seq = hid
        probs = _probs(logits[-1:], sp)
        if sp.temperature <= 0:
            st.root = int(probs[0].argmax())
        else:
            u = seeded_coins(torch.tensor([sp.seed]), torch.tensor([len(prompt) - 1]), 1)[0, 0]
            from .sampling import sample_from
            st.root = int(sample_from(probs, u[None])[0])
        st.out.append(st.root)
        while len(st.out) < sp.max_new_tokens:
            tree = self._draft_tree(st, hidden_seq) if self.spec.mode == "tree" else self._draft_chain(st, hidden_seq)
            base = st.kv.length()
            n = tree.n
            mask = torch.zeros(n, base + n, dtype=torch.bool)
            mask[:, :base] = True
            mask[:, base:] = tree.ancestor_mask()
            logits, hid = tgt.forward(tree.tokens, base + tree.depth, st.kv, mask)
            probs = _probs(logits, sp)
            greedy = sp.temperature <= 0
            coins = final = None
            if not greedy:
                cc = seeded_coins(torch.tensor([sp.seed]), torch.tensor([base]), self.spec.depth + 1 + 1)[0]
                coins, final = cc[:-1], float(cc[-1])
            path, bonus = accept_tree(tree.tokens, tree.children(), probs, greedy, coins, final)
            if self.spec.accept == "geometric":
                nacc = int(geometric_accept_len(self.spec.accept_seed, torch.tensor([st.steps]),
                                                torch.tensor([rid]), self.spec.accept_p, self.spec.accept_cap)[0])
                # follow the first-child chain of the tree for the synthetic length
                kids = tree.children()
                path, cur = [], 0
                while len(path) < nacc and kids[cur]:
                    cur = kids[cur][0]
                    path.append(cur)
                bonus = int(probs[cur].argmax()) if greedy else bonus
            keep = [0] + path
            keep_idx = torch.tensor(list(range(base)) + [base + i for i in keep])
            st.kv.keep(keep_idx)
            hidden_seq = torch.cat([hidden_seq, hid[keep]], 0)
            st.committed = st.committed + [int(tree.tokens[i]) for i in keep]
            new = [int(tree.tokens[i]) for i in path] + [bonus]
            st.out.extend(new)
            st.accepted.append(len(path))
            st.root = bonus
            st.steps += 1
        st.out = st.out[: sp.max_new_tokens]
        return st
