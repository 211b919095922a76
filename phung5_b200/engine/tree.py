"""Draft-tree construction shared by the CPU oracle and the batched engine.

A speculative step verifies a tree of N nodes per request: node 0 is the root (the pending token,
sampled by the previous step and not yet in the target's KV cache); every other node is a draft
token with a parent. Chain speculation is the special case parent[i] = i - 1.

The dynamic tree is built EAGLE-2 style: starting from the root, `depth` rounds each expand the
`topk` best frontier nodes into their `topk` most likely children (by draft probability); every
candidate carries the cumulative draft log-probability of its path; the final tree keeps the
N - 1 best candidates (ties broken toward shallower nodes so the kept set is ancestor-closed) and
orders them by (depth, score). The reference's DFlash path only drafts chains (tree verify raises in
docker/opt/kern/braw/kernels.py:477-478); the tree is the benchmark's 64-node top-k=8 tree.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List

import torch


@dataclass
class Tree:
    tokens: torch.Tensor   # [N] int64, node 0 = root
    parent: torch.Tensor   # [N] int64, parent[0] = -1
    depth: torch.Tensor    # [N] int64, depth[0] = 0

    @property
    def n(self) -> int:
        return int(self.tokens.shape[0])

    def children(self) -> List[List[int]]:
        kids: List[List[int]] = [[] for _ in range(self.n)]
        for i in range(1, self.n):
            kids[int(self.parent[i])].append(i)
        return kids

    def ancestor_mask(self) -> torch.Tensor:
        """[N, N] bool: mask[i, j] = j is i or an ancestor of i."""
        n = self.n
        m = torch.zeros(n, n, dtype=torch.bool)
        for i in range(n):
            j = i
            while j >= 0:
                m[i, j] = True
                j = int(self.parent[j])
        return m

    def mask_bits(self) -> torch.Tensor:
        """[N] int64 bitmasks of ancestor_mask (requires N <= 64); bit j set = node j visible."""
        assert self.n <= 64
        m = self.ancestor_mask().to(torch.int64)
        w = (torch.ones(64, dtype=torch.int64) << torch.arange(64))[: self.n]
        return (m * w[None, :]).sum(-1)

    def path_to(self, i: int) -> List[int]:
        p = []
        while i > 0:
            p.append(i)
            i = int(self.parent[i])
        return p[::-1]


def chain_tree(root: int, drafts: List[int]) -> Tree:
    n = len(drafts) + 1
    return Tree(tokens=torch.tensor([root] + list(drafts), dtype=torch.int64),
                parent=torch.arange(-1, n - 1, dtype=torch.int64),
                depth=torch.arange(n, dtype=torch.int64))


def select_tree(root: int, cand_tokens: List[int], cand_parent: List[int], cand_score: List[float],
                cand_depth: List[int], n_nodes: int) -> Tree:
    """Pick the best n_nodes-1 candidates (candidate parents index the candidate list, -1 = root) and
    renumber them into a Tree ordered by (depth, -score)."""
    order = sorted(range(len(cand_tokens)), key=lambda i: (-cand_score[i], cand_depth[i], i))
    keep = set(order[: max(0, n_nodes - 1)])
    # ancestor closure (guards exotic ties with -inf scores)
    for i in list(keep):
        j = cand_parent[i]
        while j >= 0 and j not in keep:
            keep.add(j)
            j = cand_parent[j]
    kept = sorted(keep, key=lambda i: (cand_depth[i], -cand_score[i], i))
    kept = kept[: n_nodes - 1]
    newid = {c: k + 1 for k, c in enumerate(kept)}
    tokens = [root] + [cand_tokens[c] for c in kept]
    parent = [-1] + [newid.get(cand_parent[c], 0) if cand_parent[c] >= 0 else 0 for c in kept]
    depth = [0] + [cand_depth[c] for c in kept]
    return Tree(torch.tensor(tokens, dtype=torch.int64), torch.tensor(parent, dtype=torch.int64),
                torch.tensor(depth, dtype=torch.int64))
