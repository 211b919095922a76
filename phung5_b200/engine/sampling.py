"""Sampling: temperature / top-k / top-p target distributions, per-request seeded coins and the
speculative accept rules (greedy and target-only tree sampling).

Coins. The reference draws its verify coins from ``murmur_hash32(seed, prefix_len, column)``
(docker/opt/v3/seed/dflash_seed.patch:8-51): column 0..B-1 are the per-depth coins of one step and
column B the coin of the final (bonus) draw, and prefix_len grows every step, so no key repeats. We
keep that key scheme and define the hash concretely as MurmurHash3_x86_32 (Appleby, public domain)
over the three 32-bit words (prefix_len lo, prefix_len hi, column) with the request seed as the hash
seed; coin = h / (2^32 - 1) rounded to fp32 and clamped below 1.0 (a 1.0 coin could pick a
zero-probability token, dflash_seed.patch:44-48).

Accept rule (target-only tree speculative sampling). At the current node with target distribution
p and ordered children c_1..c_m, one coin u: accept the first child i with u < p(c_1)+...+p(c_i);
if none, draw the bonus token from p with the children's tokens removed (renormalised) using the
final coin. For distinct child tokens this emits each token with probability exactly p(token).
Greedy (temperature 0) accepts the child equal to argmax p and takes argmax p as the bonus.
"""
from __future__ import annotations

from typing import Optional, Sequence, Tuple

import torch

_M32 = 0xFFFFFFFF


def _rotl(x: torch.Tensor, r: int) -> torch.Tensor:
    return ((x << r) | (x >> (32 - r))) & _M32


def murmur3_32(words: Sequence[torch.Tensor], seed: torch.Tensor) -> torch.Tensor:
    """Vectorised MurmurHash3_x86_32 of a sequence of uint32 words (int64 tensors holding values
    in [0, 2^32)), broadcasting over the tensors. Returns int64 in [0, 2^32)."""
    c1, c2 = 0xCC9E2D51, 0x1B873593
    h = seed.to(torch.int64) & _M32
    for k in words:
        k = k.to(torch.int64) & _M32
        k = (k * c1) & _M32
        k = _rotl(k, 15)
        k = (k * c2) & _M32
        h = h ^ k
        h = _rotl(h, 13)
        h = (h * 5 + 0xE6546B64) & _M32
    h = h ^ (4 * len(words))
    h = h ^ (h >> 16)
    h = (h * 0x85EBCA6B) & _M32
    h = h ^ (h >> 13)
    h = (h * 0xC2B2AE35) & _M32
    h = h ^ (h >> 16)
    return h


_ONE_MINUS = float(torch.nextafter(torch.tensor(1.0), torch.tensor(0.0)))


def seeded_coins(seed: torch.Tensor, prefix_len: torch.Tensor, ncols: int) -> torch.Tensor:
    """[B] seeds, [B] committed lengths -> [B, ncols] fp32 coins in [0, 1)."""
    seed = seed.to(torch.int64)[:, None]
    pl = prefix_len.to(torch.int64)[:, None]
    col = torch.arange(ncols, device=seed.device, dtype=torch.int64)[None, :]
    h = murmur3_32([pl & _M32, (pl >> 32) & _M32, col.expand(pl.shape[0], ncols)], seed)
    u = (h.double() / float(_M32)).float()
    return u.clamp(max=_ONE_MINUS)


def target_probs(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
                 top_p: torch.Tensor) -> torch.Tensor:
    """logits [R, V] (any float), per-row temperature/top_k/top_p [R] -> probs [R, V] fp32.

    Temperature divides with IEEE division (the reference's topkbf kernel uses div.rn.f32,
    docker/opt/v5/topkbf_normcfg/topkbf/kopt_topkbf.py:134-141). top_k <= 0 means no top-k cut;
    top_p >= 1 means no nucleus cut. Rows with temperature 0 become one-hot at the argmax."""
    x = logits.float()
    greedy = temperature <= 0
    t = torch.where(greedy, torch.ones_like(temperature), temperature).float()
    x = x / t[:, None]
    v = x.shape[-1]
    k = torch.where(top_k <= 0, torch.full_like(top_k, v), top_k).clamp(max=v)
    # stable: equal values keep vocab order, so the top-k cut and the nucleus break ties toward the lower index
    sv, si = torch.sort(x, dim=-1, descending=True, stable=True)
    pos = torch.arange(v, device=x.device)[None, :]
    keep = pos < k[:, None]
    sv = sv.masked_fill(~keep, float("-inf"))
    sp = torch.softmax(sv, dim=-1)
    cum = torch.cumsum(sp, dim=-1)
    # keep the smallest prefix whose mass reaches top_p (the first token is always kept)
    keep_p = (cum - sp) < top_p[:, None].float()
    sp = sp * keep_p
    sp = sp / sp.sum(-1, keepdim=True)
    probs = torch.zeros_like(x).scatter_(-1, si, sp)
    if greedy.any():
        onehot = torch.zeros_like(x).scatter_(-1, logits.float().argmax(-1, keepdim=True), 1.0)
        probs = torch.where(greedy[:, None], onehot, probs)
    return probs


def tree_accept_reference(logits, tokens: torch.Tensor, parent: torch.Tensor, temp: torch.Tensor, top_k: torch.Tensor,
                          top_p: torch.Tensor, coins: torch.Tensor, depth: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Seeded target-only tree sampling for a batch (the definition the device path implements).

    logits: callable(rows [R] node ids) -> full-vocab logits [R, V] of each request's node (so a
    vocab-sharded caller can gather only the visited rows), or a tensor [R, N, V]. tokens/parent [R, N]
    (parent -1 for the root), per-request temp/top_k/top_p [R], coins [R, depth + 2] (column d-1 for depth d,
    column depth+1 for the bonus draw). Returns (accepted node ids [R, depth], -1 padded; bonus tokens [R])."""
    R, N = tokens.shape
    D = depth
    dev = tokens.device
    get = logits if callable(logits) else (lambda cur: logits[torch.arange(R, device=dev), cur])
    cur = torch.zeros(R, dtype=torch.int64, device=dev)
    acc = torch.full((R, D), -1, dtype=torch.int64, device=dev)
    nidx = torch.arange(N, device=dev)[None, :]
    bonus = torch.zeros(R, dtype=torch.int64, device=dev)
    done = torch.zeros(R, dtype=torch.bool, device=dev)
    for d in range(1, D + 2):
        p = target_probs(get(cur), temp, top_k, top_p)                       # [R, V]
        kids = (parent == cur[:, None]) & ~done[:, None] & (d <= D)
        kp = torch.where(kids, p.gather(1, tokens.clamp(min=0)), torch.zeros_like(p[:, :N]))
        cum = torch.cumsum(kp, 1)
        u = coins[:, d - 1]
        hit = kids & (u[:, None] < cum)
        has = hit.any(1) & ~done
        first = torch.where(hit, nidx.expand(R, N), torch.full_like(tokens, N)).min(1).values
        # rows that stop here draw the bonus from p minus the children's tokens
        stop = ~has & ~done
        if stop.any():
            hitcnt = torch.zeros(p.shape, dtype=torch.int32, device=dev).scatter_add_(
                1, tokens.clamp(min=0), kids.to(torch.int32))
            q = p.masked_fill(hitcnt > 0, 0.0)
            empty = q.sum(1) <= 0
            q = torch.where(empty[:, None], p, q)
            samp = sample_from(q, coins[:, D + 1])
            samp = torch.where(temp <= 0, p.argmax(1), samp)
            bonus = torch.where(stop, samp, bonus)
        if d <= D:
            acc[:, d - 1] = torch.where(has, first, torch.full_like(first, -1))
            cur = torch.where(has, first, cur)
        done |= stop
        if bool(done.all()):
            break
    return acc, bonus


def sample_from(probs: torch.Tensor, coin: torch.Tensor) -> torch.Tensor:
    """Inverse-CDF draw: first index whose cumulative mass exceeds coin (coins in [0,1))."""
    cum = torch.cumsum(probs.double(), dim=-1)
    total = cum[:, -1:]
    idx = torch.searchsorted(cum, (coin.double()[:, None] * total), right=True).squeeze(-1)
    return idx.clamp(max=probs.shape[-1] - 1)


def accept_tree(node_tokens: torch.Tensor, children: Sequence[Sequence[int]], probs: torch.Tensor,
                greedy: bool, coins: Optional[torch.Tensor] = None,
                final_coin: Optional[float] = None) -> Tuple[list, int]:
    """Walk one request's verified tree.

    node_tokens [N] (node 0 = root), children[i] = ordered child node ids, probs [N, V] = target
    distribution after each node. Returns (accepted node ids after the root, bonus token id)."""
    cur, path = 0, []
    depth = 0
    while True:
        kids = list(children[cur])
        p = probs[cur]
        chosen = -1
        if kids:
            if greedy:
                best = int(torch.argmax(p))
                for c in kids:
                    if int(node_tokens[c]) == best:
                        chosen = c
                        break
            else:
                u = float(coins[depth])
                acc = 0.0
                for c in kids:
                    acc += float(p[int(node_tokens[c])])
                    if u < acc:
                        chosen = c
                        break
        if chosen < 0:
            if greedy:
                bonus = int(torch.argmax(p))
            else:
                q = p.clone()
                for c in kids:
                    q[int(node_tokens[c])] = 0.0
                if float(q.sum()) <= 0.0:
                    q = p.clone()
                bonus = int(sample_from(q[None], torch.tensor([final_coin]))[0])
            return path, bonus
        path.append(chosen)
        cur = chosen
        depth += 1


def geometric_accept_len(seed: int, step: torch.Tensor, rid: torch.Tensor, p: float, cap: int) -> torch.Tensor:
    """Seeded synthetic accept length: Geometric(p) on {0,1,...} (number of accepted drafts before the
    first rejection), capped at `cap`. Drawn from the request's own hash stream (seed, request id,
    step) so it is independent of batch order."""
    h = murmur3_32([rid.to(torch.int64), step.to(torch.int64), torch.full_like(rid, 0x5EED, dtype=torch.int64)],
                   torch.full_like(rid, seed, dtype=torch.int64))
    u = (h.double() + 0.5) / 4294967296.0
    n = torch.floor(torch.log(u) / torch.log(torch.tensor(1.0 - p, dtype=torch.float64)))
    return n.clamp(max=cap).to(torch.int64)
