"""First-iteration stages: K coders at once -> dedup -> validate -> streaming single-elimination bracket ->
optional round robin among the last four.

Reference: `multigen_first_iter` (pipeline_service/pipeline/stages.py:1048-1217), `_CandidateFactory`
(:702-950), `_resolve_bracket` (:589-677), `_round_robin_top4` (:320-427).

- Leaves: position k runs coder k (coders are assigned round-robin over the configured coder pool, seed
  `task.seed + k`), the checker, dedup by whitespace-insensitive code digest (the first position to reach
  a digest keeps it), judge-view renders (white + gray) and view embeddings. A leaf that fails or
  duplicates is a walkover for its opponent (no judge call).
- Bracket: pairing is by position, independent of which leaves drop, so results are reproducible for a
  seed. A duel starts as soon as both of its subtree winners are known, so judging overlaps coding and
  rendering of other leaves.
- Draws are settled by a coin keyed on (seed, stem, positions): reproducible, no bias toward a side.
- Round robin: with `round_robin = 4` (or 8) and at least that many live winners of the bracket's quarter
  (eighth) subtrees, all pairs of them are judged; 1 point per win (a draw is settled by the coin first); ties
  go to the bracket winner. Verdicts already computed in the bracket are reused, not re-judged.
- Judge alignment (reference pgh_jalign.py): S1 early stop can be limited to the first bracket rounds.
- Shadow picks (reference pgh_shadow.py): after the shipped pick is final, the pick a listed feature would
  have made (rr4 / rr8) is computed with a bounded number of extra duels and recorded on the task, never
  shipped.
"""
from __future__ import annotations

import asyncio
import hashlib
import time
from dataclasses import dataclass
from typing import Awaitable, Callable, Dict, List, Optional, Sequence

from .agents import JudgeAgent, SceneCoderAgent
from .jscheck import code_digest
from .renderer import RendererModule
from .schemas import JudgeVerdict
from .state import Candidate, PipelineTask


def coin(seed: int, *keys) -> bool:
    h = hashlib.sha256(repr((seed,) + keys).encode()).digest()
    return h[0] & 1 == 1


@dataclass
class StageLimits:
    coder: asyncio.Semaphore
    judge: asyncio.Semaphore
    render: asyncio.Semaphore


class CandidateFactory:
    """Builds one Candidate per bracket position (or None)."""

    def __init__(self, task: PipelineTask, coders: Sequence[SceneCoderAgent], renderer: RendererModule, embedder,
                 limits: StageLimits, prompt_url: str, plan: Optional[str] = None, deadline: Optional[float] = None,
                 on_event: Optional[Callable[[str, dict], None]] = None, ref_vec=None, checker=None,
                 orient=None, brake=None):
        self.task, self.coders, self.renderer, self.embedder = task, coders, renderer, embedder
        self.limits, self.prompt_url, self.plan, self.deadline = limits, prompt_url, plan, deadline
        # orientation stage (app/orient.py): needs the prompt's embedding and a checker for the rewritten module
        self.ref_vec, self.checker, self.orient = ref_vec, checker, orient
        self.seen: Dict[str, int] = {}
        self.on_event = on_event or (lambda kind, d: None)
        self.brake = brake                  # kpolicy.RenderBrake or None
        self.code_bytes: Dict[int, Optional[int]] = {}    # position -> bytes of its draft (None: no draft)
        self._arrived = asyncio.Condition()

    async def _note_draft(self, k: int, nbytes: Optional[int]) -> None:
        async with self._arrived:
            self.code_bytes[k] = nbytes
            self._arrived.notify_all()

    async def drafts_of(self, positions: Sequence[int]) -> List[int]:
        """Wait until every listed position's coder call has returned; their draft sizes in bytes."""
        async with self._arrived:
            await self._arrived.wait_for(lambda: all(p in self.code_bytes for p in positions))
        return [self.code_bytes[p] for p in positions if self.code_bytes[p]]

    async def _render(self, coro):
        if self.brake is None:
            return await coro
        await self.brake.enter_render()
        try:
            return await coro
        finally:
            await self.brake.leave_render()

    def _left(self) -> Optional[float]:
        return None if self.deadline is None else self.deadline - time.monotonic()

    async def build(self, k: int) -> Optional[Candidate]:
        coder = self.coders[k % len(self.coders)]
        t = self.task
        try:
            if self.brake is not None:
                await self.brake.before_coder()
            async with self.limits.coder:
                left = self._left()
                if left is not None and left <= 0:
                    await self._note_draft(k, None)
                    return None
                res = await asyncio.wait_for(coder.generate(self.prompt_url, t.seed + k, plan=self.plan), left)
        except (asyncio.TimeoutError, Exception) as e:  # noqa: BLE001 - a failed leaf is a walkover
            t.js_errors.append(f"k{k} {coder.name}: {type(e).__name__}: {str(e)[:160]}")
            self.on_event("coder_error", {"k": k})
            await self._note_draft(k, None)
            return None
        await self._note_draft(k, len(res.check.code or "") or None)
        t.n_generated += 1
        if not res.check.ok:
            t.js_errors.append(f"k{k} {coder.name}: {res.check.summary()[:300]}")
            self.on_event("invalid", {"k": k})
            return None
        t.n_valid += 1
        dg = code_digest(res.check.code)
        if dg in self.seen:
            t.n_duplicates += 1
            self.on_event("duplicate", {"k": k, "of": self.seen[dg]})
            return None
        self.seen[dg] = k
        cand = Candidate(code=res.check.code, digest=dg, coder=coder.name, scene=res.check.scene,
                         stats={**res.check.stats, "k": k, "repairs": res.repairs})
        if self.orient is not None and self.orient.enabled and self.checker is not None and self.ref_vec is not None:
            from .orient import orient_candidate
            async with self.limits.render:
                cand.code, cand.scene, ores = await self._render(orient_candidate(
                    cand.code, cand.scene, renderer=self.renderer, embedder=self.embedder, ref_vec=self.ref_vec,
                    checker=self.checker, settings=self.orient))
            cand.stats["orient"] = ores.reason if not ores.applied else f"{ores.best}:{len(ores.steps)}"
            self.on_event("orient", {"k": k, "applied": ores.applied, "best": ores.best})
        try:
            async with self.limits.render:
                views = await self._render(self.renderer.judge_views(cand.scene, gray=True))
        except (asyncio.TimeoutError, Exception) as e:  # noqa: BLE001
            t.js_errors.append(f"k{k} render: {type(e).__name__}: {str(e)[:160]}")
            self.on_event("render_error", {"k": k})
            return None
        cand.views, cand.gray_views = views["white"], views.get("gray", [])
        if self.embedder is not None:
            cand.embed = await self.embedder.embed(cand.views)
        t.candidates.append(cand)
        if t.js_code is None:          # something to salvage if the deadline hits before any duel
            t.js_code, t.scene_json, t.lead_round = cand.code, cand.scene, 0
        self.on_event("candidate", {"k": k})
        return cand


DuelFn = Callable[[Candidate, Candidate, str], Awaitable[Candidate]]


def make_duel(task: PipelineTask, judge: JudgeAgent, limits: StageLimits, prompt_url: str, ref_vec,
              on_duel: Optional[Callable[[float, float], None]] = None, es_max_round: int = 0) -> DuelFn:
    cache: Dict[tuple, Candidate] = {}

    async def duel(left: Candidate, right: Candidate, label: str) -> Candidate:
        key = (left.digest, right.digest)
        if key in cache:                    # a pair the bracket already judged (round robin reuses it)
            return cache[key]
        if (right.digest, left.digest) in cache:
            return cache[(right.digest, left.digest)]
        rnd_s = label[1:].split()[0] if label.startswith("R") and label[1:2].isdigit() else ""
        early = not (es_max_round > 0 and rnd_s and int(rnd_s) > es_max_round)
        tq = time.monotonic()
        async with limits.judge:
            ts = time.monotonic()
            v: JudgeVerdict = await judge.duel(prompt_url, left, right, task.seed, ref_vec, early_stop=early)
        te = time.monotonic()
        if on_duel is not None:
            on_duel(te - ts, ts - tq)
        task.duels += 1
        if v.winner == "draw":
            w = left if coin(task.seed, task.stem, label, left.digest, right.digest) else right
            how = f"{v.decided_by} -> coin"
        else:
            w = left if v.winner == "A" else right
            how = v.decided_by
        task.judge_log.append({"label": label, "left": left.stats.get("k"), "right": right.stats.get("k"),
                               "winner": w.stats.get("k"), "decided_by": how, "verdict": v.winner})
        w.wins += 1
        rnd = int(label[1:].split()[0]) if label.startswith("R") and label[1:2].isdigit() else 0
        if rnd >= task.lead_round:     # the deepest bracket winner so far leads (salvage)
            task.js_code, task.scene_json, task.lead_round = w.code, w.scene, rnd
        cache[key] = w
        return w
    return duel


async def resolve_bracket(leaves: Dict[int, "asyncio.Future"], duel: DuelFn, n: int, tops=None) -> tuple:
    """-> (winner or None, the live winners of the bracket's four quarter subtrees when n >= 4). `tops`, a dict
    {depth: []}, also collects the live winners of the subtrees at other depths (3 = eighths)."""
    semis: List[Candidate] = []

    async def winner_of(lo: int, hi: int, depth: int) -> Optional[Candidate]:
        if hi - lo <= 1:
            res = await leaves[lo]
        else:
            mid = (lo + hi) // 2
            left, right = await asyncio.gather(winner_of(lo, mid, depth + 1), winner_of(mid, hi, depth + 1))
            if left is None:
                res = right
            elif right is None:
                res = left
            else:
                rnd = (hi - lo - 1).bit_length()
                res = await duel(left, right, f"R{rnd} {lo}-{hi}")
        if depth == 2 and res is not None:
            semis.append(res)
        if tops is not None and depth in tops and res is not None:
            tops[depth].append(res)
        return res

    if n == 0:
        return None, []
    w = await winner_of(0, n, 0)
    return w, semis


async def round_robin(cands: List[Candidate], duel: DuelFn, bracket_winner: Candidate) -> Candidate:
    pts = {id(c): 0.0 for c in cands}
    pairs = [(a, b) for i, a in enumerate(cands) for b in cands[i + 1:]]
    winners = await asyncio.gather(*(duel(a, b, f"RR {a.stats.get('k')}-{b.stats.get('k')}") for a, b in pairs))
    for w in winners:
        pts[id(w)] += 1.0
    for c in cands:
        c.rr_points = pts[id(c)]
    best = max(pts.values())
    top = [c for c in cands if pts[id(c)] == best]
    return bracket_winner if any(c is bracket_winner for c in top) else top[0]


async def multigen_first_iter(task: PipelineTask, factory: CandidateFactory, duel: DuelFn, k: int,
                              round_robin_size: int = 0, shadow: Sequence[str] = (),
                              shadow_max_duels: int = 12,
                              final_turn: Optional[Callable[[Candidate], Awaitable[Candidate]]] = None,
                              budget=None) -> Optional[Candidate]:
    """`budget` (kpolicy.BudgetK): once it has reference prompts, the first K_lo positions start at once, their
    draft sizes set this prompt's K_i in [K_lo, K_hi], positions K_lo..K_i-1 start then, and positions from K_i
    on are walkovers of a bracket laid out for K_hi positions (pairing stays by position)."""
    size = k
    extra = None
    if budget is not None and budget.active(k):
        k_lo = budget.initial(k)
        size = max(k_lo, int(round(budget.hi * k)))
        decided = asyncio.Event()
        k_final = [k]

        async def decide():
            try:
                sizes = await factory.drafts_of(list(range(k_lo)))
                k_final[0] = budget.decide(k, [float(b) for b in sizes]) if sizes else k
                task.budget_k = k_final[0]
            finally:
                decided.set()

        async def gated(i):
            await decided.wait()
            return await factory.build(i) if i < k_final[0] else None
        extra = asyncio.ensure_future(decide())
        leaves = {i: asyncio.ensure_future(factory.build(i) if i < k_lo else gated(i)) for i in range(size)}
    else:
        leaves = {i: asyncio.ensure_future(factory.build(i)) for i in range(k)}
    tops = {3: []}
    try:
        winner, semis = await resolve_bracket(leaves, duel, size, tops)
    finally:
        for f in list(leaves.values()) + ([extra] if extra is not None else []):
            if not f.done():
                f.cancel()
    if winner is None:
        return None
    players = {4: semis, 8: tops[3]}
    bracket_winner = winner
    if round_robin_size in players and len(players[round_robin_size]) >= round_robin_size:
        winner = await round_robin(players[round_robin_size][:round_robin_size], duel, winner)
    if shadow:
        task.shadow = await shadow_picks(task, shadow, players, duel, bracket_winner, shadow_max_duels)
        task.shadow["shipped"] = winner.stats.get("k")
    if final_turn is not None:          # turned copies of the final (app/orient.py turn_final)
        winner = await final_turn(winner)
    return winner


async def shadow_picks(task: PipelineTask, features: Sequence[str], players: Dict[int, List[Candidate]], duel: DuelFn,
                       bracket_winner: Candidate, max_duels: int) -> dict:
    """What each listed selection feature would have picked (recorded on the task, not shipped). Extra duels are
    bounded by max_duels; pairs already judged come from the duel cache."""
    out: Dict[str, object] = {}
    budget = [max_duels]

    async def capped(a, b, label):
        if budget[0] <= 0:
            raise RuntimeError("shadow duel budget spent")
        budget[0] -= 1
        return await duel(a, b, "SH " + label)
    for f in features:
        n = {"rr4": 4, "rr8": 8}.get(f)
        if n is None or len(players.get(n, [])) < n:
            out[f] = None
            continue
        try:
            pick = await round_robin(players[n][:n], capped, bracket_winner)
            out[f] = pick.stats.get("k")
        except RuntimeError:
            out[f] = "budget"
    return out
