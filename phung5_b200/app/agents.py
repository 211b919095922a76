"""Model roles: scene coder, critic, planner and the multi-stage pairwise judge.

References: `SceneCoderAgent` (pipeline_service/modules/scene_coder/agent.py:27-278), critic
(modules/critic/agent.py:78-258), planner (modules/scene_planner/agent.py:37-114), `JudgeAgent.compare`
(modules/judge/agent.py:106-212) and `evaluate_duel` (modules/judge/multi_stage.py:1570-1754).

Judge duel (own design, same stage structure as the reference):
  S1  prompt match at 4 front angles; each angle is asked in both orders (A,B) and (B,A) to cancel position
      bias, an angle whose two orders disagree in sign counts as a draw; weighted mean penalty difference
      >= `s1_threshold` decides. Both-bad (both means >= `s1_both_bad`, small gap) is a draw. Angles are
      evaluated in order and S1 stops early once the remaining weight cannot change the outcome.
  S2  three sub-judges: best view (each model's view most similar to the target by the embedder), artifact
      penalties and a feature checklist. A strong voter (best-view gap >= 2 or checklist gap >= 6) decides
      alone; otherwise at least 2 of 3 votes must agree.
  S3  gray rescue (only on a draw): when either model is mostly pale, white-background renders hide it; the
      same question is asked on gray renders.
  S4  side guard (only on a decision): side and back views; if `s4_k` of them prefer the loser, the
      decision is withdrawn (draw).
  Tie-break: the model whose best view is most similar to the target by embedding; with no embedder, the
      seeded coin of the bracket decides.
Every model call goes through `SessionAgent` (schema-validated JSON, bounded retries); a call that still
fails yields a neutral answer so one bad reply never aborts a batch.
"""
from __future__ import annotations

import asyncio
import base64
import hashlib
import json
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple

import numpy as np
import torch

from . import prompts as P
from .jscheck import CheckResult, JSChecker
from .renderer import RendererModule, compose_grid, data_url, to_png
from .schemas import (AnglePenalty, ArtifactReply, BestViewReply, ChecklistReply, CriticReport, JudgeVerdict,
                      ObjectPlan, PreferenceReply)
from .session import SessionAgent, purpose_var
from .state import Candidate


def image_part(url: str) -> dict:
    return {"type": "image_url", "image_url": {"url": url}}


def user_content(text: str, *urls: str) -> list:
    return [*(image_part(u) for u in urls), {"type": "text", "text": text}]


def bytes_to_data_url(data: bytes, mime: str = "image/png") -> str:
    return f"data:{mime};base64," + base64.b64encode(data).decode()


# ----------------------------------------------------------------------------------------------------- coder


@dataclass
class CoderResult:
    text: str
    check: CheckResult
    turns: int
    repairs: int
    usage: Dict[str, int] = field(default_factory=dict)
    history: List[dict] = field(default_factory=list)


class SceneCoderAgent:
    def __init__(self, backend, model: str, checker: JSChecker, name: str = "coder", max_repairs: int = 2,
                 max_tokens: int = 8192, temperature: float = 0.7, top_p: float = 0.95):
        self.name = name
        self.checker = checker
        self.max_repairs = max_repairs
        self.session = SessionAgent(backend, model, P.CODER_SYSTEM, max_tokens=max_tokens, temperature=temperature,
                                    top_p=top_p, max_turns=1)

    async def generate(self, prompt_url: str, seed: int, plan: Optional[str] = None,
                       history: Optional[List[dict]] = None, user_text: Optional[str] = None) -> CoderResult:
        """One candidate: generate, check, and repair with the checker's failures up to `max_repairs` times."""
        purpose_var.set(f"{self.name}:generate")
        text = user_text or (P.CODER_USER_WITH_PLAN.format(plan=plan) if plan else P.CODER_USER)
        r = await self.session.run(user_content(text, prompt_url), history=history, seed=seed)
        usage = dict(r.usage)
        check = await self.checker.check_async(r.content, seed=seed)
        repairs = 0
        msgs = r.messages
        while not check.ok and repairs < self.max_repairs:
            repairs += 1
            purpose_var.set(f"{self.name}:repair")
            fails = "\n".join(f"- [{f['rule']}] {f['detail']}" for f in check.failures[:8])
            r = await self.session.run(P.REPAIR_USER.format(failures=fails), history=msgs, seed=seed + 7919 * repairs)
            for k, v in r.usage.items():
                usage[k] = usage.get(k, 0) + v
            msgs = r.messages
            check = await self.checker.check_async(r.content, seed=seed)
        return CoderResult(r.content, check, 1 + repairs, repairs, usage, msgs)


# ------------------------------------------------------------------------------------------ critic / planner


class CriticAgent:
    def __init__(self, backend, model: str, max_tokens: int = 2048):
        self.session = SessionAgent(backend, model, P.CRITIC_SYSTEM, schema=CriticReport, max_tokens=max_tokens,
                                    temperature=0.0, max_turns=3)

    async def review(self, prompt_url: str, grid_png: bytes, seed: int) -> CriticReport:
        purpose_var.set("critic")
        try:
            r = await self.session.run(user_content("Target, then renders of the model.", prompt_url,
                                                    data_url(grid_png)), seed=seed)
            return r.parsed
        except (ValueError, RuntimeError):
            return CriticReport()


class PlannerAgent:
    def __init__(self, backend, model: str, max_tokens: int = 2048):
        self.session = SessionAgent(backend, model, P.PLANNER_SYSTEM, schema=ObjectPlan, max_tokens=max_tokens,
                                    temperature=0.0, max_turns=3)

    async def plan(self, prompt_url: str, seed: int) -> Optional[ObjectPlan]:
        purpose_var.set("planner")
        try:
            r = await self.session.run(user_content("Describe this object.", prompt_url), seed=seed)
            return r.parsed
        except (ValueError, RuntimeError):
            return None


# ------------------------------------------------------------------------------------------------------ judge


@dataclass
class JudgeSettings:
    s1_angles: Tuple[Tuple[int, float, str], ...] = ((0, 1.0, "from the front"), (1, 0.8, "from the front left"),
                                                     (2, 0.8, "from the front right"), (3, 0.6, "from the side"))
    s1_threshold: float = 0.7
    s1_both_bad: float = 8.0
    s2_bv_gap: float = 1.0
    s2_ac_gap: float = 1.0
    s2_cl_gap: int = 2
    s2_strong_bv: float = 2.0
    s2_strong_cl: int = 6
    s2_min_consensus: int = 2
    s2_features: Tuple[int, int] = (4, 7)
    s3_pale_luma: float = 175.0
    s3_pale_sat: float = 0.35
    s3_pale_fraction: float = 0.10
    s3_diff: float = 2.0
    s4_views: Tuple[Tuple[int, str], ...] = ((3, "from the side"), (4, "from behind"), (5, "from above"))
    s4_k: int = 3
    max_stage: int = 4
    concurrency: int = 8
    max_tokens: int = 512


class CandidateViews:
    """Lazily encoded PNG data URLs of a candidate's white and gray views."""

    def __init__(self, cand: Candidate):
        self.c = cand
        self._white: Dict[int, str] = {}
        self._gray: Dict[int, str] = {}

    def white(self, i: int) -> str:
        if i not in self._white:
            self._white[i] = data_url(to_png(self.c.views[i]))
        return self._white[i]

    def gray(self, i: int) -> str:
        if i not in self._gray:
            self._gray[i] = data_url(to_png(self.c.gray_views[i] if self.c.gray_views else self.c.views[i]))
        return self._gray[i]


def pale_fraction(views: List[torch.Tensor], bg=(255, 255, 255), luma_min=175.0, sat_max=0.35, step=4) -> float:
    """Share of the object's pixels (not background) that are pale: bright and unsaturated."""
    if not views:
        return 0.0
    img = views[0][::step, ::step, :3].float()
    bgt = torch.tensor(bg, dtype=torch.float32, device=img.device)
    obj = (img - bgt).abs().amax(-1) > 18
    if not bool(obj.any()):
        return 0.0
    px = img[obj]
    mx, mn = px.amax(-1), px.amin(-1)
    luma = 0.299 * px[:, 0] + 0.587 * px[:, 1] + 0.114 * px[:, 2]
    sat = torch.where(mx > 0, (mx - mn) / mx.clamp(min=1), torch.zeros_like(mx))
    return float(((luma >= luma_min) & (sat <= sat_max)).float().mean())


class JudgeAgent:
    def __init__(self, backend, model: str, settings: Optional[JudgeSettings] = None, embedder=None):
        self.s = settings or JudgeSettings()
        self.embedder = embedder
        self.sem = asyncio.Semaphore(self.s.concurrency)
        mk = lambda schema: SessionAgent(backend, model, P.JUDGE_SYSTEM, schema=schema, max_tokens=self.s.max_tokens,
                                         temperature=0.0, max_turns=4, validation_retries=3)
        self.s1 = mk(AnglePenalty)
        self.bv = mk(BestViewReply)
        self.ac = mk(ArtifactReply)
        self.cl = mk(ChecklistReply)
        self.pref = mk(PreferenceReply)
        self.calls = 0

    async def _ask(self, agent: SessionAgent, content, seed, neutral):
        async with self.sem:
            self.calls += 1
            try:
                return (await agent.run(content, seed=seed)).parsed
            except (ValueError, RuntimeError):
                return neutral

    # S1
    async def _s1(self, prompt, A: CandidateViews, B: CandidateViews, seed, early_stop: bool = True) -> dict:
        neutral = AnglePenalty(penalty_a=5, penalty_b=5, reason="JSON_FAILED")
        total_w = sum(w for _, w, _ in self.s.s1_angles)
        acc, used_w, angles = 0.0, 0.0, []
        sum_a = sum_b = 0.0
        for i, (view, w, desc) in enumerate(self.s.s1_angles):
            txt = P.S1_USER.format(angle=desc)
            ab, ba = await asyncio.gather(
                self._ask(self.s1, user_content(txt, prompt, A.white(view), B.white(view)), seed, neutral),
                self._ask(self.s1, user_content(txt, prompt, B.white(view), A.white(view)), seed, neutral))
            d1 = ab.penalty_a - ab.penalty_b             # > 0: A worse
            d2 = ba.penalty_b - ba.penalty_a
            contradictory = (d1 > 0 > d2) or (d1 < 0 < d2) or "JSON_FAILED" in (ab.reason, ba.reason)
            d = 0.0 if contradictory else (d1 + d2) / 2
            pa, pb = (ab.penalty_a + ba.penalty_b) / 2, (ab.penalty_b + ba.penalty_a) / 2
            sum_a += w * pa
            sum_b += w * pb
            acc += w * d
            used_w += w
            angles.append({"view": view, "diff": d, "pen_a": pa, "pen_b": pb, "contradictory": contradictory})
            rest = total_w - used_w
            # the weighted mean cannot cross the threshold back: stop
            if early_stop and i < len(self.s.s1_angles) - 1 and abs(acc) - rest * 10 >= self.s.s1_threshold * total_w:
                break
        mean = acc / used_w
        mean_a, mean_b = sum_a / used_w, sum_b / used_w
        if mean_a >= self.s.s1_both_bad and mean_b >= self.s.s1_both_bad and abs(mean) < max(1.5, self.s.s1_threshold):
            choice = "draw"
        elif mean <= -self.s.s1_threshold:
            choice = "A"
        elif mean >= self.s.s1_threshold:
            choice = "B"
        else:
            choice = "draw"
        return {"choice": choice, "mean_diff": round(mean, 3), "pen_a": round(mean_a, 3), "pen_b": round(mean_b, 3),
                "angles": angles, "early_stop": len(angles) < len(self.s.s1_angles)}

    # S2
    def _best_view(self, cand: Candidate, ref_vec) -> int:
        if ref_vec is None or cand.embed is None:
            return 0
        return int(np.argmax(cand.embed[: len(cand.views)] @ ref_vec))

    async def _s2(self, prompt, A, B, ref_vec, seed) -> dict:
        ia, ib = self._best_view(A.c, ref_vec), self._best_view(B.c, ref_vec)
        lo, hi = self.s.s2_features
        bv, ac, cl = await asyncio.gather(
            self._ask(self.bv, user_content(P.S2_BEST_VIEW_USER, prompt, A.white(ia), B.white(ib)), seed,
                      BestViewReply(penalty_a=5, penalty_b=5)),
            self._ask(self.ac, user_content(P.S2_ARTIFACT_USER, prompt, A.white(0), B.white(0)), seed,
                      ArtifactReply(artifacts_a=5, artifacts_b=5)),
            self._ask(self.cl, user_content(P.S2_CHECKLIST_USER.format(lo=lo, hi=hi), prompt, A.white(0), B.white(0)),
                      seed, ChecklistReply()))
        bv_diff = bv.penalty_a - bv.penalty_b
        ac_diff = ac.artifacts_a - ac.artifacts_b
        n = min(len(cl.features), len(cl.has_a), len(cl.has_b))
        cl_gap = (sum(cl.has_a[:n]) - sum(cl.has_b[:n])) * 2 if n >= lo else 0   # > 0: A has more

        def vote(diff, gap):
            return "A" if diff <= -gap else ("B" if diff >= gap else "draw")
        votes = {"bv": vote(bv_diff, self.s.s2_bv_gap), "ac": vote(ac_diff, self.s.s2_ac_gap),
                 "cl": "A" if cl_gap >= self.s.s2_cl_gap else ("B" if cl_gap <= -self.s.s2_cl_gap else "draw")}
        if abs(bv_diff) >= self.s.s2_strong_bv:
            choice, src = votes["bv"], "strong_bv"
        elif abs(cl_gap) >= self.s.s2_strong_cl:
            choice, src = votes["cl"], "strong_cl"
        else:
            src = "consensus"
            na = sum(v == "A" for v in votes.values())
            nb = sum(v == "B" for v in votes.values())
            choice = "A" if na >= self.s.s2_min_consensus else ("B" if nb >= self.s.s2_min_consensus else "draw")
        return {"choice": choice, "source": src, "votes": votes, "diffs": {"bv": bv_diff, "ac": ac_diff, "cl": cl_gap},
                "best_views": [ia, ib]}

    async def _s3(self, prompt, A, B, seed) -> dict:
        pa = pale_fraction(A.c.views, luma_min=self.s.s3_pale_luma, sat_max=self.s.s3_pale_sat)
        pb = pale_fraction(B.c.views, luma_min=self.s.s3_pale_luma, sat_max=self.s.s3_pale_sat)
        if max(pa, pb) < self.s.s3_pale_fraction:
            return {"fired": False, "pale": [pa, pb], "choice": None}
        r = await self._ask(self.pref, user_content(P.S3_GRAY_USER, prompt, A.gray(0), B.gray(0)), seed,
                            PreferenceReply(choice="draw"))
        return {"fired": True, "pale": [round(pa, 3), round(pb, 3)], "choice": None if r.choice == "draw" else r.choice}

    async def _s4(self, prompt, A, B, winner, seed) -> dict:
        W, L = (A, B) if winner == "A" else (B, A)
        asks = [self._ask(self.pref, user_content(P.S4_SIDE_USER.format(angle=desc), prompt, W.white(v), L.white(v)),
                          seed, PreferenceReply(choice="draw")) for v, desc in self.s.s4_views]
        rs = await asyncio.gather(*asks)
        loser_pref = sum(r.choice == "B" for r in rs)          # "B" is the loser in this ordering
        return {"loser_prefs": loser_pref, "overturned": loser_pref >= self.s.s4_k}

    def _tie_break(self, A: Candidate, B: Candidate, ref_vec) -> Optional[str]:
        if ref_vec is None or A.embed is None or B.embed is None:
            return None
        sa, sb = float((A.embed @ ref_vec).max()), float((B.embed @ ref_vec).max())
        if abs(sa - sb) < 1e-6:
            return None
        return "A" if sa > sb else "B"

    async def duel(self, prompt_url: str, a: Candidate, b: Candidate, seed: int, ref_vec=None,
                   early_stop: bool = True) -> JudgeVerdict:
        purpose_var.set("judge")
        A, B = CandidateViews(a), CandidateViews(b)
        detail: Dict[str, Any] = {}
        s1 = await self._s1(prompt_url, A, B, seed, early_stop)
        detail["s1"] = s1
        winner, by = s1["choice"], "S1"
        if winner == "draw" and self.s.max_stage >= 2:
            s2 = await self._s2(prompt_url, A, B, ref_vec, seed)
            detail["s2"] = s2
            winner, by = s2["choice"], f"S2 {s2['source']}"
            if winner == "draw" and self.s.max_stage >= 3:
                s3 = await self._s3(prompt_url, A, B, seed)
                detail["s3"] = s3
                if s3["choice"]:
                    winner, by = s3["choice"], "S3 gray"
        if winner != "draw" and self.s.max_stage >= 4 and by != "S1":
            s4 = await self._s4(prompt_url, A, B, winner, seed)
            detail["s4"] = s4
            if s4["overturned"]:
                winner, by = "draw", "S4 side guard"
        if winner == "draw":
            tb = self._tie_break(a, b, ref_vec)
            if tb is not None:
                winner, by = tb, by + " -> embed tie-break"
        conf = min(1.0, 0.5 + abs(s1["mean_diff"]) / 10) if winner != "draw" else 0.5
        return JudgeVerdict(winner=winner, decided_by=by, confidence=conf, detail=detail)
