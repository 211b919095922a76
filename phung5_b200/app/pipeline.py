"""Generation pipeline: per-prompt orchestration and the batch loop.

References: `Pipeline` (pipeline_service/pipeline/orchestrator.py:22-259: prepare -> iteration 0 multigen +
bracket or code/check/render -> critic -> refine, per-stage semaphores, task deadline) and
`GenerationPipeline` (pipeline/generation_pipeline.py:83-517: builds clients and modules at startup, runs
batches with up to 3 attempts per prompt, a batch deadline with salvage of unfinished prompts, and the
coder throughput probe).

Per prompt (`Orchestrator.run_one`):
  1. prepare: fetch the prompt image (http(s), data: URL or local path) -> data URL; embed it; optional plan.
  2. iteration 0: K coders -> bracket (stages.multigen_first_iter); K == 1 is a single code/check/render.
  3. refinement (optional, `event_bus.max_iter` rounds): critic report on the current best's grid render,
     coder revision continuing the winning conversation, duel revision vs best, keep the winner; stop
     early when the critic score reaches `score_threshold`.
  The best candidate so far is kept on the task at every step, so a deadline can salvage it.
"""
from __future__ import annotations

import asyncio
import base64
import logging
import os
import time
from typing import Callable, Dict, List, Optional

import httpx

from ..serve.router import LoadBalancedClient, affinity_key
from .agents import CriticAgent, JudgeAgent, JudgeSettings, PlannerAgent, SceneCoderAgent, bytes_to_data_url
from .batch_stats import BatchStats
from .burst import BurstCoderBackend, BurstController
from .embed import Embedder, EmbedderSettings
from .jscheck import CheckerSettings, JSChecker, code_digest
from .kpolicy import BudgetK, RenderBrake, RoundGuard, detect_cores, start_k
from .renderer import RendererModule, RendererSettings
from .session import CALL_LOG, BackendError, HTTPBackend, ImageResendBackend, InstrumentedBackend, purpose_var
from .settings import Settings
from .stages import CandidateFactory, StageLimits, make_duel, multigen_first_iter
from .state import Candidate, MinerState, PipelineTask

log = logging.getLogger("phung5_b200.app")


async def fetch_image(url: str, http: Optional[httpx.AsyncClient] = None, timeout: float = 60.0) -> tuple:
    """-> (bytes, mime)."""
    if url.startswith("data:"):
        head, _, data = url.partition(",")
        mime = head[5:].split(";")[0] or "image/png"
        return base64.b64decode(data), mime
    if url.startswith(("http://", "https://")):
        client = http or httpx.AsyncClient(timeout=timeout)
        r = await client.get(url)
        r.raise_for_status()
        return r.content, r.headers.get("content-type", "image/png").split(";")[0]
    path = url[7:] if url.startswith("file://") else url
    with open(path, "rb") as f:
        data = f.read()
    return data, "image/png" if path.lower().endswith(".png") else "image/jpeg"


class Orchestrator:
    def __init__(self, coders: List[SceneCoderAgent], judge: Optional[JudgeAgent], critic: Optional[CriticAgent],
                 planner: Optional[PlannerAgent], renderer: RendererModule, embedder: Optional[Embedder],
                 settings: Settings, stats: Optional[BatchStats] = None, http: Optional[httpx.AsyncClient] = None):
        self.coders, self.judge, self.critic, self.planner = coders, judge, critic, planner
        self.renderer, self.embedder, self.s = renderer, embedder, settings
        self.stats = stats or BatchStats()
        self.http = http
        a = settings.actors
        self.limits = StageLimits(asyncio.Semaphore(a.coder.workers), asyncio.Semaphore(a.judge.workers),
                                  asyncio.Semaphore(a.renderer.workers))
        self.k = a.coder.ensemble_size
        kp = settings.pipeline.k_policy
        self.budget_k: Optional[BudgetK] = BudgetK(lo=kp.budget_lo, hi=kp.budget_hi, min_ref=kp.budget_min_ref) \
            if kp.budget else None
        self.brake: Optional[RenderBrake] = RenderBrake(a.renderer.workers, kp.render_backlog) \
            if kp.render_brake else None
        self.on_task_done: Optional[Callable[[str], None]] = None

    async def run_one(self, task: PipelineTask, deadline: Optional[float] = None) -> PipelineTask:
        task.started_at = task.started_at or time.time()
        affinity_key.set(task.stem)         # the task's LLM calls stick to one replica (prefix cache)
        try:
            await self._run(task, deadline)
        except asyncio.CancelledError:
            raise
        except Exception as e:  # noqa: BLE001 - one prompt never takes the batch down
            log.exception("task %s failed", task.stem)
            task.fail(f"{type(e).__name__}: {str(e)[:200]}")
        if not task.failed and not task.js_code:
            task.fail("no valid candidate")
        task.finished_at = time.time()
        task.done = True
        if self.on_task_done is not None:
            self.on_task_done(task.stem)
        return task

    async def _run(self, task: PipelineTask, deadline: Optional[float]):
        data, mime = await fetch_image(task.image_url, self.http)
        task.image_bytes, task.image_mime = data, mime
        prompt_url = bytes_to_data_url(data, mime)
        ref_vec = None
        if self.embedder is not None:
            v = await self.embedder.embed([data])
            ref_vec = None if v is None else v[0]
        plan_text = None
        if self.planner is not None and self.s.pipeline.use_planner:
            plan = await self.planner.plan(prompt_url, task.seed)
            if plan is not None:
                plan_text = plan.render()
                task.osd = plan_text
        cand_deadline = deadline
        if self.s.pipeline.candidate_deadline_s > 0:
            cd = time.monotonic() + self.s.pipeline.candidate_deadline_s
            cand_deadline = cd if deadline is None else min(deadline, cd)
        orient = None
        if self.s.orientation.enabled:
            from .orient import OrientSettings
            o = self.s.orientation
            orient = OrientSettings(enabled=True, img_size=o.img_size, min_side_margin=o.min_side_margin)
        checker = getattr(self.coders[0], "checker", None) if self.coders else None
        factory = CandidateFactory(task, self.coders, self.renderer, self.embedder, self.limits, prompt_url,
                                   plan_text, cand_deadline, ref_vec=ref_vec, checker=checker, orient=orient,
                                   brake=self.brake)
        duel = make_duel(task, self.judge, self.limits, prompt_url, ref_vec, on_duel=self.stats.duel,
                         es_max_round=self.s.pipeline.s1_early_stop_max_round) if self.judge is not None else None
        k = self.k
        if k > 1 and duel is not None:
            pc = self.s.pipeline
            rr = pc.round_robin
            if rr == 8 and task.batch_pos >= task.batch_size - pc.round_robin_tail:
                rr = 4                    # the batch's last prompts keep the cheaper 4-player round robin
            final_turn = None
            o = self.s.orientation
            if o.final_enabled and checker is not None and ref_vec is not None:
                from .orient import FinalTurnSettings, turn_final
                fts = FinalTurnSettings(enabled=True, turns=tuple(o.final_turns), min_margin=o.final_min_margin,
                                        both_seats=o.final_both_seats)

                judge, limits = self.judge, self.limits

                class _LimitedJudge:            # the stage's duels take the judge slots like the bracket's
                    async def duel(self, *a, **kw):
                        async with limits.judge:
                            return await judge.duel(*a, **kw)

                async def final_turn(win):
                    out, fres = await turn_final(win, renderer=self.renderer, embedder=self.embedder,
                                                 ref_vec=ref_vec, checker=checker, judge=_LimitedJudge(),
                                                 prompt_url=prompt_url, seed=task.seed, settings=fts)
                    out.stats["orient_final"] = {"picked": fres.picked, "replaced": fres.replaced,
                                                 "reason": fres.reason, "tried": fres.tried}
                    if fres.replaced:
                        task.judge_log.append({"label": "orient_final", "turn": fres.picked,
                                               "winner": "turned", "decided_by": "decisive duel"})
                    return out
            best = await multigen_first_iter(task, factory, duel, k, rr, pc.shadow, pc.shadow_max_duels,
                                             final_turn=final_turn, budget=self.budget_k)
        else:
            best = None
            for i in range(max(1, k)):
                best = await factory.build(i)
                if best is not None:
                    break
        if self.budget_k is not None and task.candidates:
            self.budget_k.observe(sum(len(c.code) for c in task.candidates) / len(task.candidates))
        if best is None:
            task.fail("no valid candidate: " + "; ".join(task.js_errors[-3:])[:400])
            return
        self._adopt(task, best)
        if not self.s.pipeline.refinement_enabled or self.critic is None:
            return
        for it in range(1, self.s.event_bus.max_iter + 1):
            if deadline is not None and time.monotonic() > deadline:
                break
            task.iteration = it
            grid = await self.renderer.grid_png(best.scene)
            report = await self.critic.review(prompt_url, grid, task.seed + it)
            task.critic_report = report.model_dump(mode="json")
            score = report.score() / 10.0
            task.score_history.append(score)
            task.best_score = max(task.best_score, score)
            if score >= self.s.event_bus.score_threshold or not report.issues:
                break
            issues = "\n".join(f"- [{i.kind.value}/{i.severity.value}] {i.target or ''}: {i.description}"
                               for i in report.worst())
            from . import prompts as P
            coder = next((c for c in self.coders if c.name == best.coder), self.coders[0])
            res = await coder.generate(prompt_url, task.seed + 1000 * it,
                                       user_text=P.REFINE_USER.format(issues=issues),
                                       history=[{"role": "assistant", "content": f"```js\n{best.code}\n```"}])
            if not res.check.ok:
                continue
            cand = Candidate(code=res.check.code, digest=code_digest(res.check.code), coder=coder.name,
                             scene=res.check.scene, stats={**res.check.stats, "k": f"refine{it}"})
            views = await self.renderer.judge_views(cand.scene)
            cand.views, cand.gray_views = views["white"], views.get("gray", [])
            if self.embedder is not None:
                cand.embed = await self.embedder.embed(cand.views)
            if duel is not None:
                best = await duel(best, cand, f"refine{it}")
            else:
                best = cand
            self._adopt(task, best)

    @staticmethod
    def _adopt(task: PipelineTask, c: Candidate) -> None:
        task.js_code = c.code
        task.scene_json = c.scene


class GenerationPipeline:
    """Owns the clients, modules and agents; runs batches into a MinerState."""

    def __init__(self, settings: Settings, state: MinerState, backends: Optional[Dict[str, object]] = None,
                 http: Optional[httpx.AsyncClient] = None):
        self.s = settings
        self.state = state
        self._backends_override = backends or {}
        self.http = http
        self.stats = BatchStats(CALL_LOG)
        self.checker = self.renderer = self.embedder = None
        self.orch: Optional[Orchestrator] = None
        kp = settings.pipeline.k_policy
        self.guard = RoundGuard(mode=kp.guard, round_batches=kp.round_batches, round_s=kp.round_s,
                                margin_s=kp.margin_s, overhead_s=kp.overhead_s, steps=tuple(kp.steps),
                                k_floor=kp.k_floor, idle_reset_s=kp.idle_reset_s)
        self.k0: Optional[int] = None
        self.burst: Optional[BurstController] = None
        self.current: Dict[str, PipelineTask] = {}
        self.probe_tps: Optional[float] = None

    # -------------------------------------------------------------------------------------------- startup

    def _backend(self, name: str):
        if name in self._backends_override:
            raw = self._backends_override[name]
        else:
            c = self.s.llm_clients[name]
            raw = HTTPBackend(c.base_url.rstrip("/").removesuffix("/v1"), c.request_timeout_s, api_key=c.key())
        return raw

    def _role_inner(self, role: str):
        """The raw backend of a role: one client; several real clients of a judging role (replicas of one model)
        -> a LoadBalancedClient (weighted, per-task affinity for the engines' prefix caches, load-aware
        migration); the coder's clients (a mix of coder models: every prompt's drafts spread over them) or
        injected backends -> a weighted per-call spread."""
        a = getattr(self.s.actors, role)
        names = [a.client, *a.extra_clients] if a.client else []
        if not names:
            return None
        weights = a.client_weights or [1] * len(names)
        if len(names) == 1:
            return self._backend(names[0])
        if role == "coder" or any(n in self._backends_override for n in names):
            return _MultiBackend([self._backend(n) for n in names], weights)
        cs = [self.s.llm_clients[n] for n in names]
        return LoadBalancedClient([c.base_url.rstrip("/").removesuffix("/v1") for c in cs], weights,
                                  client=self.http,
                                  headers=[{"Authorization": f"Bearer {c.key()}"} if c.key() else {} for c in cs],
                                  error=BackendError)

    def _wrap(self, role: str, inner):
        if inner is None:
            return None
        self.stats.roles[role] = role
        return InstrumentedBackend(ImageResendBackend(inner), role)

    def _role_backend(self, role: str):
        return self._wrap(role, self._role_inner(role))

    def _setup_burst(self, judge_inner) -> Optional[BurstController]:
        """The burst controller over the judge's load-balanced client, or None (off, or nothing to lend to)."""
        b = self.s.burst
        if not b.enabled:
            return None
        lb = judge_inner
        if isinstance(lb, HTTPBackend):
            lb = LoadBalancedClient([lb.url], headers=[lb.headers], error=BackendError)
        if not (hasattr(lb, "add_replicas") and hasattr(lb, "set_active")) or not b.proxy_url or not b.judge_replicas:
            log.warning("burst: needs a load-balanced judge client, burst.proxy_url and burst.judge_replicas; off")
            return None
        idxs = lb.add_replicas(b.judge_replicas, active=False)
        return BurstController(lb, idxs, b.proxy_url, b.coder_upstreams, http=self.http, delay_s=b.delay_s,
                               drain_s=b.drain_s)

    def startup(self) -> None:
        a = self.s.actors
        self.checker = JSChecker(CheckerSettings(workers=a.checker.workers, processes=a.checker.processes))
        self.renderer = RendererModule(RendererSettings(slots=a.renderer.workers))
        e = self.s.embedder
        self.embedder = Embedder(EmbedderSettings(enabled=e.enabled, model_dir=e.model_dir, device=e.device,
                                                  batch_size=e.batch_size)) if e.enabled else None
        coder_inner, judge_inner = self._role_inner("coder"), self._role_inner("judge")
        self.role_inner = {"coder": coder_inner, "judge": judge_inner}
        if coder_inner is None:
            raise ValueError("actors.coder.client is required")
        self.burst = self._setup_burst(judge_inner)
        if self.burst is not None:
            coder_inner, judge_inner = BurstCoderBackend(coder_inner, self.burst), self.burst.lb
        coder_be = self._wrap("coder", coder_inner)
        coders = [SceneCoderAgent(coder_be, a.coder.model, self.checker, name="coder", max_repairs=a.coder.max_repairs,
                                  max_tokens=a.coder.max_tokens, temperature=a.coder.temperature, top_p=a.coder.top_p)]
        judge_be = self._wrap("judge", judge_inner)
        judge = JudgeAgent(judge_be, a.judge.model, JudgeSettings(max_stage=a.judge.max_stage,
                                                                  concurrency=a.judge.workers,
                                                                  max_tokens=min(a.judge.max_tokens, 2048)),
                           embedder=self.embedder) if judge_be is not None else None
        critic_be = self._role_backend("critic")
        critic = CriticAgent(critic_be, a.critic.model) if critic_be is not None else None
        planner_be = self._role_backend("planner")
        planner = PlannerAgent(planner_be, a.planner.model) if planner_be is not None else None
        self.orch = Orchestrator(coders, judge, critic, planner, self.renderer, self.embedder, self.s, self.stats,
                                 self.http)
        if self.burst is not None:
            self.orch.on_task_done = self.burst.task_done
        kp = self.s.pipeline.k_policy
        cores = detect_cores()[0] if kp.start == "cpu" else None
        self.k0, src = start_k(kp.start, a.coder.ensemble_size, cores, kp.cpu_per_candidate, kp.k_min)
        self.orch.k = self.k0
        self.state.diag["k"], self.state.diag["k_src"] = self.k0, src

    # ----------------------------------------------------------------------------------------------- probe

    async def run_coder_probe(self) -> Optional[float]:
        """Aggregate coder output tokens/s at `concurrency` concurrent text-only requests: one untimed burst first
        (a fresh engine pays its CUDA-graph captures and first-touch allocations on it), then the timed burst.
        Records probe_tps (and probe_tps_cold, probe_errors) in the diag header; None if every call failed."""
        cfg = self.s.pipeline.coder_probe
        if not cfg.enabled or self.orch is None:
            return None
        be = self.orch.coders[0].session.backend
        model = self.orch.coders[0].session.model
        body = {"model": model, "max_tokens": cfg.max_tokens, "temperature": 0.7,
                "messages": [{"role": "user", "content": "Write a three.js function that builds a chair."}]}
        purpose_var.set("coder:probe")

        async def burst():
            t0 = time.monotonic()
            outs = await asyncio.wait_for(
                asyncio.gather(*(be.chat({**body, "seed": i}) for i in range(cfg.concurrency)),
                               return_exceptions=True), cfg.timeout_s)
            toks = sum(int((o.get("usage") or {}).get("completion_tokens", 0)) for o in outs if isinstance(o, dict))
            errs = [o for o in outs if not isinstance(o, dict)]
            return toks, max(time.monotonic() - t0, 1e-3), errs
        try:
            toks, dt, _ = await burst()
            self.state.diag["probe_tps_cold"] = round(toks / dt)
        except Exception as e:  # noqa: BLE001
            log.warning("coder probe warm-up burst failed (%s); timing the probe anyway", e)
        try:
            toks, dt, errs = await burst()
        except (asyncio.TimeoutError, Exception) as e:  # noqa: BLE001
            log.warning("coder probe failed: %s", e)
            self.state.diag["probe_tps"] = 0
            return 0.0
        self.state.diag["probe_errors"] = len(errs)
        if errs and not toks:
            self.state.diag["probe_tps"] = "?"
            return None
        self.probe_tps = toks / dt
        self.state.diag["probe_tps"] = f"{self.probe_tps:.0f}"
        log.info("coder probe: %d x %d tokens -> %d in %.1f s = %.0f tok/s (errors %d, min_tps %.0f)",
                 cfg.concurrency, cfg.max_tokens, toks, dt, self.probe_tps, len(errs), cfg.min_tps)
        return self.probe_tps

    def probe_ok(self, tps: Optional[float]) -> bool:
        """False when the coder probe measured less than pipeline.coder_probe.min_tps (0 = no floor)."""
        m = self.s.pipeline.coder_probe.min_tps
        return not (m > 0 and tps is not None and tps < m)

    # ----------------------------------------------------------------------------------------------- batch

    async def run_batch(self, tasks: List[PipelineTask]) -> None:
        if self.orch is None:
            self.startup()
        self.stats.reset()
        self.orch.k = self.guard.before_batch(self.k0)
        self.state.diag["k"] = self.orch.k
        if self.burst is not None:
            self.burst.batch_start(len(tasks), [t.stem for t in tasks])
        budget = self.s.pipeline.batch_time_budget
        eff = max(1.0, budget - self.s.pipeline.batch_margin_s)
        t_start = time.monotonic()
        deadline = t_start + eff
        task_deadline = self.s.event_bus.task_deadline_s

        for i, t in enumerate(tasks):
            t.batch_pos, t.batch_size = i, len(tasks)

        async def one(task: PipelineTask):
            attempt = 0
            while True:
                task.attempts = attempt + 1
                self.current[task.stem] = task
                dl = min(deadline, time.monotonic() + task_deadline) if task_deadline > 0 else deadline
                res = await self.orch.run_one(task, dl)
                if not res.failed or attempt + 1 >= self.s.pipeline.max_attempts or time.monotonic() >= deadline:
                    self.state.record_task(res)
                    return
                attempt += 1
                task = PipelineTask(stem=task.stem, image_url=task.image_url, seed=task.seed + 7 * attempt,
                                    batch_pos=task.batch_pos, batch_size=task.batch_size)

        try:
            await asyncio.wait_for(asyncio.gather(*(one(t) for t in tasks)), timeout=eff)
        except asyncio.TimeoutError:
            for t in tasks:
                rec = self.state.tasks.get(t.stem)
                if rec is not None and rec.done and not rec.failed:
                    continue
                cur = self.current.get(t.stem, t)
                if self.s.pipeline.salvage and cur.js_code:
                    cur.salvaged = True
                    cur.failed = False
                    cur.failure_reason = None
                else:
                    cur.fail(f"batch budget exceeded ({budget:.0f}s)")
                cur.done = True
                cur.finished_at = time.time()
                self.state.record_task(cur)
        finally:
            self.stats.end()
            wall = time.monotonic() - t_start
            self.guard.after_batch(self.orch.k, wall)
            if self.burst is not None:
                self.burst.batch_end()
                self.state.diag["burst"] = self.burst.state
            if self.orch is not None and self.orch.budget_k is not None:
                self.orch.budget_k.batch_end()
            self.state.stats_header = self.stats.header_parts()
            self.state.diag["last_wall"] = round(wall, 1)

    def close(self):
        for m in (self.checker, self.renderer):
            if m is not None:
                m.close()


class _MultiBackend:
    """Weighted spread over several clients of one role (e.g. two coder models, a mix)."""

    def __init__(self, backends: List[object], weights: List[int]):
        self.sched = [i for i, w in enumerate(weights) for _ in range(max(0, int(w)))] or [0]
        self.backends = backends
        self.i = 0

    async def chat(self, body: dict) -> dict:
        b = self.backends[self.sched[self.i % len(self.sched)]]
        self.i += 1
        return await b.chat(body)
