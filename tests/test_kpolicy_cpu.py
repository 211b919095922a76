"""K policies (app/kpolicy.py) and their wiring: start-up K from the cores, the round-budget guard, the per-prompt
token budget's top-up inside the bracket, and the render brake around the candidate factory."""
import asyncio
import math

from phung5_b200.app import kpolicy
from phung5_b200.app.agents import CoderResult
from phung5_b200.app.jscheck import CheckResult
from phung5_b200.app.kpolicy import BudgetK, RenderBrake, RoundGuard, detect_cores, guard_cut, replay, start_k
from phung5_b200.app.stages import CandidateFactory, StageLimits, multigen_first_iter
from phung5_b200.app.state import Candidate, PipelineTask


def test_detect_cores_takes_the_smallest_known_limit(tmp_path):
    (tmp_path / "cpu.max").write_text("400000 100000\n")
    assert detect_cores(str(tmp_path), lambda: 16, lambda: 64) == (4.0, "quota")
    (tmp_path / "cpu.max").write_text("max 100000\n")
    assert detect_cores(str(tmp_path), lambda: 16, lambda: 64) == (16.0, "affinity")
    v1 = tmp_path / "v1"
    (v1 / "cpu").mkdir(parents=True)
    (v1 / "cpu" / "cpu.cfs_quota_us").write_text("250000")
    (v1 / "cpu" / "cpu.cfs_period_us").write_text("100000")
    assert detect_cores(str(v1), lambda: 16, lambda: 64) == (2.5, "quota")
    assert detect_cores(str(tmp_path / "none"), lambda: None, lambda: None) == (None, "unknown")


def test_start_k_modes():
    assert start_k("fixed", 64, 4.0) == (64, "fixed")
    assert start_k("cpu", 64, 4.0) == (16, "cpu:4")
    assert start_k("cpu", 64, 100.0) == (64, "cpu:100")
    assert start_k("cpu", 64, None) == (64, "cpu:unknown-cores")
    assert start_k("off", 64, 4.0) == (64, "off")
    assert kpolicy.cpu_k(64, math.inf) == 64


def test_guard_cut_picks_the_largest_step_that_fits():
    # one 1800 s batch at K 64 (overhead 90 s): unit 26.7 s/draft; 3 batches left of 7000 s -> 1733 s each
    k, rec = guard_cut(64, 64, [(64, 1800.0)], 1, 4, 7200, 200, 90, (0.85, 0.7, 0.55), 2)
    assert k == 54 and rec["cut_to"] == 54 and rec["allowed"] == 1733.3
    # within budget: unchanged
    assert guard_cut(64, 64, [(64, 1500.0)], 1, 4, 7200, 200, 90, (0.85,), 2)[0] == 64
    # nothing fits: the floor
    assert guard_cut(64, 64, [(64, 7000.0)], 1, 4, 7200, 200, 90, (0.85, 0.5), 3)[0] == 3


def test_round_guard_rounds_idle_reset_shadow_and_replay():
    t = [0.0]
    g = RoundGuard(mode="live", round_s=7200, margin_s=200, clock=lambda: t[0])
    ks = []
    for wall in (1800, 1700, 1700, 1700, 1000):
        k = g.before_batch(64)
        ks.append(k)
        t[0] += wall
        g.after_batch(k, wall)
    assert ks == [64, 54, 54, 54, 64]          # cut inside the first round, never raised; new round -> start K
    t[0] += 2000                                # an idle gap longer than idle_reset_s starts a new round
    g.walls.append((64, 3000.0))
    assert g.before_batch(64) == 64 and g.walls == []
    sh = RoundGuard(mode="shadow", round_s=7200, margin_s=200, clock=lambda: 0.0)
    sh.before_batch(64)
    sh.after_batch(64, 1800)
    assert sh.before_batch(64) == 64 and sh.log[-1]["cut_to"] == 54     # decided and logged, not applied
    off = RoundGuard()
    off.after_batch(64, 99999)
    assert off.before_batch(64) == 64 and off.walls == []
    assert replay([1800] * 4 + [2500] * 4, 64, round_s=7200, margin_s=200) == [64, 54, 54, 54, 64, 35, 35, 35]


class _Factory:
    """multigen's view of a candidate factory: build(position) and drafts_of(positions)."""

    def __init__(self, nbytes):
        self.nbytes, self.built = nbytes, []
        self.sizes = {}
        self.cond = asyncio.Condition()

    async def build(self, k):
        self.built.append(k)
        await asyncio.sleep(0)
        async with self.cond:
            self.sizes[k] = self.nbytes
            self.cond.notify_all()
        return Candidate(code="x" * self.nbytes, digest=f"d{k}", coder="c", scene={}, stats={"k": k})

    async def drafts_of(self, positions):
        async with self.cond:
            await self.cond.wait_for(lambda: all(p in self.sizes for p in positions))
        return [self.sizes[p] for p in positions]


def _budget():
    b = BudgetK(min_ref=4, floor=4)
    for c in (1000, 2000, 4000, 8000):
        b.observe(c)
    b.batch_end()
    return b


def test_budget_k_tops_up_short_drafts_and_trims_long_ones_inside_the_bracket():
    async def duel(a, b, label):
        return a if a.stats["k"] < b.stats["k"] else b

    async def go(nbytes, budget):
        f = _Factory(nbytes)
        task = PipelineTask(stem="s", image_url="u")
        w = await multigen_first_iter(task, f, duel, 32, budget=budget)
        return sorted(f.built), task, w

    built, task, w = asyncio.run(go(800, _budget()))
    assert built[:16] == list(range(16)) and len(built) == task.budget_k > 32          # short drafts: more
    built, task, w = asyncio.run(go(9000, _budget()))
    assert len(built) == task.budget_k and 16 <= task.budget_k < 32 and w.stats["k"] == 0   # long: fewer
    built, task, _ = asyncio.run(go(800, BudgetK(min_ref=4)))                    # no reference yet: fixed K
    assert built == list(range(32)) and task.budget_k is None


class _Coder:
    name = "c"

    async def generate(self, prompt_url, seed, plan=None):
        code = f"export default function generate(THREE) {{ const s = {seed}; }}"
        return CoderResult(code, CheckResult(True, [], code, scene={"k": seed}), 1, 0)


class _Renderer:
    def __init__(self):
        self.backlog_seen = []

    async def judge_views(self, scene, gray=True):
        await asyncio.sleep(0.01)
        return {"white": [b"w"], "gray": [b"g"]}


def test_render_brake_counts_renders_and_holds_coders():
    async def go():
        brake = RenderBrake(slots=1, max_backlog=1.0)
        limits = StageLimits(asyncio.Semaphore(8), asyncio.Semaphore(8), asyncio.Semaphore(8))
        r = _Renderer()
        orig = r.judge_views

        async def views(scene, gray=True):
            r.backlog_seen.append(brake.backlog)
            return await orig(scene, gray)
        r.judge_views = views
        fac = CandidateFactory(PipelineTask(stem="s", image_url="u"), [_Coder()], r, None, limits, "data:", brake=brake)
        out = await asyncio.gather(*(fac.build(i) for i in range(6)))
        assert all(c is not None for c in out)
        assert brake.backlog == 0 and max(r.backlog_seen) >= 1
        assert sorted(fac.code_bytes) == list(range(6))
    asyncio.run(go())
