"""Per-batch accounting for the results header: LLM calls per role, duels, renders, engine counters, cgroup CPU.

Reference: `BatchStats` (pipeline_service/pipeline/batch_stats.py:109-271), which also scrapes engine
counters and cgroup CPU time. Engine counters come from this framework's server `/metrics` (phx_* series, summed over
replicas); the CPU axis is cgroup v2 `cpu.stat` (v1 cpuacct fallback).
Header tokens: end=<s> coder=<n>/<err>/<p50 s>/<ctok> judge=... duels=<n>/<p50>/<p95>/<wait p95>
render=<n>/<fail>/<p50>/<p95> tail=<s since last coder reply> <tag>=<tokens>/<steps>/<accept> cpu=<cores>/<thr%>.
"""
from __future__ import annotations

import time
from collections import Counter
from pathlib import Path
from typing import Any, Dict, List, NamedTuple, Optional

from .session import CALL_LOG, CallLog

ENGINE_COUNTERS = ("phx_generated_tokens_total", "phx_engine_steps_total", "phx_accepted_draft_tokens_total")
ENGINE_GAUGES = ("phx_num_running", "phx_num_waiting", "phx_kv_free_pages")


def _close_brace(s: str) -> int:
    """Index of the '}' that closes the label set opening s (s[0] == '{'); quoted label values may hold
    braces, spaces and escaped quotes. -1 if the set is not closed."""
    in_str = escaped = False
    for i in range(1, len(s)):
        ch = s[i]
        if in_str:
            if escaped:
                escaped = False
            elif ch == "\\":
                escaped = True
            elif ch == '"':
                in_str = False
        elif ch == '"':
            in_str = True
        elif ch == "}":
            return i
    return -1


def iter_samples(text: str):
    """(metric name, value) of every sample line of a Prometheus text exposition (labels and the optional
    timestamp are skipped; malformed lines are ignored)."""
    for raw in text.splitlines():
        line = raw.strip()
        if not line or line.startswith("#"):
            continue
        cut = next((i for i, ch in enumerate(line) if ch == "{" or ch.isspace()), len(line))
        name, rest = line[:cut], line[cut:]
        if rest.startswith("{"):
            end = _close_brace(rest)
            if end < 0:
                continue
            rest = rest[end + 1:]
        fields = rest.split()
        if not fields:
            continue
        try:
            yield name, float(fields[0])
        except ValueError:
            continue


def parse_metrics(text: str, names=ENGINE_COUNTERS + ENGINE_GAUGES) -> Dict[str, float]:
    """Per metric name in `names`: the sum over all of its labelled series."""
    wanted = set(names)
    totals: Counter = Counter()
    for name, value in iter_samples(text):
        if name in wanted:
            totals[name] += value
    return dict(totals)


class CpuTimes(NamedTuple):
    """CPU time charged to this cgroup since it was created."""
    used_s: float
    throttled_s: float
    periods: int
    throttled_periods: int


def _int_table(path: Path) -> Dict[str, int]:
    """'key value' lines with integer values (cgroup stat files); {} if the file cannot be read."""
    try:
        lines = path.read_text().splitlines()
    except OSError:
        return {}
    table = {}
    for line in lines:
        parts = line.split()
        if len(parts) == 2 and parts[1].isdigit():
            table[parts[0]] = int(parts[1])
    return table


def read_cgroup_cpu(root: str = "/sys/fs/cgroup") -> Optional[CpuTimes]:
    """CPU usage and throttling of this cgroup: cgroup v2 `cpu.stat` (microseconds), else the v1 pair
    `cpuacct/cpuacct.usage` (nanoseconds) + `cpu/cpu.stat`; None when neither is readable."""
    base = Path(root)
    v2 = _int_table(base / "cpu.stat")
    if "usage_usec" in v2:
        return CpuTimes(v2["usage_usec"] * 1e-6, v2.get("throttled_usec", 0) * 1e-6, v2.get("nr_periods", 0),
                        v2.get("nr_throttled", 0))
    try:
        used_ns = int((base / "cpuacct" / "cpuacct.usage").read_text().strip())
    except (OSError, ValueError):
        return None
    v1 = _int_table(base / "cpu" / "cpu.stat")
    return CpuTimes(used_ns * 1e-9, v1.get("throttled_time", 0) * 1e-9, v1.get("nr_periods", 0),
                    v1.get("nr_throttled", 0))


def cpu_quota(root: str = "/sys/fs/cgroup") -> Optional[float]:
    """CPUs allowed by the cgroup (cpu.max quota/period), None when unlimited or unknown."""
    try:
        p = Path(root) / "cpu.max"
        if p.exists():
            q, per = p.read_text().split()[:2]
            return None if q == "max" else float(q) / float(per)
        q = Path(root) / "cpu" / "cpu.cfs_quota_us"
        per = Path(root) / "cpu" / "cpu.cfs_period_us"
        if q.exists() and per.exists():
            qv = float(q.read_text())
            return None if qv <= 0 else qv / float(per.read_text())
    except (OSError, ValueError):
        return None
    return None


def _pct(xs: List[float], q: float) -> Optional[float]:
    if not xs:
        return None
    s = sorted(xs)
    return s[min(len(s) - 1, int(q * (len(s) - 1) + 0.5))]


def _fmt(x: Optional[float]) -> str:
    return "?" if x is None else f"{x:.1f}"


class BatchStats:
    def __init__(self, log: CallLog = CALL_LOG):
        self.log = log
        self.reset(time.time())

    def reset(self, now: Optional[float] = None) -> None:
        self.started_at = now or time.time()
        self.ended_at: Optional[float] = None
        self.log_idx = len(self.log.records)
        self.t_last_coder: Optional[float] = None
        self.duels = {"lat": [], "wait": []}
        self.render = {"n": 0, "fail": 0, "lat": []}
        self.engine: Dict[str, List[Dict[str, float]]] = {}
        self.cpu0 = read_cgroup_cpu()
        self.cpu1: Optional[CpuTimes] = None
        self.roles: Dict[str, str] = {}

    def end(self) -> None:
        self.ended_at = time.time()
        self.cpu1 = read_cgroup_cpu()

    def duel(self, seconds: float, wait: float) -> None:
        self.duels["lat"].append(seconds)
        self.duels["wait"].append(wait)

    def rendered(self, seconds: float, ok: bool) -> None:
        self.render["n"] += 1
        self.render["fail"] += 0 if ok else 1
        self.render["lat"].append(seconds)

    def engine_snapshot(self, name: str, metrics_text: str) -> None:
        self.engine.setdefault(name, []).append(parse_metrics(metrics_text))

    def _llm(self, role: str) -> str:
        recs = [r for r in self.log.since(self.log_idx) if self.roles.get(r.client, r.client).startswith(role)]
        if not recs:
            return f"{role}=0"
        err = sum(not r.ok for r in recs)
        ctok = sum(r.completion_tokens for r in recs)
        return f"{role}={len(recs)}/{err}/{_fmt(_pct([r.seconds for r in recs], 0.5))}/{ctok}"

    def header_parts(self) -> List[str]:
        end = self.ended_at or time.time()
        parts = [f"end={end - self.started_at:.0f}", self._llm("coder"), self._llm("judge")]
        d = self.duels
        parts.append(f"duels={len(d['lat'])}/{_fmt(_pct(d['lat'], .5))}/{_fmt(_pct(d['lat'], .95))}/{_fmt(_pct(d['wait'], .95))}")
        r = self.render
        parts.append(f"render={r['n']}/{r['fail']}/{_fmt(_pct(r['lat'], .5))}/{_fmt(_pct(r['lat'], .95))}")
        coder_recs = [x for x in self.log.since(self.log_idx) if self.roles.get(x.client, x.client).startswith("coder")]
        if coder_recs:
            last = self.started_at + sum(x.seconds for x in coder_recs[-1:])
            parts.append(f"tail={max(0.0, end - last):.0f}")
        for name, snaps in sorted(self.engine.items()):
            if len(snaps) >= 2:
                a, b = snaps[0], snaps[-1]
                dtok = b.get("phx_generated_tokens_total", 0) - a.get("phx_generated_tokens_total", 0)
                dst = b.get("phx_engine_steps_total", 0) - a.get("phx_engine_steps_total", 0)
                dacc = b.get("phx_accepted_draft_tokens_total", 0) - a.get("phx_accepted_draft_tokens_total", 0)
                parts.append(f"{name}={dtok:.0f}/{dst:.0f}/{(dacc / dst if dst else 0):.2f}")
        if self.cpu0 and self.cpu1:
            wall = max(1e-6, (self.ended_at or end) - self.started_at)
            cores = (self.cpu1.used_s - self.cpu0.used_s) / wall
            thr = (self.cpu1.throttled_s - self.cpu0.throttled_s) / wall
            parts.append(f"cpu={cores:.1f}/{100 * thr:.0f}")
        return parts

    def summary(self) -> Dict[str, Any]:
        return {"llm": self.log.summary(self.log.since(self.log_idx)), "duels": len(self.duels["lat"]),
                "renders": self.render["n"], "render_failures": self.render["fail"]}
