"""Per-batch service state: the task envelope, the miner state machine and the results diagnostics header.

Reference: `MinerState` / `MinerStatus` / `ServiceState` (pipeline_service/pipeline/state.py:11-102),
`PipelineTask` (pipeline/task.py:32-...), `_diag_header` (serve.py:107-137).

State machine:  WARMING_UP --(engines healthy, probe done)--> READY --(POST /generate)--> GENERATING
                --(batch done)--> COMPLETE --(POST /generate)--> GENERATING ...
                any --(engine down with no replacement budget)--> REPLACE; a /status poll reporting
                replacements_remaining == 0 on REPLACE forces WARMING_UP (try to generate anyway).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Dict, List, Optional

from .schemas import StatusResponse


class ServiceState(Enum):
    STARTING = "starting"
    RUNNING = "running"
    DOWN = "down"


class MinerStatus(str, Enum):
    WARMING_UP = "warming_up"
    READY = "ready"
    GENERATING = "generating"
    COMPLETE = "complete"
    REPLACE = "replace"


@dataclass(eq=False)
class Candidate:
    """One coder output that passed the checker, with what the judge needs."""
    code: str
    digest: str
    coder: str
    scene: dict
    views: List[Any] = field(default_factory=list)        # judge views (HxWx4 uint8 tensors), white background
    gray_views: List[Any] = field(default_factory=list)   # same on gray (stage-3 rescue)
    embed: Optional[Any] = None                           # [V, D] view embeddings
    stats: Dict[str, Any] = field(default_factory=dict)
    wins: int = 0
    rr_points: float = 0.0


@dataclass(eq=False)
class PipelineTask:
    """The envelope threaded through every stage of one prompt's generation."""
    stem: str
    image_url: str
    seed: int = 42
    image_bytes: Optional[bytes] = None
    image_mime: str = "image/png"
    osd: Optional[str] = None                       # planner output (object structure description)
    js_code: Optional[str] = None                   # the answer
    scene_json: Optional[dict] = None
    js_errors: List[str] = field(default_factory=list)
    candidates: List[Candidate] = field(default_factory=list)
    n_generated: int = 0
    n_valid: int = 0
    n_duplicates: int = 0
    duels: int = 0
    iteration: int = 0
    score_history: List[float] = field(default_factory=list)
    best_score: float = -1.0
    critic_report: Optional[dict] = None
    judge_log: List[dict] = field(default_factory=list)
    started_at: float = 0.0
    finished_at: float = 0.0
    failed: bool = False
    failure_reason: Optional[str] = None
    done: bool = False
    attempts: int = 0
    salvaged: bool = False
    lead_round: int = -1                            # bracket round of the current leader (salvage)
    shadow: Optional[dict] = None                   # shadow picks: what unshipped selection features would pick
    budget_k: Optional[int] = None                  # drafts the per-prompt token budget gave this prompt
    batch_pos: int = 0
    batch_size: int = 1

    @property
    def elapsed(self) -> float:
        end = self.finished_at or time.time()
        return end - self.started_at if self.started_at else 0.0

    def fail(self, reason: str) -> None:
        self.failed = True
        self.failure_reason = reason

    def view(self, full: bool = False) -> dict:
        d = {"stem": self.stem, "status": "completed" if self.done else "pending", "failed": self.failed,
             "failure_reason": self.failure_reason, "generated": self.n_generated, "valid": self.n_valid,
             "duplicates": self.n_duplicates, "duels": self.duels, "iteration": self.iteration,
             "best_score": self.best_score, "elapsed_s": round(self.elapsed, 2), "salvaged": self.salvaged,
             "attempts": self.attempts, "code_bytes": len(self.js_code or "")}
        if full:
            d.update({"osd": self.osd, "js_code": self.js_code, "js_errors": self.js_errors[-10:],
                      "critic": self.critic_report, "judge_log": self.judge_log[-32:], "shadow": self.shadow,
                      "score_history": self.score_history})
        elif self.osd:
            d["osd_preview"] = (self.osd[:80] + "...") if len(self.osd) > 80 else self.osd
        return d


class MinerState:
    def __init__(self) -> None:
        self.status = MinerStatus.WARMING_UP
        self.total = 0
        self.batch_stems: List[str] = []
        self.seed = 0
        self.tasks: Dict[str, PipelineTask] = {}
        self.llm_status: Dict[str, ServiceState] = {}
        self.replacements_remaining = 0
        self.diag: Dict[str, Any] = {}
        self.batch_started_at: Optional[float] = None
        self.batch_index = 0
        self.stats_header: List[str] = []

    def reset_for_batch(self, stems: List[str], seed: int) -> None:
        self.total = len(stems)
        self.tasks = {}
        self.batch_stems = list(stems)
        self.seed = seed
        self.status = MinerStatus.GENERATING
        self.batch_started_at = time.time()
        self.batch_index += 1

    def record_task(self, task: PipelineTask) -> None:
        self.tasks[task.stem] = task

    @property
    def progress(self) -> int:
        return sum(1 for t in self.tasks.values() if t.done)

    @property
    def results(self) -> Dict[str, str]:
        return {s: t.js_code for s, t in self.tasks.items() if t.done and not t.failed and t.js_code}

    @property
    def failed(self) -> Dict[str, str]:
        out = {s: (t.failure_reason or "no code generated") for s, t in self.tasks.items()
               if t.done and (t.failed or not t.js_code)}
        for s in self.batch_stems:            # stems the batch never reached
            if s not in self.tasks and self.status == MinerStatus.COMPLETE:
                out[s] = "not processed"
        return out

    def mark_complete(self) -> None:
        self.status = MinerStatus.COMPLETE

    def set_llm_status(self, name: str, st: ServiceState) -> None:
        self.llm_status[name] = st

    def models_ready(self) -> bool:
        return all(s == ServiceState.RUNNING for s in self.llm_status.values())

    def any_down(self) -> bool:
        return any(s == ServiceState.DOWN for s in self.llm_status.values())

    def to_status_response(self) -> StatusResponse:
        payload = {"batch": self.batch_index, "failed": len(self.failed) if self.status == MinerStatus.COMPLETE else 0,
                   "llm": {k: v.value for k, v in self.llm_status.items()}}
        return StatusResponse(status=self.status.value, progress=self.progress, total=self.total, payload=payload)

    def diag_header(self) -> str:
        """One printable-ASCII comment line describing the host and the batch, prepended to each result."""
        d = self.diag

        def lst(v):
            if isinstance(v, list):
                return "/".join("?" if x is None else f"{float(x):.0f}" for x in v)
            return "?" if v is None else str(v)
        wall = int(time.time() - self.batch_started_at) if self.batch_started_at else None
        parts = [f"gpus={d.get('gpus', '?')}", f"tflops={lst(d.get('tflops'))}", f"hbm={lst(d.get('hbm_gbs'))}",
                 f"power={lst(d.get('power_w'))}", f"gsm={lst(d.get('gpu_sm'))}", f"gtemp={d.get('gpu_temp', '?')}",
                 f"gthr={d.get('gpu_thr', '?')}", f"gbad={d.get('gpu_bad', '?')}",
                 f"probe_tps={d.get('probe_tps', '?')}", f"cpu_quota={d.get('cpu_quota', '?')}/{d.get('nproc', '?')}",
                 f"net={d.get('net_mbps', '?')}", f"batch={self.batch_index}",
                 f"wall={wall if wall is not None else '?'}", f"seed={self.seed}"]
        if "k" in d:
            parts.append(f"k={d['k']}/{d.get('k_src', '?')}")
        parts += list(self.stats_header)
        line = "// miner-diag: " + " ".join(parts)
        return "".join(ch for ch in line if 32 <= ord(ch) < 127) + "\n"
