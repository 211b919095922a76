"""Generation-service settings: YAML -> environment rewriters -> validated pydantic model.

Reference: `SettingsConf` and its sections (pipeline_service/config/settings.py:20-347), loaded from
configuration.yaml, with environment rewriters applied to the raw dict before validation
(pipeline_service/pgh_mix.py two-coder mix, pgh_rslots.py render slots, pgh_gsplit.py GPU split,
pgh_mcache.py cache sizing).

Rewriters here (all act on the raw dict, before validation, and record what they changed in `notes`):
  PHX_K=<int>                      coder ensemble size (K candidates per prompt)
  PHX_RENDER_SLOTS=<int>           concurrent renders
  PHX_MIX=<clientA>:<w>,<clientB>:<w>  spread coder calls over several coder clients with weights
  PHX_GPU_SPLIT=<client>=<ids>;... GPU ids per local engine client
  PHX_SET=a.b.c=value;...          generic dotted overrides (values parsed as YAML scalars)
"""
from __future__ import annotations

import copy
import os
from typing import Any, Dict, List, Optional

import yaml
from pydantic import BaseModel, Field, field_validator, model_validator


class APIConfig(BaseModel):
    host: str = "0.0.0.0"
    port: int = 10006
    debug: bool = False


class CoderProbeConfig(BaseModel):
    enabled: bool = True
    concurrency: int = 16
    max_tokens: int = 256
    min_tps: float = 0.0
    timeout_s: float = 300.0


class PreflightConfig(BaseModel):
    min_tflops: Optional[float] = None
    min_hbm_gbs: Optional[float] = None
    min_power_limit_w: Optional[float] = None
    min_download_mbps: Optional[float] = None


class KPolicyConfig(BaseModel):
    """Candidate-count policies (app/kpolicy.py); every one is off unless configured."""
    start: str = "fixed"               # start-up K: fixed | cpu (cores / cpu_per_candidate cap) | off
    cpu_per_candidate: float = 0.25
    k_min: int = 2
    guard: str = "off"                 # round-budget guard: live | shadow | off
    round_batches: int = 4
    round_s: float = 7200.0
    margin_s: float = 250.0
    overhead_s: float = 90.0
    steps: List[float] = Field(default_factory=lambda: [0.85, 0.7, 0.55, 0.4, 0.25])
    k_floor: int = 2
    idle_reset_s: float = 900.0
    budget: bool = False               # per-prompt token budget K (BudgetK)
    budget_lo: float = 0.5
    budget_hi: float = 1.5
    budget_min_ref: int = 8
    render_brake: bool = False         # hold coder launches while renders are backed up
    render_backlog: float = 4.0

    @field_validator("start")
    @classmethod
    def _start(cls, v):
        if v not in ("fixed", "cpu", "off"):
            raise ValueError(f"k_policy.start must be fixed, cpu or off, got {v!r}")
        return v

    @field_validator("guard")
    @classmethod
    def _guard(cls, v):
        if v not in ("live", "shadow", "off"):
            raise ValueError(f"k_policy.guard must be live, shadow or off, got {v!r}")
        return v


class PipelineConfig(BaseModel):
    batch_time_budget: float = 1800.0
    batch_margin_s: float = 120.0
    candidate_deadline_s: float = 0.0
    prompt_timeout: float = 120.0
    use_planner: bool = False
    refinement_enabled: bool = False
    round_robin: int = 0               # 0 off; 4: the last four (quarter winners) play all pairs; 8: the last eight
    round_robin_tail: int = 4          # with 8: the batch's last N prompts keep the 4-player round robin
    s1_early_stop_max_round: int = 0   # judge S1 early stop only in bracket rounds <= this (0 = every round)
    shadow: List[str] = Field(default_factory=list)   # selection features to record without shipping: rr4, rr8
    shadow_max_duels: int = 12
    max_attempts: int = 3
    salvage: bool = True
    seed_offset: int = 0
    coder_probe: CoderProbeConfig = Field(default_factory=CoderProbeConfig)
    k_policy: KPolicyConfig = Field(default_factory=KPolicyConfig)

    @field_validator("round_robin", mode="before")
    @classmethod
    def _rr(cls, v):
        if isinstance(v, bool):              # a yes/no switch means the 4-player round robin
            return 4 if v else 0
        if v not in (0, 4, 8):
            raise ValueError(f"pipeline.round_robin must be 0, 4 or 8 (or a bool), got {v!r}")
        return v


class EngineServeConfig(BaseModel):
    """How to launch a local engine (phung5_b200.serve.server) for a client."""
    model: str = "small-bf16"
    port: Optional[int] = None
    gpu_ids: str = "auto"
    tensor_parallel_size: int = 1
    data_parallel_size: int = 1
    spec: str = "tree"
    max_num_seqs: int = 64
    extra_args: List[str] = Field(default_factory=list)


class LLMClientConfig(BaseModel):
    base_url: str
    api_key_env: str = ""
    api_key: str = ""
    enabled: bool = False
    request_timeout_s: float = 900.0
    engine: Optional[EngineServeConfig] = None

    @property
    def local(self) -> bool:
        u = self.base_url.lower()
        return any(h in u for h in ("localhost", "127.0.0.1", "0.0.0.0"))

    def key(self) -> str:
        return self.api_key or (os.environ.get(self.api_key_env, "") if self.api_key_env else "")


class ActorConfig(BaseModel):
    client: str = ""
    extra_clients: List[str] = Field(default_factory=list)
    client_weights: List[int] = Field(default_factory=list)
    model: str = ""
    workers: int = 16
    max_tokens: int = 4096
    temperature: float = 0.7
    top_p: float = 0.95
    seed: int = 42
    ensemble_size: int = 1
    max_repairs: int = 2
    max_stage: int = 4


class CoderConfig(ActorConfig):
    ensemble_size: int = 8
    workers: int = 64
    max_tokens: int = 8192


class JudgeConfig(ActorConfig):
    temperature: float = 0.0
    workers: int = 32


class WorkerPoolConfig(ActorConfig):
    workers: int = 4
    processes: bool = False          # checker: a process pool (the interpreter is CPU-bound Python) instead of threads


class ActorsConfig(BaseModel):
    planner: ActorConfig = Field(default_factory=ActorConfig)
    coder: CoderConfig = Field(default_factory=CoderConfig)
    critic: ActorConfig = Field(default_factory=ActorConfig)
    judge: JudgeConfig = Field(default_factory=JudgeConfig)
    checker: WorkerPoolConfig = Field(default_factory=lambda: WorkerPoolConfig(workers=8))
    renderer: WorkerPoolConfig = Field(default_factory=WorkerPoolConfig)


class EmbedderConfig(BaseModel):
    enabled: bool = True
    model_dir: Optional[str] = None
    device: Optional[str] = None
    batch_size: int = 8


class OrientationConfig(BaseModel):
    """Orientation stage (app/orient.py): probe renders + embeddings decide a rotation written into the module."""
    enabled: bool = True
    img_size: int = 160
    min_side_margin: float = 0.0
    # turned copies of the bracket's final (y180 / xm90 / xp90 / y180xm90), kept only after a decisive duel win
    final_enabled: bool = False
    final_turns: List[str] = Field(default_factory=lambda: ["y180", "xm90", "xp90"])
    final_min_margin: float = 0.05
    final_both_seats: bool = False


class EventBusConfig(BaseModel):
    max_iter: int = 2
    task_deadline_s: float = 2700.0
    score_threshold: float = 0.55


class BurstConfig(BaseModel):
    """Lend the coder GPUs to sleeping judge replicas in a batch's judge-only tail (app/burst.py)."""
    enabled: bool = False
    proxy_url: str = ""                                   # the coder engines' router (park / unpark)
    coder_upstreams: List[str] = Field(default_factory=list)   # engines behind it to park (empty: all active)
    judge_replicas: List[str] = Field(default_factory=list)    # sleeping judge engines on the coder GPUs
    delay_s: float = 2.0                                  # quiet period after coding ends before the swap
    drain_s: float = 60.0


class Settings(BaseModel):
    api: APIConfig = Field(default_factory=APIConfig)
    pipeline: PipelineConfig = Field(default_factory=PipelineConfig)
    preflight: PreflightConfig = Field(default_factory=PreflightConfig)
    benchmark: bool = True
    warmup: bool = True
    llm_clients: Dict[str, LLMClientConfig] = Field(default_factory=dict)
    embedder: EmbedderConfig = Field(default_factory=EmbedderConfig)
    orientation: OrientationConfig = Field(default_factory=OrientationConfig)
    actors: ActorsConfig = Field(default_factory=ActorsConfig)
    event_bus: EventBusConfig = Field(default_factory=EventBusConfig)
    burst: BurstConfig = Field(default_factory=BurstConfig)
    notes: List[str] = Field(default_factory=list)

    @field_validator("llm_clients")
    @classmethod
    def _urls(cls, v):
        for name, c in v.items():
            if not c.base_url.startswith(("http://", "https://")):
                raise ValueError(f"llm_clients.{name}.base_url must be http(s)")
        return v

    @model_validator(mode="after")
    def _actors_reference_clients(self):
        for role in ("planner", "coder", "critic", "judge"):
            a: ActorConfig = getattr(self.actors, role)
            for c in [a.client, *a.extra_clients]:
                if c and c not in self.llm_clients:
                    raise ValueError(f"actors.{role} names unknown client {c!r}")
            if a.client_weights and len(a.client_weights) != 1 + len(a.extra_clients):
                raise ValueError(f"actors.{role}.client_weights needs one weight per client")
        if self.actors.coder.ensemble_size < 1:
            raise ValueError("actors.coder.ensemble_size must be >= 1")
        return self

    def enabled_clients(self) -> Dict[str, LLMClientConfig]:
        return {k: v for k, v in self.llm_clients.items() if v.enabled}


# ------------------------------------------------------------------------------------------------ rewriters


def _set_path(d: dict, path: str, value) -> None:
    keys = path.split(".")
    cur = d
    for k in keys[:-1]:
        cur = cur.setdefault(k, {})
    cur[keys[-1]] = value


def apply_env(raw: dict, env: Optional[dict] = None) -> dict:
    env = os.environ if env is None else env
    d = copy.deepcopy(raw)
    notes = d.setdefault("notes", [])
    k = env.get("PHX_K", "").strip()
    if k:
        if not k.isdigit() or int(k) < 1:
            notes.append(f"!! PHX_K={k!r} ignored (want a positive integer)")
        else:
            _set_path(d, "actors.coder.ensemble_size", int(k))
            notes.append(f"coder ensemble K={k}")
    rs = env.get("PHX_RENDER_SLOTS", "").strip()
    if rs.isdigit() and int(rs) > 0:
        _set_path(d, "actors.renderer.workers", int(rs))
        notes.append(f"render slots={rs}")
    mix = env.get("PHX_MIX", "").strip()
    if mix:
        try:
            pairs = [p.split(":") for p in mix.split(",") if p]
            names = [p[0] for p in pairs]
            weights = [int(p[1]) if len(p) > 1 else 1 for p in pairs]
            coder = d.setdefault("actors", {}).setdefault("coder", {})
            coder["client"], coder["extra_clients"], coder["client_weights"] = names[0], names[1:], weights
            for n in names:
                d.setdefault("llm_clients", {}).get(n, {})["enabled"] = True
            notes.append(f"coder mix {dict(zip(names, weights))}")
        except (ValueError, IndexError):
            notes.append(f"!! PHX_MIX={mix!r} ignored (want name:weight,...)")
    split = env.get("PHX_GPU_SPLIT", "").strip()
    if split:
        for part in split.split(";"):
            if "=" not in part:
                continue
            name, ids = part.split("=", 1)
            cl = d.setdefault("llm_clients", {}).get(name.strip())
            if cl is None:
                notes.append(f"!! PHX_GPU_SPLIT names unknown client {name!r}")
                continue
            cl.setdefault("engine", {})["gpu_ids"] = ids.strip()
            notes.append(f"{name.strip()} gpus={ids.strip()}")
    gen = env.get("PHX_SET", "").strip()
    if gen:
        for part in gen.split(";"):
            if "=" in part:
                path, val = part.split("=", 1)
                _set_path(d, path.strip(), yaml.safe_load(val))
                notes.append(f"set {path.strip()}={val.strip()}")
    return d


def load_settings(path: Optional[str] = None, env: Optional[dict] = None, raw: Optional[dict] = None) -> Settings:
    if raw is None:
        raw = {}
        if path:
            with open(path) as f:
                raw = yaml.safe_load(f) or {}
    return Settings.model_validate(apply_env(raw, env))
