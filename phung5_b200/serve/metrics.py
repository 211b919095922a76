"""Engine metrics in Prometheus text format (tokens, steps, accept length, step latency, TPOT).

The reference scrapes vLLM/SGLang /metrics at batch start and end (pipeline_service/pipeline/
batch_stats.py:58-75); this is the engine's own exporter, built on prometheus_client with a private
registry so several engines in one process do not collide.
"""
from __future__ import annotations

from typing import List

from prometheus_client import CollectorRegistry, Counter, Gauge, Histogram, generate_latest


class EngineMetrics:
    def __init__(self):
        self.registry = CollectorRegistry()
        r = self.registry
        self.tokens = Counter("phx_generated_tokens", "output tokens emitted", registry=r)
        self.steps = Counter("phx_engine_steps", "engine steps", registry=r)
        self.accepted = Counter("phx_accepted_draft_tokens", "accepted draft tokens", registry=r)
        self.running = Gauge("phx_num_running", "running requests", registry=r)
        self.waiting = Gauge("phx_num_waiting", "waiting requests", registry=r)
        self.step_s = Histogram("phx_step_seconds", "wall time of one engine step", registry=r,
                                buckets=(0.001, 0.005, 0.01, 0.02, 0.05, 0.1, 0.2, 0.5, 1, 2, 5))
        self.tpot_s = Histogram("phx_time_per_output_token_seconds", "step time / tokens of a request in that step",
                                registry=r, buckets=(0.001, 0.002, 0.005, 0.01, 0.02, 0.05, 0.1, 0.2, 0.5))
        self.kv_free = Gauge("phx_kv_free_pages", "free KV pages", registry=r)

    def observe_step(self, dt: float, outs: List, engine) -> None:
        self.steps.inc()
        self.step_s.observe(dt)
        n = sum(len(o.new_tokens) for o in outs)
        self.tokens.inc(n)
        for o in outs:
            if o.new_tokens:
                self.tpot_s.observe(dt / len(o.new_tokens))
        self.running.set(len(engine.running))
        self.waiting.set(len(engine.waiting))
        self.kv_free.set(engine.pool.alloc.available())
        acc = engine.stats.get("accepted", 0)
        prev = getattr(self, "_acc_prev", 0)
        if acc > prev:
            self.accepted.inc(acc - prev)
        self._acc_prev = acc

    def render(self) -> str:
        return generate_latest(self.registry).decode()
