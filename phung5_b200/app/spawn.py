"""Engine spawner: client config -> GPU allocation -> one engine server command per replica (+ a router).

Reference: `pipeline_service/llm/spawn.py:25-392` (`_allocate_gpus` :147-205, `_build_cmd` :272-294) starts one
`vllm serve` per local client. Here the engines are this framework's own server
(`python -m phung5_b200.serve.server`; tensor parallel replicas under `torch.distributed.run`, one process
per GPU, rank 0 serving HTTP), and a client with data parallelism > 1 gets one replica per GPU group behind
the least-in-flight router (`python -m phung5_b200.serve.router`) on the client's port.

GPU allocation, in order: explicit `gpu_ids` are reserved first (unknown or doubly reserved ids are
errors); then clients with an explicit tensor_parallel_size take tp * dp GPUs from what is free; the rest
("auto") split the remaining GPUs evenly, earlier clients taking the remainder. A job's tp defaults to
its GPU count / dp and must divide it exactly.
"""
from __future__ import annotations

import os
import subprocess
import sys
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional
from urllib.parse import urlparse

from .settings import LLMClientConfig, Settings


@dataclass
class EngineJob:
    name: str
    model: str
    port: int
    gpu_ids: List[str]
    tp: int
    dp: int
    spec: str = "tree"
    extra_args: List[str] = field(default_factory=list)
    max_num_seqs: int = 64

    def replica_gpus(self) -> List[List[str]]:
        return [self.gpu_ids[i * self.tp:(i + 1) * self.tp] for i in range(self.dp)]

    def replica_ports(self) -> List[int]:
        return [self.port] if self.dp == 1 else [self.port + 100 + i for i in range(self.dp)]


def detect_gpus() -> List[str]:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis is not None and vis.strip():
        return [g.strip() for g in vis.split(",") if g.strip()]
    try:
        out = subprocess.run(["nvidia-smi", "--query-gpu=index", "--format=csv,noheader"], capture_output=True,
                             text=True, timeout=30)
        return [ln.strip() for ln in out.stdout.splitlines() if ln.strip()]
    except (OSError, subprocess.TimeoutExpired):
        return []


def allocate_gpus(clients: Dict[str, LLMClientConfig], all_gpus: List[str]) -> Dict[str, List[str]]:
    specs = {n: c.engine for n, c in clients.items() if c.engine is not None}
    assigned: Dict[str, List[str]] = {}
    used: set = set()
    for n, e in specs.items():
        if e.gpu_ids not in ("", "auto"):
            ids = [g.strip() for g in e.gpu_ids.split(",") if g.strip()]
            for g in ids:
                if g not in all_gpus:
                    raise ValueError(f"{n}: gpu_ids includes {g!r} but visible GPUs are {all_gpus}")
                if g in used:
                    raise ValueError(f"{n}: GPU {g} already reserved by another client")
                used.add(g)
            assigned[n] = ids
    free = [g for g in all_gpus if g not in used]
    for n, e in specs.items():
        explicit_tp = "tensor_parallel_size" in e.model_fields_set
        if n in assigned or not explicit_tp:
            continue
        need = e.tensor_parallel_size * max(1, e.data_parallel_size)
        if len(free) < need:
            raise ValueError(f"{n}: needs {need} GPU(s) (tp {e.tensor_parallel_size} x dp {e.data_parallel_size}) "
                             f"but {len(free)} are free")
        assigned[n], free = free[:need], free[need:]
    auto = [n for n in specs if n not in assigned]
    if auto:
        if len(free) < len(auto):
            raise ValueError(f"{len(auto)} auto client(s) but only {len(free)} free GPU(s)")
        per, rem = divmod(len(free), len(auto))
        i = 0
        for j, n in enumerate(auto):
            k = per + (1 if j < rem else 0)
            assigned[n] = free[i:i + k]
            i += k
    return assigned


def build_jobs(settings: Settings, all_gpus: Optional[List[str]] = None, base_port: int = 8001) -> List[EngineJob]:
    clients = {n: c for n, c in settings.enabled_clients().items() if c.local and c.engine is not None}
    if not clients:
        return []
    gpus = detect_gpus() if all_gpus is None else all_gpus
    assigned = allocate_gpus(clients, gpus)
    jobs = []
    for n, c in clients.items():
        e = c.engine
        ids = assigned[n]
        dp = max(1, e.data_parallel_size)
        tp = e.tensor_parallel_size if "tensor_parallel_size" in e.model_fields_set else max(1, len(ids) // dp)
        if tp * dp != len(ids):
            raise ValueError(f"{n}: tp {tp} x dp {dp} != {len(ids)} assigned GPU(s) {ids}")
        port = e.port or urlparse(c.base_url).port or base_port
        jobs.append(EngineJob(n, e.model, port, ids, tp, dp, e.spec, list(e.extra_args), e.max_num_seqs))
    return jobs


def build_commands(job: EngineJob, python: str = sys.executable, master_port0: int = 29600) -> List[dict]:
    """-> [{"name", "cmd", "env"}] : one per replica, plus the router when dp > 1."""
    out = []
    for r, (gids, port) in enumerate(zip(job.replica_gpus(), job.replica_ports())):
        env = {"CUDA_VISIBLE_DEVICES": ",".join(gids)}
        serve = ["-m", "phung5_b200.serve.server", "--model", job.model, "--port", str(port), "--spec", job.spec,
                 "--max-num-seqs", str(job.max_num_seqs), *job.extra_args]
        if job.tp > 1:
            cmd = [python, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={job.tp}",
                   "--master-addr=127.0.0.1", f"--master-port={master_port0 + job.port % 1000 + r}", *serve]
        else:
            cmd = [python, *serve]
        out.append({"name": f"{job.name}-r{r}", "cmd": cmd, "env": env})
    if job.dp > 1:
        cmd = [python, "-m", "phung5_b200.serve.router", "--port", str(job.port)]
        for p in job.replica_ports():
            cmd += ["--upstream", f"http://127.0.0.1:{p}"]
        out.append({"name": f"{job.name}-router", "cmd": cmd, "env": {}})
    return out


class Spawner:
    def __init__(self, settings: Settings, log_dir: str = "logs", all_gpus: Optional[List[str]] = None):
        self.jobs = build_jobs(settings, all_gpus)
        self.log_dir = log_dir
        self.procs: List[tuple] = []

    def start(self) -> None:
        os.makedirs(self.log_dir, exist_ok=True)
        for job in self.jobs:
            for spec in build_commands(job):
                logf = open(os.path.join(self.log_dir, spec["name"] + ".log"), "ab")
                p = subprocess.Popen(spec["cmd"], env={**os.environ, **spec["env"]}, stdout=logf,
                                     stderr=subprocess.STDOUT, start_new_session=True)
                self.procs.append((spec["name"], p, logf))

    def alive(self) -> Dict[str, Optional[int]]:
        return {n: p.poll() for n, p, _ in self.procs}

    def stop(self, timeout: float = 30.0) -> None:
        import signal
        for _, p, _ in self.procs:
            if p.poll() is None:
                try:
                    os.killpg(p.pid, signal.SIGTERM)
                except ProcessLookupError:
                    pass
        t0 = time.time()
        for _, p, f in self.procs:
            try:
                p.wait(timeout=max(0.1, timeout - (time.time() - t0)))
            except subprocess.TimeoutExpired:
                try:
                    os.killpg(p.pid, signal.SIGKILL)
                except ProcessLookupError:
                    pass
            f.close()
