"""Service infrastructure on CPU: burst swaps (with undo), engine spawner GPU allocation and commands,
preflight against a fake NVML, CPU sets for worker pools, the process-pool checker."""
import asyncio
import math
import os

import httpx
import pytest

from phung5_b200.app.burst import BurstController
from phung5_b200.app.settings import load_settings
from phung5_b200.app.spawn import allocate_gpus, build_commands, build_jobs
from phung5_b200.serve.router import LoadBalancedClient
from phung5_b200.utils.affinity import core_groups, read_quota, worker_cpus
from phung5_b200.utils.preflight import run_preflight


def run(c):
    return asyncio.run(c)


class FakeNet:
    """Records POSTs; fails the paths listed in `fail`."""

    def __init__(self, fail=()):
        self.calls, self.fail = [], set(fail)

    def handler(self, req: httpx.Request):
        self.calls.append((req.method, str(req.url)))
        if str(req.url) in self.fail:
            return httpx.Response(500, text="nope")
        return httpx.Response(200, json={"ok": True})


def _burst(net, delay=0.01):
    http = httpx.AsyncClient(transport=httpx.MockTransport(net.handler))
    lb = LoadBalancedClient(["http://j0"], client=http)
    idx = lb.add_replicas(["http://c0j", "http://c1j"])          # sleeping judge replicas on the coder GPUs
    ctrl = BurstController(lb, idx, "http://proxy", ["http://c0", "http://c1"], http=http, delay_s=delay)
    return lb, idx, ctrl


def test_burst_swaps_in_the_judge_tail_and_back():
    net = FakeNet()
    lb, idx, ctrl = _burst(net)

    async def go():
        ctrl.batch_start(2, ["a", "b"])
        ca = ctrl.coder_begin("a")
        cb = ctrl.coder_begin("b")
        ctrl.coder_end(ca)
        ctrl.coder_end(ca)                           # a repeated end changes nothing
        await asyncio.sleep(0.05)
        assert ctrl.state == "coder"                 # b's coder call is still in flight
        ctrl.coder_end(cb)
        await asyncio.sleep(0.1)
        assert ctrl.state == "judge" and all(lb.active[i] for i in idx)
        assert ("POST", "http://proxy/park") in net.calls and ("POST", "http://c0j/wake_up") in net.calls
        assert await ctrl.ensure_coder("refine")
        assert ctrl.state == "coder" and not any(lb.active[i] for i in idx)
        assert net.calls[-1] == ("POST", "http://proxy/unpark")
    run(go())


def test_burst_waits_for_every_prompt_and_a_quiet_period():
    net = FakeNet()
    lb, idx, ctrl = _burst(net, delay=0.05)

    async def go():
        ctrl.batch_start(3, ["a", "b", "c"])
        ctrl.coder_end(ctrl.coder_begin("a"))
        ctrl.task_done("x")                          # not a prompt of this batch
        ctrl.coder_end(ctrl.coder_begin("b"))
        await asyncio.sleep(0.12)
        assert ctrl.state == "coder"                 # prompt c has not started coding
        ctrl.task_done("c")
        await asyncio.sleep(0.03)
        ctrl.task_done("a")                          # activity inside the quiet period delays the swap
        await asyncio.sleep(0.03)
        assert ctrl.state == "coder"
        await asyncio.sleep(0.1)
        assert ctrl.state == "judge"
        ctrl.batch_end()
        await asyncio.sleep(0.02)
        assert ctrl.state == "coder"                 # the batch end swaps back
    run(go())


def test_burst_undo_on_partial_failure():
    net = FakeNet(fail={"http://c1j/wake_up"})
    lb, idx, ctrl = _burst(net)

    async def go():
        assert not await ctrl.to_judge()
        assert ctrl.state == "coder" and not any(lb.active[i] for i in idx)
        posts = [u for m, u in net.calls]
        assert posts[-2:] == ["http://c0j/sleep", "http://proxy/unpark"]   # exactly what was done is undone
    run(go())


def test_spawner_allocation_and_commands():
    raw = {"llm_clients": {
        "coder": {"enabled": True, "base_url": "http://127.0.0.1:8001/v1",
                  "engine": {"model": "llama3-70b-fp8", "tensor_parallel_size": 2, "data_parallel_size": 2}},
        "judge": {"enabled": True, "base_url": "http://127.0.0.1:8002/v1", "engine": {"model": "llama3-8b", "gpu_ids": "7"}},
        "aux": {"enabled": True, "base_url": "http://127.0.0.1:8003/v1", "engine": {"model": "small-bf16"}},
        "remote": {"enabled": True, "base_url": "https://example.invalid/v1"}}}
    s = load_settings(raw=raw, env={})
    jobs = {j.name: j for j in build_jobs(s, all_gpus=[str(i) for i in range(8)])}
    assert jobs["judge"].gpu_ids == ["7"] and jobs["coder"].gpu_ids == ["0", "1", "2", "3"]
    assert jobs["aux"].gpu_ids == ["4", "5", "6"] and jobs["aux"].tp == 3 and "remote" not in jobs
    cmds = build_commands(jobs["coder"], python="py")
    assert len(cmds) == 3 and cmds[0]["env"]["CUDA_VISIBLE_DEVICES"] == "0,1" and cmds[1]["env"]["CUDA_VISIBLE_DEVICES"] == "2,3"
    assert "--nproc-per-node=2" in cmds[0]["cmd"] and cmds[0]["cmd"][cmds[0]["cmd"].index("--port") + 1] == "8101"
    assert cmds[0]["cmd"][cmds[0]["cmd"].index("--max-num-seqs") + 1] == "64"
    assert cmds[2]["cmd"][:3] == ["py", "-m", "phung5_b200.serve.router"] and cmds[2]["cmd"].count("--upstream") == 2
    assert build_commands(jobs["judge"], python="py")[0]["cmd"][:3] == ["py", "-m", "phung5_b200.serve.server"]
    with pytest.raises(ValueError):
        allocate_gpus({"a": s.llm_clients["judge"]}, ["0", "1"])          # GPU 7 is not visible
    raw["llm_clients"]["aux"]["engine"]["gpu_ids"] = "7"
    with pytest.raises(ValueError):
        build_jobs(load_settings(raw=raw, env={}), all_gpus=[str(i) for i in range(8)])  # reserved twice


class FakeNVML:
    def __init__(self, n=4, slow=(), throttled=()):
        self.n, self.slow, self.throttled = n, set(slow), set(throttled)

    def nvmlInit(self):
        pass

    def nvmlDeviceGetCount(self):
        return self.n

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetName(self, h):
        return b"NVIDIA B200"

    def nvmlDeviceGetEnforcedPowerLimit(self, h):
        return 1_000_000

    def nvmlDeviceGetPowerUsage(self, h):
        return 150_000

    def nvmlDeviceGetTemperature(self, h, kind):
        return 40 + h

    def nvmlDeviceGetClockInfo(self, h, kind):
        return 1965

    def nvmlDeviceGetMaxClockInfo(self, h, kind):
        return 1965

    def nvmlDeviceGetCurrentClocksEventReasons(self, h):
        return 0x40 if h in self.throttled else 0x4


def test_preflight_flags_outliers_thresholds_and_throttling():
    from phung5_b200.utils.preflight import NvmlReader
    nv = NvmlReader(FakeNVML(4, throttled={3}))

    def bench(i):
        return {"tflops": 1500.0 if i != 2 else 900.0, "copy_gbs": 6600.0, "stream48_gbs": 5000.0}
    res = run_preflight(nvml=nv, bench=bench, thresholds={"min_power_limit_w": 700})
    g = res["gpus"]
    assert not res["ok"] and res["diag"]["gpu_bad"] == 2 and res["diag"]["gpu_thr"] == 1
    assert any(f.startswith("tflops_outlier") for f in g[2]["flags"]) and "tflops<1000" in g[2]["flags"]
    assert g[3]["reasons"] == ["hw_thermal_slowdown"] and "throttled" in g[3]["flags"]
    assert g[0]["flags"] == [] and g[0]["reasons"] == ["sw_power_cap"] and res["diag"]["gpu_temp"] == 43
    ok = run_preflight(nvml=NvmlReader(FakeNVML(2)), bench=lambda i: {"tflops": 1500.0, "copy_gbs": 6600.0})
    assert ok["ok"] and ok["diag"]["tflops"] == [1500.0, 1500.0]


def test_worker_cpus_from_quota_and_topology(tmp_path):
    cg = tmp_path / "cg"
    cg.mkdir()
    (cg / "cpu.max").write_text("2400000 100000\n")          # 24 CPUs
    sysd = tmp_path / "sys"
    for c in range(32):                                        # 16 cores x 2 threads: c and c+16 are siblings
        d = sysd / f"cpu{c}" / "topology"
        d.mkdir(parents=True)
        d.joinpath("thread_siblings_list").write_text(f"{c % 16},{c % 16 + 16}\n")
    assert read_quota(str(cg)) == 24.0
    assert len(core_groups(list(range(32)), str(sysd))) == 16
    cpus = worker_cpus(reserve=14, min_cpus=8, cgroup_root=str(cg), allowed=list(range(32)), sys_root=str(sysd))
    assert cpus == list(range(6, 16))                          # 10 CPUs, one per core, highest cores first
    cpus = worker_cpus(reserve=4, min_cpus=8, cgroup_root=str(cg), allowed=list(range(32)), sys_root=str(sysd))
    assert len(cpus) == 20 and set(range(16)) <= set(cpus)     # all 16 cores, then 4 siblings
    assert worker_cpus(reserve=20, min_cpus=8, cgroup_root=str(cg), allowed=list(range(32)), sys_root=str(sysd)) is None
    (cg / "cpu.max").write_text("max 100000\n")
    assert read_quota(str(cg)) == math.inf
    assert worker_cpus(reserve=0, min_cpus=1, cgroup_root=str(cg), allowed=list(range(32)), sys_root=str(sysd)) is None


def test_checker_process_pool():
    from phung5_b200.app.jscheck import CheckerSettings, JSChecker
    from test_app_cpu import GOOD
    c = JSChecker(CheckerSettings(workers=2, processes=True))
    try:
        async def go():
            return await asyncio.gather(c.check_async(GOOD), c.check_async("export default 1"))
        good, bad = run(go())
        assert good.ok and good.scene["object"]["children"] and not bad.ok
        assert c.counts == {"checked": 2, "passed": 1}
    finally:
        c.close()


def test_pipeline_lends_coder_gpus_to_judge_replicas_in_the_judge_only_tail():
    """The burst controller wired into the service: a batch's judge-only tail parks the coder engines behind
    their proxy, wakes the judge replica and routes judge calls to it too; the batch end swaps back."""
    import asyncio
    import json as _json

    import httpx

    from phung5_b200.app.pipeline import GenerationPipeline
    from phung5_b200.app.session import BackendError
    from phung5_b200.app.state import MinerState, PipelineTask
    from phung5_b200.serve.router import LoadBalancedClient
    from test_app_cpu import StubLLM, _png, _settings

    stub = StubLLM()
    seen = []

    async def handler(req):
        host, path = req.url.host, req.url.path
        seen.append((host, path))
        if path == "/v1/chat/completions":
            await asyncio.sleep(0.02)
            return httpx.Response(200, json=await stub.chat(_json.loads(req.content)))
        if path == "/park_state":
            return httpx.Response(200, json={"active": ["http://c1"]})
        return httpx.Response(200, json={"ok": True})

    async def go():
        http = httpx.AsyncClient(transport=httpx.MockTransport(handler))
        s = _settings()
        s.burst.enabled, s.burst.proxy_url, s.burst.judge_replicas, s.burst.delay_s = True, "http://proxy", \
            ["http://jr1"], 0.01
        judge = LoadBalancedClient(["http://j0"], client=http, error=BackendError)
        pipe = GenerationPipeline(s, MinerState(), backends={"coder": stub, "judge": judge}, http=http)
        pipe.startup()
        tasks = [PipelineTask(stem=n, image_url=_png(), seed=10 + i) for i, n in enumerate(("chair", "lamp"))]
        await pipe.run_batch(tasks)
        await asyncio.sleep(0.05)                 # the batch end's swap back runs in the background
        pipe.close()
        return pipe
    pipe = asyncio.run(go())
    whats = [e["what"] for e in pipe.burst.events]
    assert "to_judge" in whats and whats.index("to_judge") < len(whats) - 1 and "to_coder" in whats
    assert ("proxy", "/park") in seen and ("jr1", "/wake_up") in seen
    assert ("jr1", "/sleep") in seen and ("proxy", "/unpark") in seen
    assert ("jr1", "/v1/chat/completions") in seen                 # the lent replica judged
    assert pipe.burst.state == "coder" and pipe.burst.parked == ["http://c1"]
    assert all(pipe.state.tasks[n].js_code for n in ("chair", "lamp"))


def test_two_judge_clients_share_load_with_per_task_affinity():
    import asyncio
    import json as _json

    import httpx

    from phung5_b200.app.pipeline import GenerationPipeline
    from phung5_b200.app.state import MinerState, PipelineTask
    from phung5_b200.serve.router import LoadBalancedClient
    from test_app_cpu import StubLLM, _png, _settings

    stub = StubLLM()
    hosts = []

    async def handler(req):
        hosts.append(req.url.host)
        if req.url.host == "j1" and len([h for h in hosts if h == "j1"]) == 1:
            # a context-length 400 comes back through the balancer as the session's BackendError: it retries
            # with a smaller max_tokens
            return httpx.Response(400, text="This model's maximum context length is 100000 tokens. However, you "
                                            "requested 100500 tokens (99000 in the messages, 1500 in the "
                                            "completion).")
        return httpx.Response(200, json=await stub.chat(_json.loads(req.content)))

    async def go():
        http = httpx.AsyncClient(transport=httpx.MockTransport(handler))
        s = _settings()
        s.llm_clients["judge"].base_url = "http://j0/v1"
        s.llm_clients["judge2"] = s.llm_clients["judge"].model_copy(update={"base_url": "http://j1/v1"})
        s.actors.judge.extra_clients = ["judge2"]
        pipe = GenerationPipeline(s, MinerState(), backends={"coder": stub}, http=http)
        pipe.startup()
        tasks = [PipelineTask(stem=n, image_url=_png(), seed=10 + i) for i, n in enumerate(("chair", "lamp"))]
        await pipe.run_batch(tasks)
        pipe.close()
        return pipe
    pipe = asyncio.run(go())
    lb = pipe.role_inner["judge"]
    assert isinstance(lb, LoadBalancedClient)
    assert sorted(lb.affinity) == ["chair", "lamp"] and sorted(lb.affinity.values()) == [0, 1]
    assert set(hosts) == {"j0", "j1"}
    assert all(pipe.state.tasks[n].js_code for n in ("chair", "lamp"))


def test_coder_probe_warm_burst_and_min_tps_replace_gate():
    import asyncio

    from phung5_b200.app.monitor import HealthWatcher
    from phung5_b200.app.pipeline import GenerationPipeline
    from phung5_b200.app.state import MinerState, MinerStatus
    from test_app_cpu import StubLLM, _settings

    class Slow(StubLLM):
        def __init__(self):
            super().__init__()
            self.n = 0

        async def chat(self, body):
            self.n += 1
            await asyncio.sleep(0.05 if self.n <= 4 else 0.01)       # the first burst pays the warm-up
            return {"choices": [{"message": {"role": "assistant", "content": "x"}, "finish_reason": "stop"}],
                    "usage": {"prompt_tokens": 5, "completion_tokens": 100}}

    s = _settings()
    s.pipeline.coder_probe.concurrency, s.pipeline.coder_probe.min_tps = 4, 1e9
    st = MinerState()
    pipe = GenerationPipeline(s, st, backends={"coder": Slow(), "judge": StubLLM()})
    pipe.startup()
    tps = asyncio.run(pipe.run_coder_probe())
    assert tps > 0 and int(st.diag["probe_tps"]) > st.diag["probe_tps_cold"] and st.diag["probe_errors"] == 0
    assert not pipe.probe_ok(tps) and pipe.probe_ok(None)
    pipe.close()

    async def on_ready():
        return False

    for remaining, want in ((1, MinerStatus.REPLACE), (0, MinerStatus.READY)):
        ms = MinerState()
        ms.replacements_remaining = remaining
        w = HealthWatcher(ms, {}, on_ready=on_ready)
        asyncio.run(w.tick())
        assert ms.status == want
