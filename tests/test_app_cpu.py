"""Generation service on CPU: JS interpreter, checker, session layer, settings, K policies, bracket, HTTP API.

The model roles are served by a stub OpenAI-compatible backend: the coder answers with seed-dependent
three.js modules (some of them invalid, to exercise the repair turn), the judge prefers the model whose
front render has more object pixels, the critic returns a fixed report.
"""
import asyncio
import base64
import io
import json
import re
import time
import zipfile

import httpx
import numpy as np
import pytest
import torch

from phung5_b200.app import jsvm
from phung5_b200.app.batch_stats import BatchStats, parse_metrics
from phung5_b200.app.jscheck import JSChecker, code_digest, mechanical_repair
from phung5_b200.app.kpolicy import BudgetK, cpu_k
from phung5_b200.app.session import (BackendError, CallLog, ImageResendBackend, InstrumentedBackend, SessionAgent,
                                     Tool, async_retry)
from phung5_b200.app.settings import load_settings
from phung5_b200.app.stages import resolve_bracket, round_robin
from phung5_b200.app.state import Candidate, MinerState, MinerStatus, ServiceState


def run(coro):
    return asyncio.run(coro)


def js(src, **kw):
    r = jsvm.run_module("export default function generate(THREE) {" + src + "}", **kw)
    assert r.error is None, r.error
    return r.root


# ------------------------------------------------------------------------------------------------ interpreter


def test_jsvm_language_features():
    src = """
      const out = [];
      const add = (a, b = 2) => a + b;
      function fact(n) { return n <= 1 ? 1 : n * fact(n - 1); }
      const {x, y: [p, q], ...rest} = {x: 1, y: [2, 3], z: 4, w: 5};
      const arr = [1, 2, 3].map(v => v * 2).filter(v => v > 2);
      let s = 0;
      for (const [i, v] of arr.entries()) s += i * v;
      for (const k in {a: 1, b: 2}) out.push(k);
      let w = 0; while (w < 5) { w++; if (w === 3) continue; if (w > 4) break; }
      const counters = [];
      for (let i = 0; i < 3; i++) counters.push(() => i);
      let sw = '';
      switch (2) { case 1: sw = 'one'; break; case 2: sw = 'two'; case 3: sw += '+'; break; default: sw = 'd'; }
      let caught = '';
      try { null.foo; } catch (e) { caught = e.name; } finally { caught += '!'; }
      const tpl = `n=${arr.length} f=${fact(5)} ${[1, 2].join('-')}`;
      const g = new THREE.Group();
      g.name = JSON_LIKE = undefined;
      return g;
    """
    r = jsvm.run_module("export default function generate(THREE) {" + src + "}")
    assert r.error and "JSON_LIKE" in r.error      # undeclared assignment is a ReferenceError
    src = src.replace("g.name = JSON_LIKE = undefined;", """
      g.userData.r = [add(1), fact(5), x, p, q, Object.keys(rest).join(','), arr.join(','), s, out.join(''), w,
                      counters.map(f => f()).join(''), sw, caught, tpl, typeof add, 7 % 3, 2 ** 10, -7 >> 1,
                      [3, 1, 2].sort((a, b) => a - b).join(''), Math.max(...[4, 9, 2]), 0.1 + 0.2 === 0.3,
                      null ?? 'dflt', (0 || 'or'), [1, [2, [3]]].flat().length, 'abc'.toUpperCase(),
                      (12.345).toFixed(1), parseInt('0x1f'), Number.isInteger(5), [..."hi"].length];""")
    g = js(src)
    vals = g.props["userData"].props["r"].items
    assert vals == [3.0, 120.0, 1.0, 2.0, 3.0, "z,w", "4,6", 6.0, "ab", 5.0, "012", "two+", "TypeError!",
                    "n=2 f=120 1-2", "function", 1.0, 1024.0, -4.0, "123", 9.0, False, "dflt", "or", 3.0,
                    "ABC", "12.3", 31.0, True, 2.0]


def test_jsvm_three_model_and_serialization():
    g = js("""
      const g = new THREE.Group();
      const mat = new THREE.MeshStandardMaterial({ color: 0x336699 });
      const box = new THREE.Mesh(new THREE.BoxGeometry(2, 1, 1), mat);
      box.position.set(1, 0, 0); box.rotation.y = Math.PI / 2; box.scale.setScalar(2);
      g.add(box);
      const geo = new THREE.CylinderGeometry(0.5, 0.5, 2, 8); geo.translate(0, 1, 0);
      const c = new THREE.Mesh(geo, mat.clone()); c.material.color.set('#ff0000'); g.add(c);
      const inst = new THREE.InstancedMesh(new THREE.SphereGeometry(0.1, 8, 4), mat, 3);
      const d = new THREE.Object3D();
      for (let i = 0; i < 3; i++) { d.position.set(i, 0, 0); d.updateMatrix(); inst.setMatrixAt(i, d.matrix); }
      g.add(inst);
      const shape = new THREE.Shape(); shape.moveTo(0, 0); shape.lineTo(1, 0); shape.lineTo(1, 1); shape.lineTo(0, 1);
      g.add(new THREE.Mesh(new THREE.ExtrudeGeometry(shape, { depth: 0.2 }), mat));
      const pts = [new THREE.Vector2(0, 0), new THREE.Vector2(1, 0.5), new THREE.Vector2(0.2, 1)];
      g.add(new THREE.Mesh(new THREE.LatheGeometry(pts, 12), mat));
      const curve = new THREE.CatmullRomCurve3([new THREE.Vector3(0,0,0), new THREE.Vector3(1,1,0), new THREE.Vector3(2,0,0)]);
      g.add(new THREE.Mesh(new THREE.TubeGeometry(curve, 16, 0.1, 6), mat));
      return g;
    """)
    sc = jsvm.to_scene_json(g)
    assert {m["color"] for m in sc["materials"]} == {0x336699, 0xFF0000}
    # box: world transform = T(1,0,0) R_y(90) S(2): its local +x (width 2) maps to world -z, scaled by 2
    from phung5_b200.render import scene as S
    tris, cols = S.scene_triangles({"geometries": [sc["geometries"][0]], "materials": sc["materials"],
                                    "object": {"children": [sc["object"]["children"][0]]}})
    p = tris.reshape(-1, 3)
    lo, hi = p.min(0).values, p.max(0).values
    assert torch.allclose(hi - lo, torch.tensor([2.0, 2.0, 4.0]), atol=1e-4)
    assert torch.allclose((hi + lo) / 2, torch.tensor([1.0, 0.0, 0.0]), atol=1e-4)
    inst = sc["object"]["children"][2]
    assert len(inst["children"]) == 3 and inst["children"][2]["matrix"][12] == 2.0
    all_tris, _ = S.scene_triangles(sc)
    assert all_tris.shape[0] > 100 and bool(torch.isfinite(all_tris).all())


def test_jsvm_budgets_and_isolation():
    r = jsvm.run_module("export default function generate(THREE) { for(;;){} }", jsvm.Limits(steps=10_000))
    assert r.error.startswith("TIMEOUT")
    r = jsvm.run_module("export default function generate(THREE) { const a = []; a.length = 1e12; }")
    assert r.error.startswith(("TIMEOUT", "HEAP")) or "RangeError" in r.error
    r = jsvm.run_module("export default function generate(THREE) { return THREE.Mesh.__class__ }")
    assert r.error is None and r.root is jsvm.UNDEF      # host internals are not reachable
    r = jsvm.run_module("export default function generate(THREE) { function f(){ return f() } return f() }")
    assert r.error is not None
    r = jsvm.run_module("export default function generate(THREE) { throw new Error('boom') }")
    assert "boom" in r.error
    a = jsvm.run_module("export default function generate(THREE){ const g=new THREE.Group(); g.userData.r=Math.random(); return g }", seed=3)
    b = jsvm.run_module("export default function generate(THREE){ const g=new THREE.Group(); g.userData.r=Math.random(); return g }", seed=3)
    assert a.root.props["userData"].props["r"] == b.root.props["userData"].props["r"]


# ---------------------------------------------------------------------------------------------------- checker


GOOD = """export default function generate(THREE) {
  const g = new THREE.Group();
  const m = new THREE.MeshStandardMaterial({ color: 0xaa3311 });
  const seat = new THREE.Mesh(new THREE.BoxGeometry(1, 0.1, 1), m); seat.position.y = 0.3; g.add(seat);
  for (const [x, z] of [[-0.4, -0.4], [0.4, -0.4], [-0.4, 0.4], [0.4, 0.4]]) {
    const leg = new THREE.Mesh(new THREE.CylinderGeometry(0.05, 0.05, 0.3, 8), m);
    leg.position.set(x, 0.15, z); g.add(leg);
  }
  return g;
}"""


def test_checker_rules_limits_and_repair():
    c = JSChecker()
    r = c.check("```js\n" + GOOD + "\n```")
    assert r.ok and r.stats["drawCalls"] == 5 and r.scene["object"]["children"]
    fixed, fixes = mechanical_repair("import * as THREE from 'three';\nexport function generate(THREE) {\n"
                                     "  const l = new THREE.DirectionalLight(0xffffff, 1);\n  l.position.set(1, 1, 1);\n"
                                     "  const g = new THREE.Group(); g.add(l);\n"
                                     "  g.add(new THREE.Mesh(new THREE.BoxBufferGeometry(1,1,1)));\n  return g;\n}")
    assert c.check(fixed).ok, (fixed, c.check(fixed).failures)
    assert len(fixes) == 4
    rules = lambda src: {f["rule"] for f in c.check(src).failures}
    assert rules("const x = 1;") == {"MISSING_DEFAULT_EXPORT"}
    assert "FORBIDDEN_IDENTIFIER" in rules("export default function generate(THREE) { eval('1'); return new THREE.Group() }")
    assert "UNKNOWN_THREE_API" in rules("export default function generate(THREE) { return new THREE.Blob() }")
    assert "FORBIDDEN_THREE_API" in rules("export default function generate(THREE) { return new THREE.PerspectiveCamera() }")
    assert "COMPUTED_PROPERTY_ACCESS" in rules("export default function generate(THREE) { return new THREE['Group']() }")
    assert "FORBIDDEN_PROPERTY_ACCESS" in rules("export default function generate(THREE) { const g = new THREE.Group(); g.constructor; return g }")
    assert "LITERAL_BUDGET_EXCEEDED" in rules("export default function generate(THREE) { const s = '" + "a" * 60000 + "'; return new THREE.Group() }")
    assert "EXECUTION_THREW" in rules("export default function generate(THREE) { return undefinedThing.x }".replace(
        "undefinedThing", "(null)"))
    assert "EMPTY_SCENE" in rules("export default function generate(THREE) { return new THREE.Group() }")
    assert "PARSE_ERROR" in rules("export default function generate(THREE) { return (( }")
    assert code_digest(GOOD) == code_digest(GOOD.replace("\n", "\n   // comment\n"))


# ---------------------------------------------------------------------------------------------------- session


class ScriptBackend:
    def __init__(self, replies):
        self.replies = list(replies)
        self.bodies = []

    async def chat(self, body):
        self.bodies.append(json.loads(json.dumps(body)))
        r = self.replies.pop(0)
        if isinstance(r, Exception):
            raise r
        return r


def reply(content="", tool_calls=None, ptok=10, ctok=5):
    return {"choices": [{"message": {"role": "assistant", "content": content, "tool_calls": tool_calls}}],
            "usage": {"prompt_tokens": ptok, "completion_tokens": ctok}}


def test_session_tools_schema_retry_and_context_cap():
    from pydantic import BaseModel

    class Out(BaseModel):
        value: int

    be = ScriptBackend([
        reply(tool_calls=[{"id": "t1", "function": {"name": "double", "arguments": '{"x": 21}'}}]),
        reply("not json"),
        BackendError(400, "This model's maximum context length is 4096 tokens. However, you requested 5000 tokens "
                          "(3000 in the messages, 2000 in the completion)."),
        reply('```json\n{"value": 42}\n```'),
    ])
    agent = SessionAgent(be, "m", "sys", tools=[Tool("double", "x2", {"type": "object"}, lambda x: {"y": 2 * x})],
                         schema=Out, max_tokens=2000)
    r = run(agent.run("go", seed=5))
    assert r.parsed.value == 42 and r.turns == 3
    assert be.bodies[1]["messages"][-1]["role"] == "tool" and '"y": 42' in be.bodies[1]["messages"][-1]["content"]
    assert "schema" in be.bodies[2]["messages"][-1]["content"]
    assert be.bodies[3]["max_tokens"] == 4096 - 3000 - 16      # lowered to what the prompt leaves
    assert [b["seed"] for b in be.bodies] == [5, 6, 7, 7]


def test_retry_backoff_and_image_resend():
    n = {"k": 0}

    async def flaky():
        n["k"] += 1
        if n["k"] < 3:
            raise ConnectionError("reset")
        return "ok"
    assert run(async_retry(flaky, attempts=3, base_delay=0.001)) == "ok"

    async def slow():
        raise asyncio.TimeoutError()
    with pytest.raises(asyncio.TimeoutError):
        run(async_retry(slow, attempts=3, base_delay=0.001))

    img = "data:image/png;base64," + base64.b64encode(b"\x89PNG fake").decode()
    body = {"messages": [{"role": "user", "content": [{"type": "image_url", "image_url": {"url": img}},
                                                     {"type": "text", "text": "hi"}]}]}
    inner = ScriptBackend([reply("a"), reply("b"), BackendError(400, "unknown mm uuid"), reply("c")])
    log = CallLog()
    be = InstrumentedBackend(ImageResendBackend(inner), "judge", log)
    for _ in range(3):
        run(be.chat(body))
    sent = [b["messages"][0]["content"][0] for b in inner.bodies]
    assert sent[0]["image_url"]["url"] == img and sent[1]["image_url"] is None and sent[2]["image_url"] is None
    assert sent[3]["image_url"]["url"] == img           # resent in full after the 400
    assert log.summary()["judge"]["calls"] == 3 and log.summary()["judge"]["errors"] == 0


# ------------------------------------------------------------------------------------------ settings / policy


def test_settings_env_rewriters_and_validation():
    raw = {"llm_clients": {"a": {"base_url": "http://127.0.0.1:8001/v1"}, "b": {"base_url": "http://127.0.0.1:8002/v1"}},
           "actors": {"coder": {"client": "a"}}}
    s = load_settings(raw=raw, env={"PHX_K": "16", "PHX_MIX": "a:3,b:1", "PHX_GPU_SPLIT": "a=0,1;b=2",
                                    "PHX_SET": "pipeline.batch_time_budget=900;event_bus.max_iter=0"})
    assert s.actors.coder.ensemble_size == 16
    assert s.actors.coder.extra_clients == ["b"] and s.actors.coder.client_weights == [3, 1]
    assert s.llm_clients["a"].engine.gpu_ids == "0,1" and s.pipeline.batch_time_budget == 900
    assert s.event_bus.max_iter == 0 and len(s.notes) == 6
    with pytest.raises(Exception):
        load_settings(raw={"actors": {"coder": {"client": "missing"}}}, env={})
    s = load_settings(raw=raw, env={"PHX_K": "zero"})
    assert s.actors.coder.ensemble_size == 8 and s.notes[0].startswith("!!")


def test_k_policies():
    assert cpu_k(64, None) == 64 and cpu_k(64, 4.0) == 16 and cpu_k(64, 0.1) == 2
    bk = BudgetK(min_ref=4, floor=4)
    assert bk.decide(32, [1000]) == 32                  # no reference yet: fixed K
    for c in (1000, 2000, 4000, 8000):
        bk.observe(c)
    bk.batch_end()
    assert bk.initial(32) == 16
    k_short, k_long = bk.decide(32, [800, 900]), bk.decide(32, [9000, 9500])
    assert 16 <= k_long < 32 < k_short <= 48


def test_batch_stats_parsing_and_header():
    text = "# HELP x\nphx_generated_tokens_total{rank=\"0\"} 100\nphx_generated_tokens_total{rank=\"1\"} 50\n" \
           "phx_engine_steps_total 10\nother_metric 5\n"
    assert parse_metrics(text) == {"phx_generated_tokens_total": 150.0, "phx_engine_steps_total": 10.0}
    # label values may hold spaces, braces and escaped quotes; a timestamp may follow the value
    odd = 'phx_num_running{route="a b}c",q="x\\"y"} 3 1700000000\nphx_num_running 2\nphx_num_waiting{bad 1\n'
    assert parse_metrics(odd) == {"phx_num_running": 5.0}
    st = BatchStats(CallLog())
    st.engine_snapshot("vc", text)
    st.engine_snapshot("vc", text.replace("100", "400").replace("steps_total 10", "steps_total 40"))
    st.duel(2.0, 0.5)
    st.rendered(0.1, True)
    st.end()
    h = " ".join(st.header_parts())
    assert "duels=1/2.0/2.0/0.5" in h and "render=1/0" in h and "vc=300/30/0.00" in h


# ----------------------------------------------------------------------------------------------------- bracket


def _cand(k):
    return Candidate(code=f"c{k}", digest=f"d{k}", coder="c", scene={}, stats={"k": k})


def test_bracket_walkovers_duels_and_round_robin():
    async def go():
        loop = asyncio.get_running_loop()
        leaves = {}
        for k in range(8):
            f = loop.create_future()
            f.set_result(None if k in (1, 6) else _cand(k))
            leaves[k] = f
        duels = []

        async def duel(a, b, label):
            duels.append((a.stats["k"], b.stats["k"]))
            return a if a.stats["k"] > b.stats["k"] else b        # higher position wins
        w, semis = await resolve_bracket(leaves, duel, 8)
        assert w.stats["k"] == 7
        assert sorted(c.stats["k"] for c in semis) == [0, 3, 5, 7]   # 1 and 6 were walkovers
        assert len(duels) == 5                                    # 6 live leaves -> 5 duels
        rr = await round_robin(semis, duel, w)
        assert rr is w and w.rr_points == 3
    run(go())


# ------------------------------------------------------------------------------------------------ HTTP service


def _png(color=(200, 30, 30)):
    from PIL import Image
    im = Image.new("RGB", (64, 64), (255, 255, 255))
    for x in range(16, 48):
        for y in range(8, 56):
            im.putpixel((x, y), color)
    b = io.BytesIO()
    im.save(b, format="PNG")
    return "data:image/png;base64," + base64.b64encode(b.getvalue()).decode()


CODE_T = """export default function generate(THREE) {
  const g = new THREE.Group();
  const m = new THREE.MeshStandardMaterial({ color: 0x%06x });
  const body = new THREE.Mesh(new THREE.BoxGeometry(%s, %s, 0.5), m);
  g.add(body);
  g.scale.setScalar(1 / Math.max(%s, 1));        // fit the unit cube
  return g;
}"""


class StubLLM:
    """Coder: box sizes from the seed (seed % 5 == 0 -> invalid first reply); judge: prefers more object pixels."""

    def __init__(self):
        self.calls = {"coder": 0, "judge": 0, "critic": 0}
        self.mm_cache = {}          # the server-side multimodal cache that image uuids refer to

    def _url(self, part):
        if part.get("image_url"):
            url = part["image_url"]["url"]
            if part.get("uuid"):
                self.mm_cache[part["uuid"]] = url
            return url
        return self.mm_cache[part["uuid"]]

    @staticmethod
    def _object_pixels(url):
        from PIL import Image
        im = np.asarray(Image.open(io.BytesIO(base64.b64decode(url.split(",", 1)[1]))).convert("RGB")).astype(int)
        return int(((255 - im).sum(-1) > 30).sum())

    async def chat(self, body):
        await asyncio.sleep(0)
        system = body["messages"][0]["content"] if body["messages"][0]["role"] == "system" else ""
        last = body["messages"][-1]["content"]
        text = last if isinstance(last, str) else " ".join(p.get("text", "") for p in last if p.get("type") == "text")
        if "three.js module" in system or "ES module" in system:
            self.calls["coder"] += 1
            seed = body.get("seed", 0)
            if seed % 5 == 0 and "failed validation" not in text:
                return reply("```js\nexport default function generate(THREE) { return new THREE.Group() }\n```")
            w = 0.4 + (seed % 7) * 0.2
            return reply("```js\n" + CODE_T % (0x10 * (seed % 13) + 0x204060, w, 1.0, w) + "\n```", ctok=120)
        if "review a 3D model" in system:
            self.calls["critic"] += 1
            return reply(json.dumps({"issues": [{"kind": "wrong_size", "description": "too small", "severity": 8}],
                                     "scores": {"shape": 6, "color": 7}, "summary": "ok"}))
        self.calls["judge"] += 1
        imgs = [self._url(p) for m in body["messages"] if isinstance(m["content"], list)
                for p in m["content"] if p.get("type") == "image_url"]
        a, b = (self._object_pixels(u) for u in imgs[1:3])
        pa, pb = (3.0, 6.0) if a > b else ((6.0, 3.0) if b > a else (5.0, 5.0))
        if '"penalty_a"' in text and "best-matching" not in text:
            return reply(json.dumps({"penalty_a": pa, "penalty_b": pb, "reason": "size"}))
        if "best-matching" in text:
            return reply(json.dumps({"best_view_a": 0, "best_view_b": 0, "penalty_a": pa, "penalty_b": pb}))
        if "artifacts_a" in text:
            return reply(json.dumps({"artifacts_a": 1, "artifacts_b": 1}))
        if "features" in text:
            return reply(json.dumps({"features": ["a", "b", "c", "d"], "has_a": [True] * 4, "has_b": [True] * 4}))
        return reply(json.dumps({"choice": "draw"}))


def _settings(**pipeline):
    raw = {"llm_clients": {"coder": {"base_url": "http://127.0.0.1:9/v1"}, "judge": {"base_url": "http://127.0.0.1:9/v1"}},
           "actors": {"coder": {"client": "coder", "ensemble_size": 6, "workers": 4},
                      "judge": {"client": "judge", "workers": 4}, "renderer": {"workers": 2}},
           "pipeline": {"batch_time_budget": 300, "batch_margin_s": 10, **pipeline},
           "embedder": {"enabled": False}, "warmup": False}
    return load_settings(raw=raw, env={})


def test_service_end_to_end_with_stub_models():
    from fastapi.testclient import TestClient

    from phung5_b200.app.serve import build_app
    stub = StubLLM()
    app = build_app(_settings(), backends={"coder": stub, "judge": stub}, watch=False,
                    preflight={"gpus": 1, "tflops": [1500.0]})
    with TestClient(app) as cl:
        assert cl.get("/health").status_code == 200
        assert cl.get("/status").json()["status"] == "ready"
        assert cl.get("/results").status_code == 409
        prompts = [{"stem": "chair", "image_url": _png()}, {"stem": "lamp", "image_url": _png((20, 20, 200))}]
        r = cl.post("/generate", json={"prompts": prompts, "seed": 10})
        assert r.json() == {"accepted": 2}
        assert cl.post("/generate", json={"prompts": prompts[::-1], "seed": 10}).json() == {"accepted": 2}
        for _ in range(600):
            st = cl.get("/status").json()
            if st["status"] == "complete":
                break
            time.sleep(0.05)
        assert st["status"] == "complete" and st["progress"] == 2 and st["total"] == 2
        z = zipfile.ZipFile(io.BytesIO(cl.get("/results").content))
        assert sorted(z.namelist()) == ["chair.js", "lamp.js"]
        code = z.read("chair.js").decode()
        assert code.startswith("// miner-diag: gpus=1 tflops=1500 ") and "seed=10" in code.splitlines()[0]
        assert "duels=" in code.splitlines()[0]
        assert JSChecker().check(code.split("\n", 1)[1]).ok
        t = cl.get("/debug/tasks/chair").json()
        assert t["status"] == "completed" and t["duels"] >= 1 and t["valid"] >= 4 and t["generated"] == 6
        # views are normalised to the largest extent, so a (w x 1) box covers min(w, 1/w) of the frame: the
        # judge (more object pixels wins) must pick the candidate closest to square
        widths = [0.4 + ((10 + k) % 7) * 0.2 for k in range(6)]
        w = float(re.search(r"BoxGeometry\(([\d.]+)", code).group(1))
        assert w == pytest.approx(max(widths, key=lambda x: min(x, 1 / x)))
        assert cl.get("/debug/tasks/nope").status_code == 404
        assert cl.get("/debug/tasks").json()["completed"]
        assert "lines" in cl.get("/debug/logs").json()
        stats = cl.get("/debug/stats").json()
        assert stats["renderer"]["renders"] >= 8 and stats["checker"]["passed"] >= 8
    assert stub.calls["judge"] > 0


def test_service_state_machine_and_warmup(monkeypatch):
    from fastapi.testclient import TestClient

    from phung5_b200.app.serve import build_app
    st = MinerState()
    st.set_llm_status("a", ServiceState.RUNNING)
    assert st.models_ready()
    st.set_llm_status("b", ServiceState.DOWN)
    assert not st.models_ready() and st.any_down()

    s = _settings()
    s.llm_clients["coder"].enabled = True
    app = build_app(s, backends={"coder": StubLLM(), "judge": StubLLM()}, watch=False)
    with TestClient(app) as cl:
        r = cl.post("/generate", json={"prompts": [{"stem": "a", "image_url": _png()}]})
        assert r.status_code == 503                                   # warming up: engines not probed yet
        miner = app.state.miner
        miner.status = MinerStatus.REPLACE
        assert cl.get("/status", params={"replacements_remaining": 2}).json()["status"] == "replace"
        assert cl.post("/generate", json={"prompts": [{"stem": "a", "image_url": _png()}]}).status_code == 409
        assert cl.get("/status", params={"replacements_remaining": 0}).json()["status"] == "warming_up"


def test_health_watcher_transitions():
    from phung5_b200.app.monitor import HealthWatcher

    class FakeProber:
        def __init__(self, seq):
            self.seq, self.state, self.last_error = list(seq), ServiceState.STARTING, ""

        async def probe(self):
            self.state = self.seq.pop(0) if len(self.seq) > 1 else self.seq[0]
            return self.state

    st = MinerState()
    ready = []

    async def on_ready():
        ready.append(1)
    w = HealthWatcher(st, {"coder": FakeProber([ServiceState.STARTING, ServiceState.RUNNING, ServiceState.RUNNING,
                                                ServiceState.DOWN])}, on_ready=on_ready)

    async def go():
        await w.tick()
        assert st.status == MinerStatus.WARMING_UP
        await w.tick()
        assert st.status == MinerStatus.READY and ready == [1]
        st.replacements_remaining = 1
        await w.tick()
        assert st.status == MinerStatus.READY
        await w.tick()
        assert st.status == MinerStatus.REPLACE
    run(go())


def test_round_robin_eight_reuses_bracket_verdicts_and_records_shadow_picks():
    from phung5_b200.app.stages import multigen_first_iter
    from phung5_b200.app.state import PipelineTask

    class Factory:
        async def build(self, i):
            return _cand(i)

    calls = []

    async def raw(a, b, label):
        calls.append((a.stats["k"], b.stats["k"], label))
        # a non-transitive preference: higher k wins except 7 always loses to 2
        if {a.stats["k"], b.stats["k"]} == {2, 7}:
            return a if a.stats["k"] == 2 else b
        return a if a.stats["k"] > b.stats["k"] else b

    cache = {}

    async def duel(a, b, label):          # the pair cache of make_duel
        key = tuple(sorted((a.digest, b.digest)))
        if key not in cache:
            cache[key] = await raw(a, b, label)
        return cache[key]

    task = PipelineTask(stem="s", image_url="x")
    w = run(multigen_first_iter(task, Factory(), duel, 16, round_robin_size=8, shadow=["rr4"], shadow_max_duels=12))
    assert task.shadow["shipped"] == w.stats["k"]
    assert task.shadow["rr4"] is not None
    pairs = {tuple(sorted(c[:2])) for c in calls}
    assert len(pairs) == len(calls)                  # no pair was judged twice
