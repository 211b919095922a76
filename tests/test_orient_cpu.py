"""Orientation stage (app/orient.py) on CPU: the source rewrite turns the module's own output about world axes
and re-centres it, the decision table, and an end-to-end probe with the rasterizer's CPU restatement and an
embedder made of downsampled pixels: a model whose marked side faces right is turned to face front, and the
rewritten module still passes the checker."""
import asyncio
import math

import numpy as np
import pytest
import torch

from phung5_b200.app import jsvm
from phung5_b200.app.jscheck import JSChecker
from phung5_b200.app.orient import (OrientSettings, decide, orient_candidate, probe_rotations, rotate_source,
                                    rotated_scene, steps_matrix)

BOX = """export default function generate(THREE) {
  const g = new THREE.Group();
  const body = new THREE.Mesh(new THREE.BoxGeometry(0.6, 0.3, 0.15), new THREE.MeshStandardMaterial({ color: 0xdddddd }));
  g.add(body);
  const mark = new THREE.Mesh(new THREE.BoxGeometry(0.06, 0.24, 0.12), new THREE.MeshStandardMaterial({ color: 0xff0000 }));
  mark.position.set(0.33, 0, 0);         // on the +x side: seen by the right-hand camera
  g.add(mark);
  g.position.set(0.05, 0, 0);
  return g;
}
"""


def _bbox(src):
    r = jsvm.run_module(src)
    assert r.error is None, r.error
    return np.array(jsvm.world_bbox(r.root))


def test_rewrite_turns_and_recentres_the_module_output():
    lo, hi = _bbox(BOX)
    ext = hi - lo
    for steps in ([("y", "-Math.PI / 2")], [("y", "Math.PI / 2"), ("x", "Math.PI / 2")]):
        out = rotate_source(BOX, steps)
        assert out is not None and out.count("export default") == 1
        lo2, hi2 = _bbox(out)
        assert np.allclose((lo2 + hi2) / 2, 0, atol=1e-9)                      # re-centred
        want = np.abs(steps_matrix(steps)) @ ext                                # axis-aligned extents permute
        assert np.allclose(hi2 - lo2, want, atol=1e-9), (hi2 - lo2, want)


def test_rewrite_of_an_already_rotated_module_composes():
    """A module the per-draft stage turned can be turned again (the final draft's extra turns): the second
    block takes a fresh name and the two rotations compose."""
    once = rotate_source(BOX, [("y", "-Math.PI / 2")])
    twice = rotate_source(once, [("x", "Math.PI / 2")])
    assert twice is not None and "__oriented2" in twice
    lo, hi = _bbox(BOX)
    lo2, hi2 = _bbox(twice)
    want = np.abs(steps_matrix([("y", "-Math.PI / 2"), ("x", "Math.PI / 2")])) @ (hi - lo)
    assert np.allclose(hi2 - lo2, want, atol=1e-9) and np.allclose((lo2 + hi2) / 2, 0, atol=1e-9)


@pytest.mark.parametrize("form", [
    "export default (THREE) => { const g = new THREE.Group(); g.add(new THREE.Mesh(new THREE.BoxGeometry(1, 2, 3))); return g; };",
    "function generate(THREE) { const g = new THREE.Group(); g.add(new THREE.Mesh(new THREE.BoxGeometry(1, 2, 3))); return g; }\nexport default generate;",
    "export default function (THREE) { const g = new THREE.Group(); g.add(new THREE.Mesh(new THREE.BoxGeometry(1, 2, 3))); return g; }",
])
def test_rewrite_accepts_every_default_export_form(form):
    out = rotate_source(form, [("x", "Math.PI / 2")])
    assert out is not None
    lo, hi = _bbox(out)
    assert np.allclose(hi - lo, [1, 3, 2], atol=1e-9)


def test_rewrite_leaves_nested_helpers_alone():
    src = """export default function generate(THREE) {
  function part(w) { return new THREE.Mesh(new THREE.BoxGeometry(w, 2, 3)); }
  const make = (k) => { return part(k); };
  const g = new THREE.Group();
  if (g) { g.add(make(1)) }
  for (let i = 0; i < 1; i++) { g.add(part(1)); }
  return g
}"""
    out = rotate_source(src, [("x", "Math.PI / 2")])
    assert out is not None and out.count("rotateOnWorldAxis") == 1
    lo, hi = _bbox(out)
    assert np.allclose(hi - lo, [1, 3, 2], atol=1e-9)


def test_rewrite_refuses_what_it_cannot_edit():
    assert rotate_source("export default class A {}", [("y", "Math.PI")]) is None
    assert rotate_source("export default function a(T){return 1}\nexport default function b(T){return 2}",
                         [("y", "Math.PI")]) is None
    assert rotate_source(BOX, []) is None


def test_decision_table():
    assert decide({"front": 0.9, "right": 0.5, "back": 0.4, "left": 0.3}) == ("front", [])
    assert decide({"front": 0.5, "right": 0.4, "back": 0.9, "left": 0.3}) == ("back", [])
    assert decide({"front": 0.5, "right": 0.9, "back": 0.4, "left": 0.3}) == ("right", [("y", "-Math.PI / 2")])
    assert decide({"front": 0.5, "right": 0.3, "back": 0.4, "left": 0.9}) == ("left", [("y", "Math.PI / 2")])
    # a weak side lead is ignored when a margin is asked for
    assert decide({"front": 0.85, "right": 0.9, "back": 0.4, "left": 0.3}, min_side_margin=0.1) == ("right", [])
    tops = {k: 0.1 for k in probe_rotations() if k.startswith("top")}
    tops["top+1.57"] = 0.95
    best, steps = decide({"front": 0.5, "right": 0.3, "back": 0.4, "left": 0.2, **tops})
    assert best == "top" and steps == [("y", "Math.PI / 2"), ("x", "Math.PI / 2")]


class PixelEmbedder:
    """Downsampled RGB pixels as an L2-normalised vector: similar renders -> similar vectors."""
    disabled = False

    async def embed(self, imgs):
        v = []
        for im in imgs:
            x = im[..., :3].float().permute(2, 0, 1)[None] / 255.0
            x = torch.nn.functional.adaptive_avg_pool2d(x, 12).flatten()
            v.append((x - x.mean()).numpy())
        v = np.stack(v)
        return v / np.linalg.norm(v, axis=1, keepdims=True)

    @staticmethod
    def similarities(ref, vecs):
        return [float(x) for x in vecs @ ref]


class CpuRenderer:
    async def render(self, scene, views, size):
        from phung5_b200.render import scene as S
        tris, cols = S.scene_triangles(scene)
        tris = S.normalise(tris)
        return [S.render(tris, cols, S.view_projection(a, e), size) for a, e in views]


def test_probe_turns_a_sideways_model_to_face_front():
    try:
        from phung5_b200 import _C  # noqa: F401 - the rasterizer's CPU restatement lives in the extension
    except ImportError:
        pytest.skip("extension not built")
    chk = JSChecker()
    base = chk.check(BOX)
    assert base.ok, base.summary()
    emb, ren = PixelEmbedder(), CpuRenderer()

    async def go():
        # the reference photo: the marked (+x) side seen from the front
        ref_scene = rotated_scene(base.scene, steps_matrix([("y", "-Math.PI / 2")]))
        ref_vec = (await emb.embed(await ren.render(ref_scene, [(0.0, 10.0)], 160)))[0]
        code, scene, res = await orient_candidate(base.code, base.scene, renderer=ren, embedder=emb, ref_vec=ref_vec,
                                                  checker=chk, settings=OrientSettings(img_size=160))
        assert res.applied and res.best == "right", res
        assert res.sims["right"] > 0.99 > res.sims["front"]
        # the rewritten module, rendered from the front, now shows what the reference shows
        got = (await emb.embed(await ren.render(scene, [(0.0, 10.0)], 160)))[0]
        assert float(got @ ref_vec) > 0.99
        # an already-front model is left alone
        code2, _, res2 = await orient_candidate(code, scene, renderer=ren, embedder=emb, ref_vec=ref_vec, checker=chk)
        assert not res2.applied and res2.reason == "already_front" and code2 == code
    asyncio.run(go())
    chk.close()


class JudgeRenderer(CpuRenderer):
    """The judge's views: three front-family angles, white background (gray = white here)."""

    async def judge_views(self, scene, gray=True):
        views = await self.render(scene, [(0.0, 10.0), (35.0, 10.0), (-35.0, 10.0)], 96)
        return {"white": views, "gray": views}


class StubJudge:
    def __init__(self, winner, decided_by="S1"):
        self.winner, self.decided_by, self.calls = winner, decided_by, []

    async def duel(self, prompt_url, a, b, seed, ref_vec=None, early_stop=True):
        from phung5_b200.app.schemas import JudgeVerdict
        self.calls.append((a.stats.get("turn"), b.stats.get("turn")))
        return JudgeVerdict(winner=self.winner, decided_by=self.decided_by, confidence=0.9, detail={})


def test_final_turn_replaces_a_back_facing_final_only_on_a_decisive_duel():
    """The bracket's final shows its back to the camera (the photo shows its marked front): the y180 copy beats it
    on best-view similarity by far, duels the final from seat B, and is shipped only on a decisive win; a
    tie-break win, a margin gate above every gain, or a disabled stage keep the final."""
    try:
        from phung5_b200 import _C  # noqa: F401 - the rasterizer's CPU restatement lives in the extension
    except ImportError:
        pytest.skip("extension not built")
    from phung5_b200.app.jscheck import code_digest
    from phung5_b200.app.orient import FinalTurnSettings, turn_final
    from phung5_b200.app.state import Candidate
    chk = JSChecker()
    emb, ren = PixelEmbedder(), JudgeRenderer()

    async def go():
        photo = chk.check(BOX)                      # the photo's pose: the red mark on the +x side
        ref_vec = (await emb.embed((await ren.judge_views(photo.scene))["white"][:1]))[0]
        back = chk.check(rotate_source(BOX, [("y", "Math.PI")]))   # the final: turned by pi
        assert back.ok, back.summary()
        views = (await ren.judge_views(back.scene))["white"]
        final = Candidate(code=back.code, digest=code_digest(back.code), coder="c0", scene=back.scene, views=views,
                          gray_views=views, embed=await emb.embed(views), stats={"k": 3})
        st = FinalTurnSettings(enabled=True, turns=("y180", "xm90", "xp90"), min_margin=0.05)
        judge = StubJudge("B")
        out, res = await turn_final(final, renderer=ren, embedder=emb, ref_vec=ref_vec, checker=chk, judge=judge,
                                    prompt_url="p", seed=1, settings=st)
        assert res.replaced and res.picked == "y180" and out is not final, res
        assert res.tried["y180"] > 0.05 and judge.calls == [(None, "y180")]   # the final sat in seat A
        assert out.stats["turn"] == "y180" and out.stats["k"] == 3
        got = (await emb.embed(out.views[:1]))[0]
        assert float(got @ ref_vec) > float(np.asarray(final.embed)[0] @ ref_vec)
        # a win decided by the embedding tie-break is not decisive
        out2, res2 = await turn_final(final, renderer=ren, embedder=emb, ref_vec=ref_vec, checker=chk,
                                      judge=StubJudge("B", "S2 consensus -> embed tie-break"), prompt_url="p",
                                      seed=1, settings=st)
        assert out2 is final and res2.reason == "not_decisive"
        # both seats: the copy must also win from seat A
        out3, res3 = await turn_final(final, renderer=ren, embedder=emb, ref_vec=ref_vec, checker=chk,
                                      judge=StubJudge("B"), prompt_url="p", seed=1,
                                      settings=FinalTurnSettings(enabled=True, both_seats=True))
        assert out3 is final and res3.reason == "not_decisive"
        # no turned copy clears an unreachable margin; a disabled stage does nothing
        out4, res4 = await turn_final(final, renderer=ren, embedder=emb, ref_vec=ref_vec, checker=chk,
                                      judge=StubJudge("B"), prompt_url="p", seed=1,
                                      settings=FinalTurnSettings(enabled=True, min_margin=5.0))
        assert out4 is final and res4.reason == "no_contender" and set(res4.tried) == {"y180", "xm90", "xp90"}
        out5, res5 = await turn_final(final, renderer=ren, embedder=emb, ref_vec=ref_vec, checker=chk,
                                      judge=StubJudge("B"), prompt_url="p", seed=1, settings=FinalTurnSettings())
        assert out5 is final and res5.reason == "disabled"
    asyncio.run(go())
    chk.close()
