"""Orientation stage: turn a candidate so that the side matching the reference photo faces the judge's camera.

The judge compares candidates from front-family angles, so a model built sideways or lying down loses its duels
whatever its geometry is worth. Reference: `orient_task` (pipeline_service/pipeline/orientation.py:175), which
renders five low-resolution probe views (front, right, back, left, top-down), embeds them, and when a side or
the top matches the photo best writes a rotation into the candidate's own generate()
(`rotate_source`, pipeline_service/modules/js_checker/module.py:78 with rotate_runner.mjs), re-checks it and
keeps it only if the rewritten module still validates.

Here the probe is one batch of front renders of the candidate under each candidate rotation (rotating the model
by -90 deg about y shows from the front what the right-hand camera sees; a +90 deg tip about x brings the top
to the front, and four yaws before the tip cover the top's in-plane turn), rendered by the CUDA rasterizer (or
its CPU restatement) and embedded with the pipeline's embedder. Decision (same table as the reference):
  front or back best                -> unchanged
  right / left best                 -> yaw -pi/2 / +pi/2 about the world y axis (optionally only when the
                                       side beats both front and back by `min_side_margin`)
  top best                          -> the yaw (0, +-pi/2, pi) whose tipped front render matches best, then a
                                       +pi/2 tip about the world x axis
The rotation is written into the module's own default-exported function (found with the interpreter's
tokenizer): each of its value-returning `return` statements (not those of nested helpers) turns the returned
root with `rotateOnWorldAxis` per step, in order, and re-centres it on its bounding box -- so the submitted
code itself produces the oriented object, with THREE used only as `THREE.Member` (the checker's rule).
Every failure leaves the candidate untouched; a candidate is never dropped for failing to rotate.
"""
from __future__ import annotations

import math
import re
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

_AXES = {"x": (1.0, 0.0, 0.0), "y": (0.0, 1.0, 0.0), "z": (0.0, 0.0, 1.0)}
_ANGLE = {"0": 0.0, "Math.PI / 2": math.pi / 2, "-Math.PI / 2": -math.pi / 2, "Math.PI": math.pi}
PROBE_ELEVATION = 10.0
SIDE_STEP = {"right": ("y", "-Math.PI / 2"), "left": ("y", "Math.PI / 2")}
TIP_STEP = ("x", "Math.PI / 2")
TOP_YAWS = ("0", "Math.PI / 2", "Math.PI", "-Math.PI / 2")


@dataclass
class OrientSettings:
    enabled: bool = True
    img_size: int = 160
    min_side_margin: float = 0.0     # > 0: turn a side-best model only if sim(side) - max(front, back) >= it


@dataclass
class OrientResult:
    best: Optional[str] = None
    sims: Dict[str, float] = field(default_factory=dict)
    steps: List[Tuple[str, str]] = field(default_factory=list)
    applied: bool = False
    reason: str = ""


# ---------------------------------------------------------------------------------------------- rotations

def axis_rotation(axis: str, angle: float) -> np.ndarray:
    x, y, z = _AXES[axis]
    c, s = math.cos(angle), math.sin(angle)
    t = 1 - c
    return np.array([[t * x * x + c, t * x * y - s * z, t * x * z + s * y],
                     [t * x * y + s * z, t * y * y + c, t * y * z - s * x],
                     [t * x * z - s * y, t * y * z + s * x, t * z * z + c]])


def steps_matrix(steps: Sequence[Tuple[str, str]]) -> np.ndarray:
    """World-axis steps applied in order -> one rotation (later steps multiply on the left)."""
    r = np.eye(3)
    for axis, expr in steps:
        r = axis_rotation(axis, _ANGLE[expr]) @ r
    return r


def rotated_scene(scene: dict, r: np.ndarray) -> dict:
    """The scene with its root placed under a node carrying rotation r (column-major 4x4)."""
    m = np.eye(4)
    m[:3, :3] = r
    return {**scene, "object": {"uuid": "orient-root", "type": "Group", "matrix": m.T.reshape(-1).tolist(),
                                "children": [scene.get("object", {})]}}


def probe_rotations() -> Dict[str, List[Tuple[str, str]]]:
    """Probe name -> the steps whose front render shows what that probe looks at."""
    probes = {"front": [], "right": [SIDE_STEP["right"]], "back": [("y", "Math.PI")], "left": [SIDE_STEP["left"]]}
    for yaw in TOP_YAWS:
        probes[f"top{_ANGLE[yaw]:+.2f}"] = ([("y", yaw)] if yaw != "0" else []) + [TIP_STEP]
    return probes


def decide(sims: Dict[str, float], min_side_margin: float = 0.0) -> Tuple[Optional[str], List[Tuple[str, str]]]:
    """Probe similarities -> (best view, rotation steps); no steps when the model already faces front."""
    base = {k: v for k, v in sims.items() if k in ("front", "right", "back", "left")}
    tops = {k: v for k, v in sims.items() if k.startswith("top")}
    if tops:
        base["top"] = max(tops.values())
    if not base:
        return None, []
    best = max(base, key=base.get)
    if best in ("front", "back"):
        return best, []
    if best in SIDE_STEP:
        if min_side_margin > 0 and "front" in base and "back" in base:
            if base[best] - max(base["front"], base["back"]) < min_side_margin - 1e-9:
                return best, []
        return best, [SIDE_STEP[best]]
    top_key = max(tops, key=tops.get)
    return "top", probe_rotations()[top_key]


# ------------------------------------------------------------------------------------------ source rewrite

_BLOCK_KEYWORDS = {"if", "for", "while", "switch", "catch", "with"}


def _match(toks, i, open_, close):
    """Index of the token closing the bracket opened at toks[i]."""
    depth = 0
    for j in range(i, len(toks)):
        if toks[j].kind == "p" and toks[j].val == open_:
            depth += 1
        elif toks[j].kind == "p" and toks[j].val == close:
            depth -= 1
            if depth == 0:
                return j
    return -1


def _function_body(toks, k):
    """Given toks[k] = `function` (or the `(` of an arrow's parameters), -> (THREE parameter name, index of the
    body's `{`, index of its `}`) or None."""
    j = k + 1 if toks[k].kind == "kw" and toks[k].val == "function" else k
    if toks[j].kind == "id":
        j += 1                                        # function name
    if not (toks[j].kind == "p" and toks[j].val == "("):
        return None
    close = _match(toks, j, "(", ")")
    if close < 0 or close == j + 1 or toks[j + 1].kind != "id":
        return None
    three = toks[j + 1].val
    b = close + 1
    if toks[b].kind == "p" and toks[b].val == "=>":
        b += 1
    if not (toks[b].kind == "p" and toks[b].val == "{"):
        return None
    end = _match(toks, b, "{", "}")
    return (three, b, end) if end > 0 else None


def _default_function(toks):
    """The default-exported function of a module -> (THREE name, body `{` index, body `}` index) or None."""
    ex = [i for i in range(len(toks) - 1) if toks[i].kind == "kw" and toks[i].val == "export"
          and toks[i + 1].kind == "kw" and toks[i + 1].val == "default"]
    if len(ex) != 1:
        return None
    k = ex[0] + 2
    t = toks[k]
    if t.kind == "kw" and t.val == "function" or t.kind == "p" and t.val == "(":
        return _function_body(toks, k)
    if t.kind == "id":                                # `export default generate;` -> its declaration
        for i in range(len(toks) - 2):
            if toks[i].kind == "kw" and toks[i].val == "function" and toks[i + 1].kind == "id" \
                    and toks[i + 1].val == t.val:
                return _function_body(toks, i)
    return None


def _own_returns(toks, lo, hi):
    """`return` tokens inside toks[lo..hi] (a function body) that belong to that function, not to nested ones."""
    out, skip_until = [], -1
    for i in range(lo + 1, hi):
        if i <= skip_until:
            continue
        t = toks[i]
        if t.kind == "p" and t.val == "{" and i > 0:
            prev = toks[i - 1]
            nested = prev.kind == "p" and prev.val == "=>"
            if prev.kind == "p" and prev.val == ")":
                # `) {` opens a function body unless the parentheses belong to if/for/while/switch/catch
                depth, j = 0, i - 1
                while j > lo:
                    if toks[j].kind == "p" and toks[j].val == ")":
                        depth += 1
                    elif toks[j].kind == "p" and toks[j].val == "(":
                        depth -= 1
                        if depth == 0:
                            break
                    j -= 1
                nested = not (toks[j - 1].kind == "kw" and toks[j - 1].val in _BLOCK_KEYWORDS)
            if nested:
                skip_until = _match(toks, i, "{", "}")
                continue
        if t.kind == "kw" and t.val == "return":
            out.append(i)
    return out


def _return_end(toks, i, hi):
    """-> (index of the last token of the returned expression, index of its `;` or -1)."""
    depth = 0
    for j in range(i + 1, hi + 1):
        t = toks[j]
        if t.kind == "p" and t.val in "([{":
            depth += 1
        elif t.kind == "p" and t.val in ")]}":
            if depth == 0:
                return j - 1, -1
            depth -= 1
        elif depth == 0 and t.kind == "p" and t.val == ";":
            return j - 1, j
        elif depth == 0 and t.nl and j > i + 1 and t.kind in ("kw", "id") and \
                not (toks[j - 1].kind == "p" and toks[j - 1].val not in (")", "]", "}")):
            return j - 1, -1
    return -1, -1


def _token_end(src, toks, j):
    """Source offset just past token j."""
    return toks[j + 1].pos if j + 1 < len(toks) else len(src)


def rotate_source(code: str, steps: Sequence[Tuple[str, str]]) -> Optional[str]:
    """Write `steps` into the module's own default-exported function: every `return <root>` that belongs to it
    (not to nested helpers) becomes a block that turns the root about world axes in order with
    rotateOnWorldAxis and re-centres it on its bounding box. None when the module has no shape the rewrite
    understands (the caller keeps the original)."""
    if not code or not steps:
        return None
    try:
        from .jsvm import JSError, tokenize
        toks = tokenize(code)
    except Exception:  # noqa: BLE001 - unparsable modules are left alone
        return None
    fn = _default_function(toks)
    if fn is None:
        return None
    three, lo, hi = fn
    # a name the module does not use yet: a module rotated before (the final's own turn after the per-draft
    # stage) already holds `return <name>;` inside its block, and `const <name> = (<name>)` would not run
    var, n = "__oriented", 1
    while var in code:
        n += 1
        var = f"__oriented{n}"
    edits = []
    for r in _own_returns(toks, lo, hi):
        last, semi = _return_end(toks, r, hi)
        if last <= r:
            continue                                   # bare `return;`
        expr = code[toks[r + 1].pos:_token_end(code, toks, last)].rstrip()
        lines = [f"const {var} = ({expr});"]
        for axis, angle in steps:
            x, y, z = (int(c) for c in _AXES[axis])
            lines.append(f"{var}.rotateOnWorldAxis(new {three}.Vector3({x}, {y}, {z}), {angle});")
        lines.append(f"{var}.position.sub(new {three}.Box3().setFromObject({var})"
                     f".getCenter(new {three}.Vector3()));")
        lines.append(f"return {var};")
        end = _token_end(code, toks, semi if semi >= 0 else last)
        edits.append((toks[r].pos, end, "{ " + " ".join(lines) + " }"))
    if not edits:
        return None
    out = code
    for a, b, text in sorted(edits, reverse=True):
        out = out[:a] + text + out[b:]
    return out


# ----------------------------------------------------------------------------------------------- the stage

async def probe(scene: dict, renderer, embedder, ref_vec, size: int) -> Dict[str, float]:
    """Front renders of the scene under every probe rotation -> similarity of each to the reference."""
    names, scenes = [], []
    for name, steps in probe_rotations().items():
        names.append(name)
        scenes.append(rotated_scene(scene, steps_matrix(steps)))
    imgs = []
    for sc in scenes:
        imgs += await renderer.render(sc, views=[(0.0, PROBE_ELEVATION)], size=size)
    vecs = await embedder.embed(imgs)
    if vecs is None or ref_vec is None:
        return {}
    sims = embedder.similarities(ref_vec, vecs)
    return dict(zip(names, sims))


async def orient_candidate(code: str, scene: dict, *, renderer, embedder, ref_vec, checker,
                           settings: Optional[OrientSettings] = None):
    """-> (code, scene, OrientResult): the rotated module and its scene when a rotation was decided and the
    rewritten module validates, else the inputs unchanged."""
    st = settings or OrientSettings()
    res = OrientResult()
    if not st.enabled or embedder is None or ref_vec is None or getattr(embedder, "disabled", False):
        res.reason = "disabled"
        return code, scene, res
    try:
        res.sims = await probe(scene, renderer, embedder, ref_vec, st.img_size)
    except Exception as e:  # noqa: BLE001 - the probe is optional
        res.reason = f"probe_failed: {type(e).__name__}"
        return code, scene, res
    if not res.sims:
        res.reason = "probe_failed"
        return code, scene, res
    res.best, res.steps = decide(res.sims, st.min_side_margin)
    if not res.steps:
        res.reason = "already_front"
        return code, scene, res
    rotated = rotate_source(code, res.steps)
    if rotated is None:
        res.reason = "injection_failed"
        return code, scene, res
    chk = await checker.check_async(rotated)
    if not chk.ok:
        res.reason = "checker_rejected"
        return code, scene, res
    res.applied, res.reason = True, "applied"
    return chk.code, chk.scene, res


# ------------------------------------------------------------------------------------- the final draft's turns

# Extra turns tried on the bracket's final only (the per-draft probe never flips a model to its back or tilts its
# underside toward the camera): yaw by pi, tilt the underside (-y) toward the front camera, tilt the top toward it,
# and the yaw-then-tilt pair.
FINAL_TURNS: Dict[str, List[Tuple[str, str]]] = {
    "y180": [("y", "Math.PI")],
    "xm90": [("x", "-Math.PI / 2")],
    "xp90": [("x", "Math.PI / 2")],
    "y180xm90": [("y", "Math.PI"), ("x", "-Math.PI / 2")],
}


@dataclass
class FinalTurnSettings:
    enabled: bool = False            # off by default, as in the reference
    turns: Tuple[str, ...] = ("y180", "xm90", "xp90")
    min_margin: float = 0.05         # best-view similarity gain a turned copy needs over the final to be tried
    both_seats: bool = False         # also judge with the seats swapped; the turned copy must win both


@dataclass
class FinalTurnResult:
    tried: Dict[str, object] = field(default_factory=dict)    # turn -> similarity margin, or why it was skipped
    picked: Optional[str] = None
    replaced: bool = False
    reason: str = ""


def best_view_similarity(embed, n_views: int, ref_vec) -> Optional[float]:
    """Largest cosine similarity between the reference embedding and the candidate's judge views."""
    if embed is None or ref_vec is None or n_views == 0:
        return None
    return float(np.max(np.asarray(embed)[:n_views] @ np.asarray(ref_vec)))


def _decisive(verdict, seat: str) -> bool:
    """A win for `seat` that no tie-break decided (the judge's embedding tie-break settles draws)."""
    return verdict.winner == seat and "tie-break" not in verdict.decided_by


async def turn_final(final, *, renderer, embedder, ref_vec, checker, judge, prompt_url: str, seed: int,
                     settings: Optional[FinalTurnSettings] = None):
    """Turned copies of the final draft, each written into its own module by `rotate_source`, re-checked,
    rendered with the judge's views and embedded like any draft. A copy whose best-view similarity to the
    reference beats the final's by `min_margin` is a contender; the best contender duels the final (the final in
    seat A) and replaces it only on a decisive win. -> (candidate to ship, FinalTurnResult). Every failure keeps
    the final. Reference: pipeline_service/pipeline/orient_final.py (off by default there too)."""
    from .jscheck import code_digest
    from .state import Candidate
    st = settings or FinalTurnSettings()
    res = FinalTurnResult()
    if not st.enabled:
        res.reason = "disabled"
        return final, res
    base = best_view_similarity(final.embed, len(final.views), ref_vec)
    if base is None or embedder is None or judge is None:
        res.reason = "no_signal"
        return final, res
    best = None
    for name in st.turns:
        steps = FINAL_TURNS.get(name)
        if steps is None:
            res.tried[name] = "unknown_turn"
            continue
        try:
            code = rotate_source(final.code, steps)
            if code is None:
                res.tried[name] = "injection_failed"
                continue
            chk = await checker.check_async(code)
            if not chk.ok:
                res.tried[name] = "checker_rejected"
                continue
            views = await renderer.judge_views(chk.scene, gray=True)
            emb = await embedder.embed(views["white"])
            sim = best_view_similarity(emb, len(views["white"]), ref_vec)
        except Exception as e:  # noqa: BLE001 - a failed turn is skipped
            res.tried[name] = f"failed: {type(e).__name__}"
            continue
        if sim is None:
            res.tried[name] = "no_embedding"
            continue
        margin = sim - base
        res.tried[name] = round(margin, 4)
        if margin >= st.min_margin and (best is None or margin > best[0]):
            cand = Candidate(code=chk.code, digest=code_digest(chk.code), coder=final.coder, scene=chk.scene,
                             views=views["white"], gray_views=views.get("gray", []), embed=emb,
                             stats={**final.stats, "turn": name})
            best = (margin, name, cand)
    if best is None:
        res.reason = "no_contender"
        return final, res
    _, name, cand = best
    res.picked = name
    try:
        v = await judge.duel(prompt_url, final, cand, seed, ref_vec)
        won = _decisive(v, "B")
        if won and st.both_seats:
            v2 = await judge.duel(prompt_url, cand, final, seed, ref_vec)
            won = _decisive(v2, "A")
    except Exception as e:  # noqa: BLE001 - a failed duel keeps the final
        res.reason = f"duel_failed: {type(e).__name__}"
        return final, res
    if not won:
        res.reason = "not_decisive"
        return final, res
    res.replaced, res.reason = True, "replaced"
    return cand, res
