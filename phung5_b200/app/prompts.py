"""Prompt texts of the model roles (coder, repair, critic, planner, judge stages).

The reference ships several coder prompt variants selected by an environment switch
(pipeline_service/modules/scene_coder/coder_prompt.py:31-61, prompts.py, few_shot_examples.py,
threejs_reference.py). The texts below are this framework's own; they describe the module contract that
`jscheck.JSChecker` enforces (default-exported `generate(THREE)`, the THREE subset, the limits).
"""
from __future__ import annotations

from .jscheck import LIMITS, THREE_ALLOWED

_ALLOWED = ", ".join(sorted(n for n in THREE_ALLOWED if n[0].isupper() and not n.endswith("Side")))

CODER_SYSTEM = f"""You write a single JavaScript ES module that builds a 3D model of the object in the user's image
with three.js. Contract:
- `export default function generate(THREE) {{ ... return root; }}` is the only export; `THREE` is passed in,
  never imported. `root` is a THREE.Group (or Mesh) centred near the origin, +Y up, the object's front facing +Z,
  and the whole model fits inside the cube [-0.5, 0.5] on every axis (scale it to fit).
- Use only these THREE members: {_ALLOWED}, plus MathUtils and the side/colour-space constants.
- No lights, cameras, renderers, loaders, textures from URLs, timers, console, Math.random (write a small seeded
  generator if you need variation), async code or imports. Helper functions that need THREE take it as a
  parameter named THREE.
- Budget: at most {LIMITS['vertices']} vertices, {LIMITS['drawCalls']} meshes, nesting depth {LIMITS['depth']}.
- Model the silhouette first (proportions, part count, placement), then colour and materials, then details.
Reply with the module in one ```js fenced block and nothing else."""

CODER_USER = """Build the object shown in this image as a three.js module following the contract."""

CODER_USER_WITH_PLAN = """Build the object shown in this image as a three.js module following the contract.
A structural description of the object to follow:
{plan}"""

REPAIR_USER = """The module failed validation:
{failures}
Fix these problems and reply with the complete corrected module in one ```js block."""

REFINE_USER = """A reviewer compared renders of your module with the image and found these issues:
{issues}
Revise the module to fix them without breaking what already matches. Reply with the complete module in one
```js block."""

CRITIC_SYSTEM = """You review a 3D model against the image it should reproduce. The first image is the target; the
second is a 2x2 grid of renders of the model from four directions around it. Report concrete, fixable issues.
Reply with JSON only:
{"issues": [{"kind": one of wrong_proportion|missing_part|extra_part|wrong_count|wrong_position|wrong_material|
wrong_color|wrong_orientation, "target": "<part>", "description": "<what to change>", "severity": low|medium|high}],
 "scores": {"shape": 0-10, "proportion": 0-10, "color": 0-10, "detail": 0-10}, "summary": "<one sentence>"}"""

PLANNER_SYSTEM = """Describe the structure of the object in the image so that a programmer can model it from simple
solids. Reply with JSON only: {"object": "<name>", "parts": [{"name", "shape", "color", "count", "relation"}],
"proportions": "<overall width:height:depth and key ratios>", "notes": "<anything unusual>"}"""

JUDGE_SYSTEM = """You compare two 3D models (A and B) with a target image. Judge only how well each model's shape,
proportions, part structure and colours match the object in the target image. Ignore rendering style,
lighting and background. Reply with JSON only."""

S1_USER = """Target image first, then model A and model B seen {angle}.
Give each model a penalty from 0 (matches the target) to 10 (unrelated):
{{"penalty_a": <0-10>, "penalty_b": <0-10>, "reason": "<short>"}}"""

S2_BEST_VIEW_USER = """Target image first, then model A at its best-matching view, then model B at its best-matching view.
Give each a penalty from 0 (matches) to 10 (unrelated):
{{"best_view_a": 0, "best_view_b": 0, "penalty_a": <0-10>, "penalty_b": <0-10>}}"""

S2_ARTIFACT_USER = """Target image first, then model A and model B from the front. Penalise broken geometry only:
floating or detached parts, parts intersecting wrongly, holes, noisy or degenerate shapes (0 = clean, 10 = broken).
{{"artifacts_a": <0-10>, "artifacts_b": <0-10>}}"""

S2_CHECKLIST_USER = """Target image first, then model A and model B from the front. List {lo} to {hi} visual features
that define the target object, then say for each whether A and B have it.
{{"features": ["..."], "has_a": [true|false, ...], "has_b": [true|false, ...]}}"""

S3_GRAY_USER = """The two models are shown on a gray background so that pale parts are visible. Target image first, then
model A, then model B. Which model matches the target better?
{{"choice": "A" | "B" | "draw", "reason": "<short>"}}"""

S4_SIDE_USER = """Target image first, then model A and model B seen {angle}. Which model has the more plausible
3D shape for the target object from this side?
{{"choice": "A" | "B" | "draw", "reason": "<short>"}}"""
