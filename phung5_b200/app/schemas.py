"""Request/response models of the generation service and the JSON reply schemas of its model roles.

HTTP models match the reference's wire format (pipeline_service/schemas/requests.py, responses.py):
`POST /generate {"prompts": [{"stem", "image_url"}], "seed": 42}` -> `{"accepted": n}`, and
`GET /status` -> `{"status", "progress", "total", "payload"}`.

Role schemas: the critic's issue report (reference modules/critic/schema.py:9-95, issue kinds with alias
coercion), the planner's object structure description (modules/scene_planner/schema.py:6-82), the pairwise
verdict (modules/judge/schema.py) and the per-stage duel replies used by `agents.JudgeAgent`.
"""
from __future__ import annotations

from enum import Enum
from typing import Any, Dict, List, Literal, Optional

from pydantic import BaseModel, Field, field_validator

# ------------------------------------------------------------------------------------------------------ HTTP


class PromptItem(BaseModel):
    stem: str
    image_url: str


class GenerateRequest(BaseModel):
    prompts: List[PromptItem]
    seed: int = 42


class StatusResponse(BaseModel):
    status: str
    progress: int
    total: int
    payload: Any = None


class GenerateAccepted(BaseModel):
    accepted: int


# ---------------------------------------------------------------------------------------------------- critic


class IssueKind(str, Enum):
    wrong_proportion = "wrong_proportion"
    missing_part = "missing_part"
    extra_part = "extra_part"
    wrong_count = "wrong_count"
    wrong_position = "wrong_position"
    wrong_material = "wrong_material"
    wrong_color = "wrong_color"
    wrong_orientation = "wrong_orientation"


_KIND_WORDS = {"missing": IssueKind.missing_part, "extra": IssueKind.extra_part, "count": IssueKind.wrong_count,
               "number": IssueKind.wrong_count, "position": IssueKind.wrong_position,
               "placement": IssueKind.wrong_position, "location": IssueKind.wrong_position,
               "layout": IssueKind.wrong_position, "material": IssueKind.wrong_material,
               "texture": IssueKind.wrong_material, "finish": IssueKind.wrong_material,
               "surface": IssueKind.wrong_material, "color": IssueKind.wrong_color, "colour": IssueKind.wrong_color,
               "orientation": IssueKind.wrong_orientation, "rotation": IssueKind.wrong_orientation,
               "angle": IssueKind.wrong_orientation}


def coerce_issue_kind(v: Any) -> Any:
    """Map the model's free-form kind ("missing_detail", "wrong-size", "Wrong Texture") onto IssueKind:
    exact names first, then the first keyword of the name, else proportion/shape."""
    if isinstance(v, IssueKind) or not isinstance(v, str):
        return v
    key = v.strip().lower().replace("-", "_").replace(" ", "_")
    if key in IssueKind.__members__:
        return IssueKind(key)
    for word in key.split("_"):
        if word in _KIND_WORDS:
            return _KIND_WORDS[word]
    return IssueKind.wrong_proportion


class Severity(str, Enum):
    low = "low"
    medium = "medium"
    high = "high"


class Issue(BaseModel):
    kind: IssueKind
    target: Optional[str] = None
    description: str = ""
    severity: Severity = Severity.medium

    @field_validator("kind", mode="before")
    @classmethod
    def _kind(cls, v):
        return coerce_issue_kind(v)

    @field_validator("severity", mode="before")
    @classmethod
    def _sev(cls, v):
        if isinstance(v, str) and v.strip().lower() in Severity.__members__:
            return Severity(v.strip().lower())
        if isinstance(v, (int, float)):
            return Severity.high if v >= 7 else (Severity.medium if v >= 4 else Severity.low)
        return Severity.medium


class CriticReport(BaseModel):
    issues: List[Issue] = Field(default_factory=list)
    scores: Dict[str, float] = Field(default_factory=dict)   # e.g. shape, proportion, color, detail (0-10)
    summary: str = ""

    def score(self) -> float:
        return sum(self.scores.values()) / len(self.scores) if self.scores else 0.0

    def worst(self, n: int = 5) -> List[Issue]:
        order = {Severity.high: 0, Severity.medium: 1, Severity.low: 2}
        return sorted(self.issues, key=lambda i: order[i.severity])[:n]


# --------------------------------------------------------------------------------------------------- planner


class PartSpec(BaseModel):
    name: str
    shape: str = ""
    color: str = ""
    count: int = 1
    relation: str = ""


class ObjectPlan(BaseModel):
    """Object structure description: what the coder should build, part by part."""
    object: str
    parts: List[PartSpec] = Field(default_factory=list)
    proportions: str = ""
    notes: str = ""

    def render(self) -> str:
        lines = [f"Object: {self.object}"]
        for p in self.parts:
            lines.append(f"- {p.name} x{p.count}: {p.shape} {p.color} {p.relation}".rstrip())
        if self.proportions:
            lines.append(f"Proportions: {self.proportions}")
        if self.notes:
            lines.append(f"Notes: {self.notes}")
        return "\n".join(lines)


# ----------------------------------------------------------------------------------------------------- judge


def _ab(v):
    if isinstance(v, str):
        s = v.strip().upper()
        if s in ("A", "B", "LEFT", "RIGHT", "1", "2", "DRAW", "TIE", "EQUAL", "NONE"):
            return {"LEFT": "A", "1": "A", "RIGHT": "B", "2": "B", "TIE": "draw", "EQUAL": "draw", "NONE": "draw",
                    "DRAW": "draw"}.get(s, s)
    return v


class AnglePenalty(BaseModel):
    """Stage 1: penalties (0 = perfect match to the prompt image, 10 = unrelated) of both candidates at one view."""
    penalty_a: float = Field(ge=0, le=10)
    penalty_b: float = Field(ge=0, le=10)
    reason: str = ""


class BestViewReply(BaseModel):
    """Stage 2 best-view: each candidate's penalty judged at its own best-matching view."""
    best_view_a: int = 0
    best_view_b: int = 0
    penalty_a: float = Field(ge=0, le=10)
    penalty_b: float = Field(ge=0, le=10)


class ArtifactReply(BaseModel):
    """Stage 2 artifacts: penalties for broken geometry (floating parts, interpenetration, holes, noise)."""
    artifacts_a: float = Field(ge=0, le=10)
    artifacts_b: float = Field(ge=0, le=10)


class ChecklistReply(BaseModel):
    """Stage 2 checklist: which prompt features each candidate has (the model lists the features)."""
    features: List[str] = Field(default_factory=list)
    has_a: List[bool] = Field(default_factory=list)
    has_b: List[bool] = Field(default_factory=list)


class PreferenceReply(BaseModel):
    """Stage 3 (gray rescue) and stage 4 (side guard): a direct preference."""
    choice: Literal["A", "B", "draw"]
    reason: str = ""

    @field_validator("choice", mode="before")
    @classmethod
    def _c(cls, v):
        return _ab(v)


class JudgeVerdict(BaseModel):
    winner: Literal["A", "B", "draw"]
    reason: str = ""
    confidence: float = Field(default=0.5, ge=0.0, le=1.0)
    decided_by: str = ""
    detail: Dict[str, Any] = Field(default_factory=dict)

    @field_validator("winner", mode="before")
    @classmethod
    def _w(cls, v):
        return _ab(v)
