"""Context-aware repair of misnamed three.js constants in coder drafts.

Coder models often write enum constants that three.js does not have (`THREE.RepeatWrap`,
`THREE.LinearMipMapLinear`, `THREE.sRGBEncoding`, ...); the checker then rejects the whole draft with
UNKNOWN_THREE_API and the coder spends an LLM repair turn on a typo. The reference ships a repair for this
(pipeline_service/modules/js_checker/three_repair.py, off by default). This module is its counterpart on the
interpreter's token stream:

1. It acts only when every failure of a check is UNKNOWN_THREE_API (any other failure: no rewrite).
2. Every occurrence of an unknown `THREE.<X>` is classified by where it stands in the token stream:
   the value of an assignment or object-literal property (`tex.wrapS = ...`, `{ side: ... }`), an argument of
   `setUsage(...)`, or argument 4 / 5 of `new THREE.DataTexture(...)` selects an enum family (wrapping, filter,
   colour space, side, blending, format, type, usage); anything else leaves the family open.
   A constructor (`new THREE.X`), call (`THREE.X(`) or member chain (`THREE.X.y`) is never rewritten.
3. The replacement is the family member (or, with no family, any enum constant) whose CamelCase words best
   match X's: a word scores when it equals a candidate word, one is a prefix of the other (`Wrap` /
   `Wrapping`), or it is a known synonym (`Encoding` -> `ColorSpace`, `MipMap` -> `Mipmap`). Ties, and names
   sharing no word with any member, go to the family's three.js default. Without a family the match must
   cover most of both names' words.
4. If one occurrence has no acceptable replacement nothing is rewritten; the caller checks the rewritten
   module again and keeps it only if it passes, so a draft that already passes is never touched.
"""
from __future__ import annotations

import re
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

from . import jsvm

# Each family lists three.js's default value first: a name with no word in common with any member of its
# context's family becomes that default.
FAMILIES: Dict[str, Tuple[str, ...]] = {
    "wrap": ("ClampToEdgeWrapping", "RepeatWrapping", "MirroredRepeatWrapping"),
    "filter": ("LinearFilter", "NearestFilter", "LinearMipmapLinearFilter", "LinearMipmapNearestFilter",
               "NearestMipmapLinearFilter", "NearestMipmapNearestFilter"),
    "colorspace": ("NoColorSpace", "SRGBColorSpace", "LinearSRGBColorSpace"),
    "side": ("FrontSide", "DoubleSide", "BackSide"),
    "blending": ("NormalBlending", "AdditiveBlending", "SubtractiveBlending", "MultiplyBlending", "NoBlending"),
    "format": ("RGBAFormat", "RGBFormat", "RGFormat", "RedFormat", "AlphaFormat"),
    "type": ("UnsignedByteType", "FloatType", "HalfFloatType", "ByteType", "ShortType", "UnsignedShortType",
             "IntType", "UnsignedIntType"),
    "usage": ("StaticDrawUsage", "DynamicDrawUsage", "StreamDrawUsage"),
}
ALL_CONSTANTS: Tuple[str, ...] = tuple(c for fam in FAMILIES.values() for c in fam)

# property name (assignment target or object-literal key) -> family of its value
PROPERTY_FAMILY = {"wrapS": "wrap", "wrapT": "wrap", "wrapR": "wrap", "minFilter": "filter", "magFilter": "filter",
                   "colorSpace": "colorspace", "encoding": "colorspace", "side": "side", "shadowSide": "side",
                   "blending": "blending", "format": "format", "type": "type", "usage": "usage"}
# (callee, argument index) -> family
ARGUMENT_FAMILY = {("setUsage", 0): "usage", ("DataTexture", 3): "format", ("DataTexture", 4): "type",
                   ("DataTexture", 6): "wrap", ("DataTexture", 7): "wrap", ("DataTexture", 8): "filter",
                   ("DataTexture", 9): "filter"}
# word-level synonyms (lower case): writer's word -> the word three.js uses
SYNONYMS = {"mipmap": "mipmap", "mip": "mipmap", "encoding": "colorspace", "space": "colorspace",
            "srgb": "srgb", "linearencoding": "linear", "repeat": "repeat", "mirror": "mirrored",
            "mirrored": "mirrored", "clamp": "clamp", "edge": "edge", "uint8": "unsigned", "u8": "unsigned",
            "half": "half", "f16": "half", "float16": "half", "f32": "float", "float32": "float",
            "rgba8": "rgba", "both": "double", "two": "double", "additive": "additive", "add": "additive"}

_WORD = re.compile(r"[a-z][A-Z]+(?![a-z])|[A-Z]+(?![a-z])|[A-Z]?[a-z]+|\d+")


def words(name: str) -> List[str]:
    """CamelCase / snake_case words of a name, lower case, synonyms applied (`LinearMipMapLinear` ->
    [linear, mipmap, linear]); `Mip` + `Map` join into one word, as do `sRGB`-style acronyms; numbers are
    dropped (`RGBA8` -> [rgba])."""
    raw = [w.lower() for part in re.split(r"[_\W]+", name) for w in _WORD.findall(part)]
    out: List[str] = []
    for w in raw:
        if w == "map" and out and out[-1] in ("mip", "mipmap"):
            out[-1] = "mipmap"
            continue
        if w.isdigit():
            continue
        out.append(SYNONYMS.get(w, w))
    # "ColorSpace" is one concept
    joined: List[str] = []
    for w in out:
        if w == "colorspace" and joined and joined[-1] == "color":
            joined[-1] = "colorspace"
        elif w == "space" and joined and joined[-1] == "color":
            joined[-1] = "colorspace"
        else:
            joined.append(w)
    return joined


def _word_match(a: str, b: str) -> bool:
    return a == b or (len(a) >= 3 and len(b) >= 3 and (a.startswith(b) or b.startswith(a)))


def score(name: str, candidate: str) -> float:
    """Share of the two names' words that find a partner in the other (order-aware greedy pairing)."""
    wa, wb = words(name), words(candidate)
    if not wa or not wb:
        return 0.0
    used = [False] * len(wb)
    hit = 0
    for a in wa:
        for j, b in enumerate(wb):
            if not used[j] and _word_match(a, b):
                used[j] = True
                hit += 1
                break
    return 2.0 * hit / (len(wa) + len(wb))


def best_constant(name: str, family: Optional[str]) -> Optional[str]:
    """The replacement for an unknown constant `name`, or None if nothing fits well enough."""
    pool: Sequence[str] = FAMILIES[family] if family else ALL_CONSTANTS
    ranked = sorted(((score(name, c), -i, c) for i, c in enumerate(pool)), reverse=True)
    s, _, c = ranked[0]
    if family:
        return c if s > 0 else pool[0]           # no shared word: three.js's default for the property
    return c if s >= 0.6 else None


# ------------------------------------------------------------------------------------------------ token context

def _callee_and_index(toks: List[jsvm.Tok], i: int) -> Optional[Tuple[str, int]]:
    """For the token at i inside a call's parentheses: (callee name, argument index), else None."""
    depth, arg = 0, 0
    j = i - 1
    while j >= 0:
        t = toks[j]
        if t.kind == "p":
            if t.val in (")", "]", "}"):
                depth += 1
            elif t.val in ("(", "[", "{"):
                if depth == 0:
                    if t.val != "(" or j == 0 or toks[j - 1].kind != "id":
                        return None
                    return toks[j - 1].val, arg
                depth -= 1
            elif t.val == "," and depth == 0:
                arg += 1
            elif t.val == ";" and depth == 0:
                return None
        j -= 1
    return None


def _family_at(toks: List[jsvm.Tok], i: int) -> Optional[str]:
    """Enum family implied by the context of the `THREE` token at index i (i+2 is the constant's name)."""
    if i >= 2 and toks[i - 1].kind == "p" and toks[i - 1].val in ("=", ":") and toks[i - 2].kind in ("id", "str"):
        fam = PROPERTY_FAMILY.get(str(toks[i - 2].val))
        if fam:
            return fam
    ci = _callee_and_index(toks, i)
    if ci is not None:
        return ARGUMENT_FAMILY.get(ci)
    return None


def plan(fails: Iterable[Dict[str, str]]) -> Optional[List[str]]:
    """Unknown constant names to repair, or None when a failure is anything but UNKNOWN_THREE_API."""
    names: List[str] = []
    for f in fails:
        if f.get("rule") != "UNKNOWN_THREE_API":
            return None
        m = re.search(r"THREE\.(\w+)", f.get("detail", ""))
        if m is None:
            return None
        if m.group(1) not in names:
            names.append(m.group(1))
    return names or None


def rewrite(code: str, names: Sequence[str], three: str = "THREE") -> Optional[Tuple[str, List[str]]]:
    """Replace every `three.<name>` of `names` by its context's constant -> (code, fixes); None if an
    occurrence is a constructor, call or member chain, or has no acceptable replacement."""
    try:
        toks = jsvm.tokenize(code)
    except jsvm.JSError:
        return None
    wanted = set(names)
    edits: List[Tuple[int, int, str]] = []
    fixes: List[str] = []
    for i in range(len(toks) - 2):
        t, dot, nm = toks[i], toks[i + 1], toks[i + 2]
        if not (t.kind == "id" and t.val == three and dot.kind == "p" and dot.val == "." and nm.kind == "id"
                and nm.val in wanted):
            continue
        if i > 0 and toks[i - 1].kind == "kw" and toks[i - 1].val == "new":
            return None
        nxt = toks[i + 3] if i + 3 < len(toks) else None
        if nxt is not None and nxt.kind == "p" and nxt.val in ("(", ".", "["):
            return None
        fam = _family_at(toks, i)
        target = best_constant(nm.val, fam)
        if target is None:
            return None
        edits.append((nm.pos, nm.pos + len(nm.val), target))
        fix = f"THREE.{nm.val} -> THREE.{target}" + (f" ({fam})" if fam else "")
        if fix not in fixes:
            fixes.append(fix)
    if not edits:
        return None
    out = code
    for a, b, s in sorted(edits, reverse=True):
        if out[a:b] != code[a:b]:
            return None
        out = out[:a] + s + out[b:]
    return out, fixes
