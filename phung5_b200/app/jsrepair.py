"""Failure-driven mechanical repairs of coder drafts, on the interpreter's token stream.

A draft that fails the checker for a mechanical reason costs a full LLM repair turn. The reference repairs a
few such classes deterministically (pipeline_service/modules/js_checker/mech_repair.py, off by default): the
failure text picks a class, the class rewrites the source, and the same checker runs again; the rewrite is
kept only if it passes. This module does the same for the failures this checker reports, with rewrites
planned on `jsvm.tokenize` tokens (so strings, comments and template text are never touched):

- `redeclared`  PARSE_ERROR "Identifier 'x' has already been declared": a later `let/const x = ...` in the same
                block becomes the assignment `x = ...` and the first declaration of x becomes `let`.
- `constlet`    EXECUTION_THREW "assignment to constant variable x": x's `const` declarations become `let`.
- `paren`       PARSE_ERROR "unexpected token ')'": the first `)` that closes nothing is deleted.
- `ident`       IDENTIFIER_NOT_ALLOWED `x`: if exactly one declared name equals x up to case and underscores
                (`roundedPts` / `rounded_pts`), every reference to x is renamed to it; if none does and x is only
                read as a value (never called, constructed, indexed or dereferenced), `let x = 0;` is declared at the
                top of generate().
- `console`     IDENTIFIER_NOT_ALLOWED `console` (not a global the specification allows): every `console.x(...);`
                statement is removed; a use of console anywhere but a statement of its own is not rewritten.
- `random`      FORBIDDEN_IDENTIFIER Math.random: every `Math.random` becomes a seeded generator defined at the top of
                the module (a 32-bit linear congruential generator), so the module is valid and deterministic.
- `texture`     TEXTURE_DATA_EXCEEDED "<b> bytes (limit <l>)" with b <= 4 l: every `new THREE.DataTexture(` goes
                through a helper that box-filters an RGBA Uint8Array texture of at least 256 x 256 texels (even sizes)
                down to half its width and height (a quarter of the bytes); other textures pass through unchanged.
- `retry`       TIMEOUT_EXCEEDED on the wall-clock deadline only (not the step budget): checked once more, since
                host load can push a module over the deadline.

Every class refuses (returns None) when its precondition is not met exactly; `plan` picks the classes the
failures call for, and the checker applies them for at most a few rounds.
"""
from __future__ import annotations

import re
from typing import Dict, Iterable, List, Optional, Set, Tuple

from . import jsvm

CLASSES = ("redeclared", "constlet", "paren", "ident", "console", "random", "texture", "retry")

SEEDED_RANDOM = ("const __phxRandom = (() => { let s = 0x2545F491; "
                 "return () => { s = (s * 1664525 + 1013904223) >>> 0; return s / 4294967296; }; })();\n")

HALF_TEXTURE = (
    "const __phxDataTexture = (THREE, data, w, h, ...rest) => {\n"
    "  if (data instanceof Uint8Array && w >= 256 && h >= 256 && w % 2 === 0 && h % 2 === 0 && data.length === w * h * 4) {\n"
    "    const w2 = w / 2, h2 = h / 2, out = new Uint8Array(w2 * h2 * 4);\n"
    "    for (let y = 0; y < h2; y++) {\n"
    "      for (let x = 0; x < w2; x++) {\n"
    "        const i = (2 * y * w + 2 * x) * 4, o = (y * w2 + x) * 4;\n"
    "        for (let c = 0; c < 4; c++) {\n"
    "          out[o + c] = (data[i + c] + data[i + 4 + c] + data[i + 4 * w + c] + data[i + 4 * w + 4 + c] + 2) >> 2;\n"
    "        }\n"
    "      }\n"
    "    }\n"
    "    return new THREE.DataTexture(out, w2, h2, ...rest);\n"
    "  }\n"
    "  return new THREE.DataTexture(data, w, h, ...rest);\n"
    "};\n")

def _half_texture_native(it):
    """What HALF_TEXTURE computes, for the interpreter: the same test, the same rounded 2 x 2 box mean per
    channel, the same constructor calls."""
    import numpy as np

    def call(i, this, x):
        three, data, w, h = (x + [jsvm.UNDEF] * 4)[:4]
        rest = list(x[4:])
        ctor = it.get(three, "DataTexture")
        wn = w if isinstance(w, float) else None
        hn = h if isinstance(h, float) else None
        if isinstance(data, jsvm.TypedArray) and data.kind == "Uint8Array" and wn is not None and hn is not None \
                and wn >= 256 and hn >= 256 and wn % 2 == 0 and hn % 2 == 0 and len(data.items) == wn * hn * 4:
            W, H = int(wn), int(hn)
            a = np.asarray(data.items, dtype=np.int64).reshape(H // 2, 2, W // 2, 2, 4)
            out = (a.sum(axis=(1, 3)) + 2) >> 2
            arr = jsvm.TypedArray("Uint8Array", out.reshape(-1).astype(np.float64).tolist(), coerced=True)
            return it.construct(ctor, [arr, float(W // 2), float(H // 2)] + rest)
        return it.construct(ctor, [data, w, h] + rest)
    return jsvm.Native("__phxDataTexture", fn=call)


jsvm.register_intrinsic("__phxDataTexture", HALF_TEXTURE, _half_texture_native)

_TEX = re.compile(r"^(\d+) bytes \(limit (\d+)\)")
_DUP = re.compile(r"Identifier '([A-Za-z_$][\w$]*)' has already been declared")
_CONST = re.compile(r"assignment to constant variable ([A-Za-z_$][\w$]*)")
_IDENT = re.compile(r"`([A-Za-z_$][\w$]*)` is not declared")


def plan(fails: Iterable[Dict[str, str]]) -> List[Tuple[str, str]]:
    """[(class, subject)] for the failures a mechanical class can address; [] when any failure is something
    no class handles (a partial repair cannot make the module pass)."""
    out: List[Tuple[str, str]] = []
    for f in fails:
        rule, detail = f.get("rule", ""), f.get("detail", "")
        if rule == "PARSE_ERROR" and _DUP.search(detail):
            out.append(("redeclared", _DUP.search(detail).group(1)))
        elif rule == "PARSE_ERROR" and "unexpected token ')'" in detail:
            out.append(("paren", ")"))
        elif rule == "EXECUTION_THREW" and _CONST.search(detail):
            out.append(("constlet", _CONST.search(detail).group(1)))
        elif rule == "IDENTIFIER_NOT_ALLOWED" and _IDENT.search(detail):
            name = _IDENT.search(detail).group(1)
            out.append(("console", name) if name == "console" else ("ident", name))
        elif rule == "FORBIDDEN_IDENTIFIER" and detail.startswith("Math.random"):
            out.append(("random", ""))
        elif rule == "TEXTURE_DATA_EXCEEDED" and _TEX.match(detail) and \
                int(_TEX.match(detail).group(1)) <= 4 * int(_TEX.match(detail).group(2)):
            out.append(("texture", ""))
        elif rule == "TIMEOUT_EXCEEDED" and "execution exceeded" in detail:
            out.append(("retry", ""))
        else:
            return []
    return out


def _edit(code: str, edits: List[Tuple[int, int, str]]) -> str:
    for a, b, s in sorted(edits, reverse=True):
        code = code[:a] + s + code[b:]
    return code


def _tokens(code: str) -> Optional[List[jsvm.Tok]]:
    try:
        return jsvm.tokenize(code)
    except jsvm.JSError:
        return None


def _tok_end(t: jsvm.Tok) -> int:
    return t.pos + len(str(t.val))


def _blocks(toks: List[jsvm.Tok]) -> List[int]:
    """Block id of every token: the index of the `{` that opened the innermost enclosing brace (-1 at top)."""
    out, stack = [], [-1]
    for i, t in enumerate(toks):
        if t.kind == "p" and t.val == "}" and len(stack) > 1:
            stack.pop()
        out.append(stack[-1])
        if t.kind == "p" and t.val == "{":
            stack.append(i)
    return out


def _is_binding_ref(toks: List[jsvm.Tok], i: int) -> bool:
    """Token i (an identifier) names a variable, not a property (`a.x`) or an object-literal key (`{x: 1}`)."""
    if i > 0 and toks[i - 1].kind == "p" and toks[i - 1].val in (".", "?."):
        return False
    if i + 1 < len(toks) and toks[i + 1].kind == "p" and toks[i + 1].val == ":" and i > 0 and \
            toks[i - 1].kind == "p" and toks[i - 1].val in ("{", ","):
        return False
    return True


def fix_redeclared(code: str, name: str) -> Optional[str]:
    toks = _tokens(code)
    if toks is None:
        return None
    blk = _blocks(toks)
    seen: Dict[int, int] = {}
    edits: List[Tuple[int, int, str]] = []
    for i in range(len(toks) - 2):
        t, n, eq = toks[i], toks[i + 1], toks[i + 2]
        if not (t.kind == "kw" and t.val in ("let", "const") and n.kind == "id" and n.val == name):
            continue
        if not (eq.kind == "p" and eq.val == "=") or (i > 0 and toks[i - 1].kind == "p" and toks[i - 1].val == "("):
            return None                               # destructuring, for-loop heads: not handled
        b = blk[i]
        if b not in seen:
            seen[b] = i
            if t.val == "const":
                edits.append((t.pos, _tok_end(t), "let"))
        else:
            edits.append((t.pos, n.pos, ""))          # `const x = v` -> `x = v`
    if not any(e[2] == "" for e in edits):
        return None
    return _edit(code, edits)


def fix_constlet(code: str, name: str) -> Optional[str]:
    toks = _tokens(code)
    if toks is None:
        return None
    edits = [(t.pos, _tok_end(t), "let") for i, t in enumerate(toks[:-1])
             if t.kind == "kw" and t.val == "const" and toks[i + 1].kind == "id" and toks[i + 1].val == name]
    return _edit(code, edits) if edits else None


def fix_paren(code: str) -> Optional[str]:
    toks = _tokens(code)
    if toks is None:
        return None
    depth = 0
    for t in toks:
        if t.kind != "p":
            continue
        if t.val == "(":
            depth += 1
        elif t.val == ")":
            if depth == 0:
                return code[:t.pos] + code[t.pos + 1:]
            depth -= 1
    return None


def fix_console(code: str) -> Optional[str]:
    toks = _tokens(code)
    if toks is None:
        return None
    edits: List[Tuple[int, int, str]] = []
    i = 0
    while i < len(toks):
        t = toks[i]
        if t.kind == "id" and t.val == "console":
            prev = toks[i - 1] if i > 0 else None
            ok_start = prev is None or (prev.kind == "p" and prev.val in (";", "{", "}"))
            if not (ok_start and i + 3 < len(toks) and toks[i + 1].val == "." and toks[i + 2].kind in ("id", "kw")
                    and toks[i + 3].kind == "p" and toks[i + 3].val == "("):
                return None
            depth, j = 0, i + 3
            while j < len(toks):
                if toks[j].kind == "p" and toks[j].val == "(":
                    depth += 1
                elif toks[j].kind == "p" and toks[j].val == ")":
                    depth -= 1
                    if depth == 0:
                        break
                j += 1
            if j >= len(toks):
                return None
            end = _tok_end(toks[j])
            if j + 1 < len(toks) and toks[j + 1].kind == "p" and toks[j + 1].val == ";":
                j += 1
                end = _tok_end(toks[j])
            elif j + 1 < len(toks) and not toks[j + 1].nl and not (toks[j + 1].kind == "p" and toks[j + 1].val == "}"):
                return None                                   # something follows on the same line
            edits.append((t.pos, end, ""))
            i = j + 1
            continue
        i += 1
    return _edit(code, edits) if edits else None


def fix_random(code: str) -> Optional[str]:
    toks = _tokens(code)
    if toks is None:
        return None
    edits = [(t.pos, _tok_end(toks[i + 2]), "__phxRandom") for i, t in enumerate(toks[:-2])
             if t.kind == "id" and t.val == "Math" and toks[i + 1].kind == "p" and toks[i + 1].val == "."
             and toks[i + 2].val == "random" and (i == 0 or toks[i - 1].val not in (".", "?."))]
    if not edits:
        return None
    return SEEDED_RANDOM + _edit(code, edits)


def fix_texture(code: str) -> Optional[str]:
    toks = _tokens(code)
    if toks is None:
        return None
    edits: List[Tuple[int, int, str]] = []
    for i in range(len(toks) - 4):
        a, b, c, d, e = toks[i:i + 5]
        if a.kind == "kw" and a.val == "new" and b.val == "THREE" and c.val == "." and d.val == "DataTexture" \
                and e.kind == "p" and e.val == "(":
            empty = i + 5 < len(toks) and toks[i + 5].kind == "p" and toks[i + 5].val == ")"
            edits.append((a.pos, _tok_end(e), "__phxDataTexture(THREE" + ("" if empty else ", ")))
    if not edits:
        return None
    return HALF_TEXTURE + _edit(code, edits)


def _generate_body(toks: List[jsvm.Tok]) -> Optional[int]:
    """Source offset just after the `{` that opens generate()'s body."""
    for i in range(len(toks) - 2):
        if toks[i].kind == "kw" and toks[i].val == "function" and toks[i + 1].val == "generate" and \
                toks[i + 2].val == "(":
            depth, j = 0, i + 2
            while j < len(toks):
                if toks[j].kind == "p" and toks[j].val == "(":
                    depth += 1
                elif toks[j].kind == "p" and toks[j].val == ")":
                    depth -= 1
                    if depth == 0:
                        break
                j += 1
            if j + 1 < len(toks) and toks[j + 1].kind == "p" and toks[j + 1].val == "{":
                return _tok_end(toks[j + 1])
    return None


def _stub_ident(code: str, name: str) -> Optional[str]:
    """`let name = 0;` at the top of generate() when name is only read as a plain value."""
    toks = _tokens(code)
    if toks is None:
        return None
    uses = [i for i, t in enumerate(toks) if t.kind == "id" and t.val == name and _is_binding_ref(toks, i)]
    if not uses:
        return None
    for i in uses:
        nxt = toks[i + 1] if i + 1 < len(toks) else None
        prev = toks[i - 1] if i > 0 else None
        if nxt is not None and nxt.kind == "p" and nxt.val in ("(", ".", "[", "?.", "`"):
            return None
        if prev is not None and prev.kind == "kw" and prev.val == "new":
            return None
    at = _generate_body(toks)
    if at is None:
        return None
    return code[:at] + f" let {name} = 0;" + code[at:]


def _norm(name: str) -> str:
    return name.replace("_", "").lower()


def fix_ident(code: str, name: str, declared: Set[str]) -> Optional[str]:
    same = [d for d in declared if d != name and _norm(d) == _norm(name)]
    if not same and name not in declared:
        return _stub_ident(code, name)
    if len(same) != 1:
        return None
    toks = _tokens(code)
    if toks is None:
        return None
    edits = [(t.pos, _tok_end(t), same[0]) for i, t in enumerate(toks)
             if t.kind == "id" and t.val == name and _is_binding_ref(toks, i)]
    return _edit(code, edits) if edits else None


def apply(code: str, steps: List[Tuple[str, str]], declared: Set[str]) -> Optional[Tuple[str, List[str]]]:
    """Apply every planned class -> (code, fixes), or None if one of them refuses."""
    fixes: List[str] = []
    for cls, subject in steps:
        if cls == "retry":
            fixes.append("retry after a wall-clock timeout")
            continue
        if cls == "redeclared":
            new = fix_redeclared(code, subject)
        elif cls == "constlet":
            new = fix_constlet(code, subject)
        elif cls == "paren":
            new = fix_paren(code)
        elif cls == "ident":
            new = fix_ident(code, subject, declared)
        elif cls == "console":
            new = fix_console(code)
        elif cls == "random":
            new = fix_random(code)
        elif cls == "texture":
            new = fix_texture(code)
        else:
            new = None
        if new is None:
            return None
        code = new
        fixes.append(f"{cls}: {subject}" if subject else cls)
    return code, fixes
