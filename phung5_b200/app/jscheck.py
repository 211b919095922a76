"""Candidate checker: mechanical repair -> static analysis -> sandboxed execution -> post-validation -> scene JSON.

The reference runs three Node programs for this (pipeline_service/modules/js_checker/module.py:46-240 drives
validator/{parse,staticAnalysis,execute,postValidation}.js and serialize_runner.mjs; repairs in
mech_repair.py and three_repair.py). Here the same stages run in-process on the JavaScript interpreter of
`jsvm.py`, whose AST the static rules walk directly.

Failures are reported as {"stage", "rule", "detail"} records. Rule codes keep the reference's names
(MISSING_DEFAULT_EXPORT, FORBIDDEN_IDENTIFIER, UNKNOWN_THREE_API, VERTEX_LIMIT_EXCEEDED, ...) because the
coder's repair prompt quotes them back to the model. Limits follow the reference's post-validation
(validator/postValidation.js:11-17): 250k vertices, 200 draw calls, depth 32, 50k instances, 4 MiB of
texture data; execution gets 5 s in V8 (execute.js:46), here a step budget plus a scaled wall-clock budget.
"""
from __future__ import annotations

import asyncio
import difflib
import hashlib
import math
import re
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from typing import Any, Dict, Iterable, List, Optional, Set

from . import jsrepair, jsvm, threefix, threespec

LIMITS = {"vertices": 250_000, "drawCalls": 200, "depth": 32, "instances": 50_000, "textureBytes": 4 * 1_048_576}
MAX_FILE_BYTES = 1_048_576          # source size (UTF-8)
BOUND = 0.5                         # the model must fit inside [-0.5, 0.5] on every axis
BOUND_TOL = 1e-6                    # float32 vertex storage vs the validator's doubles
LITERAL_BUDGET = 50 * 1024
ROOT_TYPES = {"Group", "Mesh", "LineSegments", "Points"}      # the returned object's type (a bare one is wrapped)
DRAW_TYPES = {"Mesh", "InstancedMesh", "Line", "LineSegments", "LineLoop", "Points"}   # isMesh / isLine / isPoints
# material slots whose DataTexture counts toward the texture-data limit
MAP_PROPS = ("map", "normalMap", "roughnessMap", "metalnessMap", "aoMap", "emissiveMap", "displacementMap", "bumpMap",
             "alphaMap", "envMap", "lightMap", "specularIntensityMap", "specularColorMap", "sheenRoughnessMap",
             "sheenColorMap", "transmissionMap", "thicknessMap", "clearcoatMap", "clearcoatNormalMap",
             "clearcoatRoughnessMap", "iridescenceMap", "iridescenceThicknessMap", "anisotropyMap")

# the output specification's tables (app/threespec.py); `arguments` is a function's implicit binding
ALLOWED_ROOTS = set(threespec.ALLOWED_ROOT_IDENTIFIERS) | {"arguments"}
FORBIDDEN_IDENTIFIERS = set(threespec.FORBIDDEN_IDENTIFIERS)
FORBIDDEN_PROPERTIES = set(threespec.FORBIDDEN_PROPERTY_NAMES)
COMPUTED_ACCESS_GATED = set(threespec.COMPUTED_ACCESS_GATED)
THREE_DISALLOWED_KNOWN = set(threespec.THREE_DISALLOWED_KNOWN)
THREE_BLOCKED_SUBMEMBERS = {k: set(v) for k, v in threespec.THREE_BLOCKED_SUBMEMBERS.items()}
THREE_ALLOWED = set(threespec.THREE_ALLOWED)


@dataclass
class CheckResult:
    ok: bool
    failures: List[Dict[str, str]] = field(default_factory=list)
    code: str = ""
    scene: Optional[dict] = None
    stats: Dict[str, Any] = field(default_factory=dict)
    repaired: List[str] = field(default_factory=list)

    @property
    def digest(self) -> str:
        return code_digest(self.code)

    def summary(self) -> str:
        return "; ".join(f"{f['rule']}: {f['detail']}" for f in self.failures[:6])


def code_digest(code: str) -> str:
    """Whitespace/comment-insensitive digest: candidates that differ only in formatting dedupe together."""
    s = re.sub(r"//[^\n]*|/\*.*?\*/", "", code, flags=re.S)
    s = re.sub(r"\s+", " ", s).strip()
    return hashlib.sha1(s.encode()).hexdigest()[:16]


# ------------------------------------------------------------------------------------------ mechanical repair

_FENCE = re.compile(r"```(?:javascript|js|typescript|ts)?\s*\n(.*?)```", re.S | re.I)


def extract_code(text: str) -> str:
    """The module inside a model reply: the longest fenced block, else the text itself."""
    blocks = _FENCE.findall(text or "")
    if blocks:
        with_export = [b for b in blocks if "export" in b]
        return max(with_export or blocks, key=len).strip()
    return (text or "").strip()


def mechanical_repair(code: str) -> tuple:
    """Fix the common, meaning-preserving mistakes of model-written modules. -> (code, [fixes])."""
    fixes = []
    c = code
    new = re.sub(r"^\s*import\s+[^;\n]*?from\s+['\"][^'\"]+['\"]\s*;?\s*$", "", c, flags=re.M)
    if new != c:
        fixes.append("removed import statements")
        c = new
    if not re.search(r"\bexport\s+default\b", c):
        m = re.search(r"\bexport\s+function\s+(\w+)", c)
        if m:
            c = c[:m.start()] + "export default function " + m.group(1) + c[m.end():]
            fixes.append("export function -> export default function")
        elif re.search(r"^\s*function\s+generate\s*\(", c, flags=re.M):
            c = re.sub(r"^(\s*)function\s+generate\s*\(", r"\1export default function generate(", c, count=1, flags=re.M)
            fixes.append("added export default to generate")
    new = re.sub(r"\bexport\s+default\s+async\s+function", "export default function", c)
    if new != c:
        fixes.append("removed async from generate")
        c = new
    # three.js r125 removed the *BufferGeometry aliases
    new = re.sub(r"\bTHREE\.(\w+)BufferGeometry\b", r"THREE.\1Geometry", c)
    new = new.replace("THREE.Geometry(", "THREE.BufferGeometry(")
    if new != c:
        fixes.append("XBufferGeometry -> XGeometry")
        c = new
    names = set(re.findall(r"\bTHREE\.([A-Za-z_]\w*)", c))
    for nm in sorted(names):
        if nm in THREE_ALLOWED or nm in THREE_DISALLOWED_KNOWN:
            continue
        close = difflib.get_close_matches(nm, sorted(THREE_ALLOWED), n=1, cutoff=0.85)
        if close:
            c = re.sub(rf"\bTHREE\.{nm}\b", f"THREE.{close[0]}", c)
            fixes.append(f"THREE.{nm} -> THREE.{close[0]}")
    # lights are the renderer's job: drop their declarations, statements on them and their .add() calls
    light_re = r"(?:AmbientLight|DirectionalLight|PointLight|SpotLight|HemisphereLight|RectAreaLight)"
    light_vars = re.findall(rf"(?:const|let|var)\s+(\w+)\s*=\s*new\s+THREE\.{light_re}\b", c)
    if light_vars:
        for v in light_vars:
            c = re.sub(rf"(?:const|let|var)\s+{v}\s*=\s*new\s+THREE\.{light_re}\b[^;\n]*;?", "", c)
            c = re.sub(rf"(?<![\w.$]){v}\.[^;\n]*;", "", c)
            c = re.sub(rf"[\w$.]+\.add\(\s*{v}\s*\)\s*;?", "", c)
            c = re.sub(rf"(\.add\([^)]*?),\s*{v}\b", r"\1", c)
            c = re.sub(rf"(\.add\(\s*){v}\s*,\s*", r"\1", c)
        fixes.append(f"removed lights {sorted(set(light_vars))}")
    return c, fixes


# ------------------------------------------------------------------------------------------- static analysis


def _walk(node, fn):
    """Depth-first over the AST (tagged tuples, plus untagged tuples/lists of them); fn(node) returning False
    stops the descent."""
    if isinstance(node, tuple) and node and isinstance(node[0], str):
        if fn(node) is False:
            return
        if node[0] == "objpat":       # entries are (key, target, default) with a plain-string key
            for key, target, default in node[1]:
                if isinstance(key, tuple):
                    _walk(key, fn)
                _walk(target, fn)
                _walk(default, fn)
            return
        for ch in node[1:]:
            _walk(ch, fn)
    elif isinstance(node, (tuple, list)):
        for ch in node:
            _walk(ch, fn)


def _declared_names(prog) -> Set[str]:
    names: Set[str] = set()

    def visit(n):
        tag = n[0]
        if tag in ("id",):
            names.add(n[1])
        elif tag in ("fundecl", "classdecl"):
            names.add(n[1])
        elif tag == "class" and n[1]:
            names.add(n[1])
        elif tag == "func":
            if n[1]:
                names.add(n[1] if isinstance(n[1], str) else "")
        elif tag == "objpat" and n[2]:
            names.add(n[2])
        return True
    _walk(prog, visit)
    return names


def _default_function(body):
    default = [s for s in body if s[0] == "export_default"]
    if not default:
        return None
    fn = default[0][1]
    if fn[0] == "ident":
        target = next((s[2] for s in body if s[0] == "fundecl" and s[1] == fn[1]), None)
        fn = target if target is not None else fn
    return fn if fn[0] == "func" else None


def three_param(prog) -> Optional[str]:
    """Name of the default-exported function's first parameter (the THREE namespace), if it has one."""
    fn = _default_function(prog[1])
    if fn is None:
        return None
    params = fn[2]
    return params[0][0][1] if params and params[0][0][0] == "id" else None


def _bound_names(p) -> List[str]:
    """Names a binding pattern declares: ("id", x), ("objpat", props, rest), ("arrpat", elems, rest)."""
    if not isinstance(p, tuple) or not p:
        return []
    if p[0] == "id":
        return [p[1]]
    if p[0] == "objpat":
        return [n for _, target, _ in p[1] for n in _bound_names(target)] + ([p[2]] if p[2] else [])
    if p[0] == "arrpat":
        return [n for target, _ in p[1] for n in _bound_names(target)] + _bound_names(p[2])
    return []


def _scope_clash(stmts, params: Iterable[str] = (), function_top: bool = False) -> Optional[str]:
    """First name declared twice in one statement list where ES modules (strict code) reject it: a let/const
    (or, outside a function's top level, function) name declared again by any declaration of the list, or
    equal to a parameter of the function whose body the list is."""
    lexical: Set[str] = set()
    other: Set[str] = set(params)
    for st in stmts:
        if not isinstance(st, tuple) or not st:
            continue
        if st[0] == "export_decl":
            st = st[1]
        if st[0] == "export_named":
            st = ("fundecl", st[2])
        if st[0] == "decl":
            names, var_like = [n for tgt, _ in st[2] for n in _bound_names(tgt)], st[1] == "var"
        elif st[0] == "fundecl":
            names, var_like = [st[1]], function_top
        elif st[0] == "classdecl":
            names, var_like = [st[1]], False
        else:
            continue
        for n in names:
            if n in lexical or (not var_like and n in other):
                return n
            (other if var_like else lexical).add(n)
    return None


def redeclared_name(prog) -> Optional[str]:
    """A name declared twice in one scope (a parse-time error for a JS engine), or None."""
    def visit(n) -> Optional[str]:
        if isinstance(n, list):
            for ch in n:
                r = visit(ch)
                if r:
                    return r
            return None
        if not isinstance(n, tuple) or not n:
            return None
        tag = n[0]
        if tag == "func":
            ps, rest, body = n[2], n[3], n[4]
            pnames = [x for tgt, _ in ps for x in _bound_names(tgt)] + _bound_names(rest)
            r = _scope_clash(body[1], pnames, True)
            if r:
                return r
            return visit([d for _, d in ps]) or visit(body[1])
        if tag == "block":
            r = _scope_clash(n[1])
            if r:
                return r
        if tag == "switch":
            r = _scope_clash([st for _, body in n[2] for st in body])
            if r:
                return r
        return visit(list(n[1:]))
    r = _scope_clash(prog[1])
    return r or visit(prog[1])


def _ctor_params(cls_node):
    for kind, _static, _key, fn in cls_node[3]:
        if kind == "ctor":
            return fn[2]
    return []


def _function_params(prog) -> Dict[str, list]:
    """name -> parameter list of the module's named functions and classes (declarations, and const / let / var
    bindings of function or class expressions); scopes are not distinguished."""
    out: Dict[str, list] = {}

    def visit(n):
        tag = n[0]
        if tag == "fundecl":
            out[n[1]] = n[2][2]
        elif tag == "classdecl":
            out[n[1]] = _ctor_params(n[2])
        elif tag == "decl":
            for target, init in n[2]:
                if target[0] == "id" and isinstance(init, tuple) and init:
                    if init[0] == "func":
                        out[target[1]] = init[2]
                    elif init[0] == "class":
                        out[target[1]] = _ctor_params(init)
        return True
    _walk(prog, visit)
    return out


def static_analyze(prog) -> List[Dict[str, str]]:
    fails: List[Dict[str, str]] = []

    def fail(rule, detail):
        fails.append({"stage": "static_analysis", "rule": rule, "detail": detail})

    body = prog[1]
    exports = [s for s in body if s[0] in ("export_default", "export_named", "export_decl")]
    default = [s for s in exports if s[0] == "export_default"]
    if not default:
        fail("MISSING_DEFAULT_EXPORT", "no `export default` found")
        return fails
    if len(exports) > 1:
        fail("MULTIPLE_TOP_LEVEL_EXPORTS", f"found {len(exports)} top-level exports, expected exactly 1")
    fn = _default_function(body)
    if fn is None:
        fail("DEFAULT_EXPORT_NOT_FUNCTION", "default export must be a function generate(THREE)")
        return fails
    three = three_param(prog)
    if three is None:
        fail("MISSING_THREE_PARAM", "generate must take THREE as its first parameter")
    declared = _declared_names(prog)
    literal_bytes = [0]
    seen_forbidden: Set[str] = set()
    # THREE flows only into member access, destructuring of allowed members, and helpers whose parameter is
    # named THREE (or destructures allowed members); `THREE` as a parameter name of such a helper counts too
    three_names = {n for n in (three, "THREE") if n is not None and (n == three or n in declared)}
    funcs = _function_params(prog)

    def is_three(e) -> bool:
        return isinstance(e, tuple) and len(e) == 2 and e[0] == "ident" and e[1] in three_names

    def member_rule(nm: str, how: str = "") -> None:
        if nm not in THREE_ALLOWED:
            if nm in THREE_DISALLOWED_KNOWN:
                fail("FORBIDDEN_THREE_API", f"THREE.{nm}{how} is a real three.js API that the output "
                                            f"specification excludes")
            else:
                fail("UNKNOWN_THREE_API", f"THREE.{nm}{how} is not a supported three.js member")

    def receive_three(p, param: bool) -> None:
        """A binding that receives THREE itself: a parameter named THREE, or object destructuring of allowed
        members (nested destructuring of MathUtils may not take its blocked members)."""
        if p[0] == "id":
            if not (param and p[1] == "THREE"):
                fail("THREE_ALIAS_FORBIDDEN", f"passing THREE to a parameter named `{p[1]}` (name it THREE)" if param
                     else f"aliasing THREE as `{p[1]}`")
            return
        if p[0] != "objpat":
            fail("THREE_ALIAS_FORBIDDEN", "THREE may only be destructured as an object of allowed members")
            return
        if p[2]:
            fail("THREE_ALIAS_FORBIDDEN", f"rest-destructure of THREE (...{p[2]})")
        for key, target, default in p[1]:
            if isinstance(key, tuple):
                fail("COMPUTED_PROPERTY_ACCESS", "computed destructure of THREE")
                continue
            member_rule(str(key), " (destructured)")
            inner = target
            if key in THREE_BLOCKED_SUBMEMBERS and inner[0] == "objpat":
                if inner[2]:
                    fail("FORBIDDEN_THREE_API", f"THREE.{key}.{{...}} rest-destructure")
                for sub, _, _ in inner[1]:
                    if isinstance(sub, str) and sub in THREE_BLOCKED_SUBMEMBERS[key]:
                        fail("FORBIDDEN_THREE_API", f"THREE.{key}.{sub} (destructured) is not allowed")
            if default is not None:
                _walk(default, visit)

    def three_args(callee, args, is_new: bool) -> None:
        ks = [k for k, a in enumerate(args) if is_three(a)]
        if not ks:
            return
        if is_new and callee[0] == "member" and is_three(callee[1]):
            fail("THREE_ALIAS_FORBIDDEN", "THREE passed to a three.js constructor")
            return
        params = None
        if callee[0] == "ident":
            params = funcs.get(callee[1])
        elif callee[0] == "func":
            params = callee[2]
        elif callee[0] == "class":
            params = _ctor_params(callee)
        if params is None:
            fail("THREE_ALIAS_FORBIDDEN", "THREE passed to a function the checker cannot resolve")
            return
        for k in ks:
            if k >= len(params):
                fail("THREE_ALIAS_FORBIDDEN", "THREE passed to a rest or missing parameter")
            else:
                receive_three(params[k][0], True)

    def visit(n):
        tag = n[0]
        if tag in ("call", "new"):
            three_args(n[1], n[2], tag == "new")
            _walk(n[1], visit)
            for a in n[2]:
                if not is_three(a):
                    _walk(a, visit)
            return False
        if tag == "decl":
            for target, init in n[2]:
                if is_three(init):
                    receive_three(target, False)
                else:
                    _walk(target, visit)
                    if init is not None:
                        _walk(init, visit)
            return False
        if tag == "assign" and n[1] == "=" and is_three(n[3]):
            fail("THREE_ALIAS_FORBIDDEN", "assigning THREE to a variable or member")
            _walk(n[2], visit)
            return False
        if tag == "assign_pat" and is_three(n[2]):
            receive_three(n[1], False)
            return False
        if tag == "spread" and is_three(n[1]):
            fail("THREE_ALIAS_FORBIDDEN", "spread of THREE")
            return False
        if tag == "ident":
            nm = n[1]
            if nm in FORBIDDEN_IDENTIFIERS:
                if nm not in seen_forbidden:
                    fail("FORBIDDEN_IDENTIFIER", f"`{nm}` is not allowed")
                    seen_forbidden.add(nm)
            elif nm in three_names:
                fail("THREE_ALIAS_FORBIDDEN", f"`{nm}` used in a position the checker cannot follow "
                                              f"(only THREE.Member, destructuring, or a helper's THREE parameter)")
            elif nm == "THREE" and nm not in declared:
                fail("THREE_AT_TOP_LEVEL", "THREE referenced outside generate")
            elif nm not in declared and nm not in ALLOWED_ROOTS:
                if nm not in seen_forbidden:
                    fail("IDENTIFIER_NOT_ALLOWED", f"`{nm}` is not declared and not an allowed global")
                    seen_forbidden.add(nm)
            return True
        if tag == "member":
            obj, key, computed = n[1], n[2], n[4]
            if key[0] == "lit" and isinstance(key[1], str) and key[1] in FORBIDDEN_PROPERTIES:
                fail("FORBIDDEN_PROPERTY_ACCESS", f"`.{key[1]}` is not allowed")
            if obj[0] == "ident" and computed and obj[1] != three and obj[1] in COMPUTED_ACCESS_GATED \
                    and obj[1] not in declared:
                fail("COMPUTED_PROPERTY_ACCESS", f"`{obj[1]}[...]` is not allowed")
            if obj[0] == "ident" and obj[1] == "Math" and not computed and key == ("lit", "random") \
                    and "Math" not in declared:
                fail("FORBIDDEN_IDENTIFIER", "Math.random is not allowed (write a seeded generator)")
            if obj[0] == "ident" and obj[1] in three_names:
                if computed or key[0] != "lit":
                    fail("COMPUTED_PROPERTY_ACCESS", f"`{obj[1]}[...]` is not allowed")
                else:
                    member_rule(str(key[1]))
                _walk(key, visit)
                return False
            if obj[0] == "ident" and obj[1] == "THREE" and "THREE" not in declared:
                fail("THREE_AT_TOP_LEVEL", "THREE referenced outside generate")
                return False
            if obj[0] == "member" and obj[1][0] == "ident" and obj[1][1] in three_names and key[0] == "lit":
                ns = obj[2][1] if obj[2][0] == "lit" else None
                if ns in THREE_BLOCKED_SUBMEMBERS and key[1] in THREE_BLOCKED_SUBMEMBERS[ns]:
                    fail("FORBIDDEN_THREE_API", f"THREE.{ns}.{key[1]} is not allowed")
            _walk(obj, visit)
            if key[0] != "lit":          # property names are not literals for the budget
                _walk(key, visit)
            return False
        if tag == "lit":
            v = n[1]
            if isinstance(v, str):
                literal_bytes[0] += len(v)
            elif isinstance(v, float):
                literal_bytes[0] += 8
            return True
        if tag == "tpl":
            literal_bytes[0] += sum(len(p) for p in n[1] if isinstance(p, str))
            return True
        return True

    # the default-exported function's parameter list declares THREE; uses of THREE elsewhere are aliases
    _walk(body, visit)
    if literal_bytes[0] > LITERAL_BUDGET:
        fail("LITERAL_BUDGET_EXCEEDED", f"{literal_bytes[0]} bytes of literals (limit {LITERAL_BUDGET})")
    return fails


# --------------------------------------------------------------------------------------------- post-validation


def declared_vertices(g, n_triangles: int = 0) -> int:
    """Vertex count three.js would build for a primitive's parameters (the preview mesh caps segments, the
    limit must not). Non-indexed three.js geometries (polyhedra, extrusions) count three vertices per triangle."""
    p = g.params

    def n(k, d):
        v = p.get(k, d)
        try:
            return max(0, int(jsvm._to_num(v)))
        except (TypeError, ValueError, OverflowError):
            return d
    t = g.gtype
    if t == "BoxGeometry":
        a, b, c = n("widthSegments", 1), n("heightSegments", 1), n("depthSegments", 1)
        return 2 * ((a + 1) * (b + 1) + (a + 1) * (c + 1) + (b + 1) * (c + 1))
    if t == "SphereGeometry":
        return (n("widthSegments", 32) + 1) * (n("heightSegments", 16) + 1)
    if t in ("CylinderGeometry", "ConeGeometry"):
        r = n("radialSegments", 32)
        caps = 0
        if not jsvm._truthy(p.get("openEnded", False)):
            radii = ((jsvm._to_num(p.get("radiusTop", 1.0)), jsvm._to_num(p.get("radiusBottom", 1.0)))
                     if t == "CylinderGeometry" else (0.0, 1.0))
            caps = sum(1 for x in radii if x > 0)
        return (r + 1) * (n("heightSegments", 1) + 1) + caps * (2 * r + 1)
    faces = {"TetrahedronGeometry": 4, "OctahedronGeometry": 8, "IcosahedronGeometry": 20, "DodecahedronGeometry": 36}
    if t in faces:
        return 3 * faces[t] * (n("detail", 0) + 1) ** 2
    if t in ("ExtrudeGeometry", "PolyhedronGeometry"):
        return 3 * n_triangles
    if t == "PlaneGeometry":
        return (n("widthSegments", 1) + 1) * (n("heightSegments", 1) + 1)
    if t == "TorusGeometry":
        return (n("radialSegments", 12) + 1) * (n("tubularSegments", 48) + 1)
    if t == "TorusKnotGeometry":
        return (n("tubularSegments", 64) + 1) * (n("radialSegments", 8) + 1)
    if t == "CircleGeometry":
        return n("segments", 32) + 2
    if t == "RingGeometry":
        return (n("thetaSegments", 32) + 1) * (n("phiSegments", 1) + 1)
    if t == "TubeGeometry":
        return (n("tubularSegments", 64) + 1) * (n("radialSegments", 8) + 1)
    if t == "LatheGeometry":
        pts = p.get("points")
        return (n("segments", 12) + 1) * (len(pts.items) if isinstance(pts, jsvm.JSArray) else 2)
    if t == "CapsuleGeometry":
        return (n("radialSegments", 8) + 1) * (2 * n("capSegments", 4) + 2)
    return 0


def async_use(code: str) -> Optional[str]:
    """The specification's ASYNC_NOT_ALLOWED detail for the first async function, async arrow or method, `for await`
    or `await` in the module, or None. (The interpreter does not run async code, so this is decided on tokens,
    before parsing.)"""
    try:
        toks = jsvm.tokenize(code)
    except jsvm.JSError:
        return None

    def line(t):
        return code.count("\n", 0, t.pos) + 1

    def val(i):
        return toks[i].val if 0 <= i < len(toks) else None
    for i, t in enumerate(toks):
        if t.val == "async" and t.kind in ("kw", "id") and val(i - 1) != ".":
            nxt = val(i + 1)
            is_async = nxt == "function" or (toks[i + 1].kind == "id" and val(i + 2) in ("=>", "(")) if nxt else False
            if nxt == "(":                                  # async (a, b) => ...
                depth, j = 0, i + 1
                while j < len(toks):
                    if toks[j].val == "(" and toks[j].kind == "p":
                        depth += 1
                    elif toks[j].val == ")" and toks[j].kind == "p":
                        depth -= 1
                        if depth == 0:
                            break
                    j += 1
                is_async = val(j + 1) == "=>"
            if is_async:
                if val(i - 1) == "default" and val(i - 2) == "export":
                    return "default export is an async function"
                return f"async function at line {line(t)}"
        if t.val == "for" and t.kind == "kw" and val(i + 1) == "await":
            return f"for await loop at line {line(t)}"
        if t.val == "await" and t.kind in ("kw", "id") and val(i - 1) != ".":
            return f"top-level await at line {line(t)}"
    return None


def post_validate(root) -> tuple:
    """Walk the returned tree once with cycle detection. -> (failures, stats)."""
    fails: List[Dict[str, str]] = []

    def fail(rule, detail):
        fails.append({"stage": "post_validation", "rule": rule, "detail": detail})

    if not isinstance(root, jsvm.Object3D):
        fail("INVALID_RETURN_TYPE", f"generate must return an Object3D, got {jsvm._typeof(root)}")
        return fails, {}
    if root.otype not in ROOT_TYPES:
        fail("INVALID_RETURN_TYPE", f"returned {root.otype}, expected Group/Mesh/LineSegments/Points")
        return fails, {}
    stats = {"vertices": 0, "drawCalls": 0, "depth": 0, "instances": 0, "textureBytes": 0, "meshes": 0}
    seen = set()
    seen_tex = set()
    stack = [(root, 0)]
    bad_numbers = False
    while stack:
        o, d = stack.pop()
        if id(o) in seen:
            fail("CYCLE_DETECTED", "the object graph contains a cycle")
            break
        seen.add(id(o))
        stats["depth"] = max(stats["depth"], d)
        if d > LIMITS["depth"]:
            fail("DEPTH_LIMIT_EXCEEDED", f"walk exceeded max depth {LIMITS['depth']}")
            break
        for k in ("position", "rotation", "scale"):
            if any(not math.isfinite(x) for x in o.props[k].v()):
                bad_numbers = True
        g = o.props.get("geometry")
        if o.otype in DRAW_TYPES and not isinstance(g, jsvm.Geometry):
            stats["drawCalls"] += 1
        if isinstance(g, jsvm.Geometry) and o.otype in DRAW_TYPES:
            try:
                v, tris = jsvm.geometry_mesh(g)
                nv = max(int(v.shape[0]), declared_vertices(g, int(tris.shape[0])))
                if v.numel() and not bool(v.isfinite().all()):
                    bad_numbers = True
            except jsvm._Throw as e:
                fail("GEOMETRY_ERROR", jsvm._to_str(e.value.props.get("message", "")) if isinstance(e.value, jsvm.JSObject) else "bad geometry")
                nv = 0
            if o.otype == "InstancedMesh":                 # one draw of the geometry, `count` instances
                stats["instances"] += int(jsvm._to_num(o.props.get("count", 0)))
            stats["vertices"] += nv
            stats["drawCalls"] += 1
            stats["meshes"] += 1
            m = o.props.get("material")
            for mm in (m.items if isinstance(m, jsvm.JSArray) else [m]):
                if isinstance(mm, jsvm.Material):
                    for key in MAP_PROPS:
                        val = mm.props.get(key)
                        if isinstance(val, jsvm.Texture) and val.props.get("isDataTexture") and id(val) not in seen_tex:
                            seen_tex.add(id(val))
                            stats["textureBytes"] += val.nbytes
        for c in o.children():
            stack.append((c, d + 1))
    if bad_numbers:
        fail("NON_FINITE_VALUE", "a transform or vertex is NaN or infinite")
    for key, rule, unit in (("vertices", "VERTEX_LIMIT_EXCEEDED", "vertices"),
                            ("drawCalls", "DRAW_CALL_LIMIT_EXCEEDED", "draw calls"),
                            ("instances", "INSTANCE_LIMIT_EXCEEDED", "instances"),
                            ("textureBytes", "TEXTURE_DATA_EXCEEDED", "bytes")):
        if stats[key] > LIMITS[key]:
            fail(rule, f"{stats[key]} {unit} (limit {LIMITS[key]})")
    if stats["meshes"] == 0 and not fails:
        fail("EMPTY_SCENE", "the returned object contains no meshes")
    elif not fails:
        bb = jsvm.world_bbox(root)
        if bb is None:
            fail("EMPTY_SCENE", "the returned object's bounding box is empty")
        else:
            lo, hi = [float(v) for v in bb[0]], [float(v) for v in bb[1]]
            stats["bbox"] = {"min": lo, "max": hi}
            if any(v < -BOUND - BOUND_TOL for v in lo) or any(v > BOUND + BOUND_TOL for v in hi):
                fail("BOUNDING_BOX_OUT_OF_RANGE", "box [" + ", ".join(f"{v:.3f}" for v in lo) + "] to [" +
                     ", ".join(f"{v:.3f}" for v in hi) + "] (must fit in [-0.5, 0.5] on every axis)")
    return fails, stats


# -------------------------------------------------------------------------------------------------- module


@dataclass
class CheckerSettings:
    # the specification gives a module 5 s in V8; this interpreter runs the same JavaScript tens of times slower,
    # so its wall-clock budget is scaled up and the step budget is what stops runaway loops
    timeout_s: float = 20.0
    max_steps: int = 20_000_000
    repair: bool = True
    constant_repair: bool = True     # context-aware repair of unknown THREE constants (app/threefix.py)
    failure_repair: bool = True      # failure-driven mechanical repairs (app/jsrepair.py)
    repair_rounds: int = 3
    workers: int = 4
    processes: bool = False          # a process pool (true parallelism) instead of threads
    pin_reserve: int = 14            # process pool: leave this many CPUs of the quota to the rest of the host


def _check_in_process(settings: "CheckerSettings", text: str, seed: int) -> "CheckResult":
    return JSChecker(settings, _inline=True).check(text, seed)


def _pin_worker(cpus):
    from ..utils.affinity import pin_current_process
    pin_current_process(cpus)


class JSChecker:
    """check(code) -> CheckResult. check_async runs in a pool: threads by default (the interpreter keeps no
    shared state, every call builds its own), or processes pinned to the CPU set of
    `utils.affinity.worker_cpus` so checks run in parallel without taking the engines' cores."""

    def __init__(self, settings: Optional[CheckerSettings] = None, _inline: bool = False):
        self.s = settings or CheckerSettings()
        self.counts = {"checked": 0, "passed": 0}
        self._pool = None
        if _inline:
            return
        if self.s.processes:
            import multiprocessing as mp
            from concurrent.futures import ProcessPoolExecutor
            from ..utils.affinity import worker_cpus
            cpus = worker_cpus(reserve=self.s.pin_reserve)
            self._pool = ProcessPoolExecutor(max_workers=self.s.workers, mp_context=mp.get_context("spawn"),
                                             initializer=_pin_worker, initargs=(cpus,))
        else:
            self._pool = ThreadPoolExecutor(max_workers=self.s.workers, thread_name_prefix="jscheck")

    def check(self, text: str, seed: int = 0) -> CheckResult:
        """extract -> mechanical repair -> checks; a module whose only failures are unknown THREE constants gets
        one context-aware constant rewrite, kept only if the rewritten module passes every check."""
        self.counts["checked"] += 1
        code = extract_code(text)
        fixes: List[str] = []
        if self.s.repair:
            code, fixes = mechanical_repair(code)
        res = self._check_code(code, seed, fixes)
        if not res.ok and self.s.constant_repair:
            names = threefix.plan(res.failures)
            rw = threefix.rewrite(code, names, res.stats.get("three") or "THREE") if names else None
            if rw is not None:
                res2 = self._check_code(rw[0], seed, fixes + rw[1])
                if res2.ok:
                    res = res2
        if not res.ok and self.s.failure_repair:
            res = self._repair_rounds(res, seed)
        if res.ok:
            self.counts["passed"] += 1
        return res

    def _repair_rounds(self, res: CheckResult, seed: int) -> CheckResult:
        """Apply the failure-driven repairs the failures call for and check again, for a few rounds (a fix can
        uncover the next failure); the first passing module is kept, else the original result stands."""
        cur = res
        for _ in range(self.s.repair_rounds):
            steps = jsrepair.plan(cur.failures)
            if not steps:
                break
            try:
                declared = _declared_names(jsvm.Parser(cur.code).program())
            except (jsvm.JSError, RecursionError):
                declared = set()
            rw = jsrepair.apply(cur.code, steps, declared)
            if rw is None:
                break
            cur = self._check_code(rw[0], seed, cur.repaired + rw[1])
            if cur.ok:
                return cur
        return res

    def _check_code(self, code: str, seed: int, fixes: List[str]) -> CheckResult:
        size = len(code.encode("utf-8"))
        if size > MAX_FILE_BYTES:
            return CheckResult(False, [{"stage": "parse", "rule": "FILE_SIZE_EXCEEDED",
                                        "detail": f"{size} bytes (limit {MAX_FILE_BYTES})"}], code, repaired=fixes)
        asy = async_use(code)
        if asy is not None:
            return CheckResult(False, [{"stage": "static_analysis", "rule": "ASYNC_NOT_ALLOWED", "detail": asy}], code,
                               repaired=fixes)
        try:
            prog = jsvm.Parser(code).program()
        except jsvm.JSError as e:
            return CheckResult(False, [{"stage": "parse", "rule": "PARSE_ERROR", "detail": e.msg}], code, repaired=fixes)
        except RecursionError:
            return CheckResult(False, [{"stage": "parse", "rule": "PARSE_ERROR", "detail": "nesting too deep"}], code,
                               repaired=fixes)
        dup = redeclared_name(prog)
        if dup is not None:
            return CheckResult(False, [{"stage": "parse", "rule": "PARSE_ERROR",
                                        "detail": f"Identifier '{dup}' has already been declared"}], code,
                               repaired=fixes)
        fails = static_analyze(prog)
        if fails:
            return CheckResult(False, fails, code, stats={"three": three_param(prog)}, repaired=fixes)
        res = jsvm.run_module(code, jsvm.Limits(steps=self.s.max_steps, seconds=self.s.timeout_s), seed=seed)
        if res.error is not None:
            rule = ("HEAP_EXCEEDED" if res.error.startswith("HEAP") else
                    "TIMEOUT_EXCEEDED" if res.error.startswith("TIMEOUT") else "EXECUTION_THREW")
            return CheckResult(False, [{"stage": "execution", "rule": rule, "detail": res.error}], code,
                               stats={"steps": res.steps, "exec_s": res.seconds}, repaired=fixes)
        fails, stats = post_validate(res.root)
        stats.update({"steps": res.steps, "exec_s": round(res.seconds, 4)})
        if fails:
            return CheckResult(False, fails, code, stats=stats, repaired=fixes)
        try:
            scene = jsvm.to_scene_json(res.root)
        except (ValueError, jsvm._Throw) as e:
            return CheckResult(False, [{"stage": "serialize", "rule": "SERIALIZE_ERROR", "detail": str(e)[:200]}],
                               code, stats=stats, repaired=fixes)
        return CheckResult(True, [], code, scene=scene, stats=stats, repaired=fixes)

    async def check_async(self, text: str, seed: int = 0) -> CheckResult:
        loop = asyncio.get_running_loop()
        if self.s.processes:
            self.counts["checked"] += 1
            r = await loop.run_in_executor(self._pool, _check_in_process, self.s, text, seed)
            self.counts["passed"] += int(r.ok)
            return r
        return await loop.run_in_executor(self._pool, self.check, text, seed)

    def close(self):
        if self._pool is not None:
            self._pool.shutdown(wait=False, cancel_futures=True)
