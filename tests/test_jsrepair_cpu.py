"""Failure-driven mechanical repairs (app/jsrepair.py) and the checker's redeclaration rule."""
from phung5_b200.app import jsrepair, jsvm
from phung5_b200.app.jscheck import CheckerSettings, JSChecker, redeclared_name

TAIL = " const g = new THREE.Group(); g.add(new THREE.Mesh(new THREE.BoxGeometry(1, 1, 1), " \
       "new THREE.MeshBasicMaterial())); return g; }"


def _module(body: str) -> str:
    return "export default function generate(THREE) {" + body + TAIL


def _checker(**kw) -> JSChecker:
    s = CheckerSettings()
    for k, v in kw.items():
        setattr(s, k, v)
    return JSChecker(s, _inline=True)


def _dup(src: str):
    return redeclared_name(jsvm.Parser(src).program())


def test_redeclaration_is_a_parse_error_only_where_js_rejects_it():
    assert _dup(_module("const a = 1; const a = 2;")) == "a"
    assert _dup(_module("let a = 1; var a = 2;")) == "a"
    assert _dup(_module("function f(p) { let p = 1; return p; } f(1);")) == "p"
    assert _dup(_module("switch (1) { case 1: let s = 1; break; default: let s = 2; }")) == "s"
    assert _dup("const t = 1; function t() {}\n" + _module("")) == "t"          # module top level
    # allowed: sibling blocks, var over a parameter, var twice, functions twice at a function's top, shadowing
    assert _dup(_module("{ let z = 1; } { let z = 2; }")) is None
    assert _dup(_module("function f(p) { var p = 1; var p = 2; return p; } f(1);")) is None
    assert _dup(_module("function h() { function k() {} function k() {} } h();")) is None
    assert _dup(_module("const a = 1; { const a = 2; }")) is None
    assert _dup(_module("for (const k of [1, 2]) { const j = k; } for (const k of [3]) {}")) is None
    res = _checker(failure_repair=False).check(_module("const a = 1; const a = 2;"))
    assert not res.ok and res.failures[0] == {"stage": "parse", "rule": "PARSE_ERROR",
                                               "detail": "Identifier 'a' has already been declared"}


def test_each_class_repairs_its_failure_and_the_result_passes():
    c = _checker()
    cases = {
        "const a = [1]; const a = [2, 3]; const n = a.length;": "redeclared: a",
        "const w = 1; w = 2;": "constlet: w",
        "let x = (1 + 2));": "paren: )",
        "const roundedPts = [1, 2]; const q = rounded_pts.length;": "ident: rounded_pts",
    }
    for body, fix in cases.items():
        res = c.check(_module(body))
        assert res.ok, (body, res.summary())
        assert fix in res.repaired
    # the redeclared name's later declaration became an assignment to the first (now `let`) binding
    res = c.check(_module("const a = [1]; const a = [2, 3];"))
    assert "let a = [1]; a = [2, 3];" in res.code


def test_repairs_chain_over_rounds_and_leave_strings_alone():
    src = _module('const label = "const w = 1; w = 2; ))"; const w = 1; w = 2; let y = (3));')
    res = _checker().check(src)
    assert res.ok, res.summary()
    assert res.repaired == ["paren: )", "constlet: w"]
    assert '"const w = 1; w = 2; ))"' in res.code                 # the string literal is untouched


def test_no_repair_when_a_failure_has_no_class_or_the_fix_is_ambiguous():
    assert jsrepair.plan([{"rule": "PARSE_ERROR", "detail": "Identifier 'a' has already been declared"},
                          {"rule": "VERTEX_LIMIT_EXCEEDED", "detail": "300000 vertices"}]) == []
    # two declared names match `my_val` up to case / underscores: no guess
    res = _checker().check(_module("const myVal = 1; const MyVal = 2; const q = my_val + 1;"))
    assert not res.ok and res.failures[0]["rule"] == "IDENTIFIER_NOT_ALLOWED" and not res.repaired
    # destructuring redeclarations are not rewritten
    assert jsrepair.fix_redeclared("const {a} = o; const a = 2;", "a") is None
    # off: the failure stands
    res = _checker(failure_repair=False).check(_module("const w = 1; w = 2;"))
    assert not res.ok and res.failures[0]["rule"] == "EXECUTION_THREW"


def test_only_the_wall_clock_timeout_is_retried():
    assert jsrepair.plan([{"rule": "TIMEOUT_EXCEEDED", "detail": "TIMEOUT: execution exceeded 5.0s"}]) == \
        [("retry", "")]
    assert jsrepair.plan([{"rule": "TIMEOUT_EXCEEDED",
                           "detail": "TIMEOUT: step budget of 20000000 exceeded"}]) == []
