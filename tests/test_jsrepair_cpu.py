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


def test_undeclared_value_gets_a_stub_only_when_it_is_a_plain_value():
    res = _checker().check(_module("const q = widthh * 2;"))
    assert res.ok and res.repaired == ["ident: widthh"] and "let widthh = 0;" in res.code
    for use in ("const q = widthh(2);", "const q = widthh.x;", "const q = new widthh();", "const q = widthh[0];"):
        res = _checker().check(_module(use))
        assert not res.ok and not res.repaired, use


TEXTURES = """export default function generate(THREE) { const g = new THREE.Group();
  for (let k = 0; k < 5; k++) {
    const n = 512; const data = new Uint8Array(n * n * 4);
    for (let i = 0; i < 64; i++) data[i] = 4 * i;
    const t = new THREE.DataTexture(data, n, n, THREE.RGBAFormat); t.needsUpdate = true;
    g.add(new THREE.Mesh(new THREE.BoxGeometry(0.1, 0.1, 0.1), new THREE.MeshStandardMaterial({map: t})));
  }
  return g; }"""


def test_texture_class_halves_large_rgba_textures():
    off = _checker(failure_repair=False).check(TEXTURES)
    assert [f["rule"] for f in off.failures] == ["TEXTURE_DATA_EXCEEDED"]
    assert off.failures[0]["detail"] == "5242880 bytes (limit 4194304)"
    res = _checker().check(TEXTURES)
    assert res.ok and res.repaired == ["texture"] and res.stats["textureBytes"] == 5 * 256 * 256 * 4
    # beyond four times the limit a halving cannot fit: no rewrite
    assert jsrepair.plan([{"rule": "TEXTURE_DATA_EXCEEDED", "detail": "16777217 bytes (limit 4194304)"}]) == []


def test_texture_helper_runs_natively_with_the_same_result():
    body = """export default function generate(THREE) { const g = new THREE.Group();
      const n = 256; const data = new Uint8Array(n * n * 4);
      for (let i = 0; i < data.length; i += 97) data[i] = (i * 7) % 256;
      const t = __phxDataTexture(THREE, data, n, n, THREE.RGBAFormat);
      const s = __phxDataTexture(THREE, new Uint8Array(16), 2, 2);
      g.userData.v = [t.image.width, t.image.height, s.image.width, Array.from(t.image.data)];
      return g; }"""
    fast = jsvm.run_module(jsrepair.HALF_TEXTURE + body, jsvm.Limits(seconds=60))
    slow_src = (jsrepair.HALF_TEXTURE + body).replace("__phxDataTexture", "__phxDataTextureInterpreted")
    slow = jsvm.run_module(slow_src, jsvm.Limits(seconds=120))
    assert fast.error is None and slow.error is None, (fast.error, slow.error)
    assert fast.steps < slow.steps // 10                       # the native ran
    a = fast.root.props["userData"].props["v"].items
    b = slow.root.props["userData"].props["v"].items
    assert a[:3] == b[:3] == [128, 128, 2]
    assert a[3].items == b[3].items and len(a[3].items) == 128 * 128 * 4
