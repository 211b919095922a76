"""Statement and scoping semantics of the module interpreter (hoisting, closures in loops, switch, try/finally,
defaults, destructuring, `this` in arrows, logical assignment, array helpers)."""
import pytest

from phung5_b200.app import jsvm


def _ev(pre, expr):
    src = ("export default function generate(THREE) { const g = new THREE.Group(); " + pre +
           " g.userData.v = " + expr + "; return g; }")
    r = jsvm.run_module(src, jsvm.Limits(steps=500_000, seconds=5))
    assert r.error is None, r.error
    v = r.root.props["userData"].props["v"]

    def norm(x):
        return [norm(y) for y in x.items] if isinstance(x, jsvm.JSArray) else x
    return norm(v)


CASES = [
 ("function f(){ x = 1; var x; return x; }", "f()", 1),
 ("var fs=[]; for (var i=0;i<3;i++) fs.push(()=>i);", "fs.map(f=>f())", [3, 3, 3]),
 ("const fs=[]; for (let i=0;i<3;i++) fs.push(()=>i);", "fs.map(f=>f())", [0, 1, 2]),
 ("let r=[]; switch (2) { case 1: r.push(1); case 2: r.push(2); case 3: r.push(3); break; case 4: r.push(4); }", "r", [2, 3]),
 ("let x=0; function f(){ try { return 1 } finally { x = 2 } }", "[f(), x]", [1, 2]),
 ("function f(){ try { throw new Error('boom') } catch (e) { return e.message } }", "f()", "boom"),
 ("function f(){ try { throw 5 } catch { return 'caught' } }", "f()", "caught"),
 ("function f(a, b = a * 2) { return b }", "f(3)", 6),
 ("function f(...xs) { return xs.length }", "f(1, 2, 3)", 3),
 ("const {a = 5, b: {c} = {c: 3}} = {};", "[a, c]", [5, 3]),
 ("const o = {v: 2, f() { return [1].map(() => this.v) }};", "o.f()", [2]),
 ("const o = {a: 1, b: 2};", "['a' in o, 'z' in o]", [True, False]),
 ("", "typeof notDefinedAnywhere", "undefined"),
 ("const o = {a: 1}; o.a++; o['b'] = 1; o['b'] += 2;", "[o.a, o.b]", [2, 3]),
 ("let n = 0; let i = 0; while (i < 10) { i++; if (i % 2) continue; if (i > 8) break; n += i; }", "n", 20),
 ("const a = [1, 2, 3]; const [x, ...rest] = a;", "rest", [2, 3]),
 ("function f() { return arguments[1]; }", "f(1, 'b')", "b"),
 ("const x = (1, 2, 3);", "x", 3),
 ("", "void 0 === undefined", True),
 ("", "[1, 2] instanceof Array", True),
 ("class A { static get k() { return 7; } }", "A.k", 7),
 ("let s = 0; for (const k in {a: 1, b: 2}) s += k.length;", "s", 2),
 ("let s = ''; for (const ch of 'abc') s = ch + s;", "s", "cba"),
 ("const m = [[1, 2], [3, 4]];", "m.map(([a, b]) => a * b)", [2, 12]),
 ("const f = (a, {b = 2} = {}) => a + b;", "f(1)", 3),
 ("let i = 0; do { i += 3 } while (i < 10);", "i", 12),
 ("const o = {['k' + 1]: 5};", "o.k1", 5),
 ("const x = 5; const y = x > 3 ? x > 4 ? 'big' : 'mid' : 'small';", "y", "big"),
 ("let a = null; a ??= 4; let b = 1; b ||= 9; let c = 1; c &&= 7;", "[a, b, c]", [4, 1, 7]),
 ("const arr = [5, 1, 4]; arr.reverse(); arr.push(...[7, 8]);", "arr", [4, 1, 5, 7, 8]),
 ("function Fib(n) { return n < 2 ? n : Fib(n - 1) + Fib(n - 2); }", "Fib(15)", 610),
 ("const o = {x: 1, y: {z: 2}}; const c = {...o, x: 3};", "[c.x, c.y.z, o.x]", [3, 2, 1]),
 ("const a = [3, 1, 2]; const b = [...a].sort();", "[a[0], b[0]]", [3, 1]),
 ("let t = 0; [1, 2, 3].forEach((v, i, arr) => { t += v * i + arr.length; });", "t", 17),
 ("const s = new Set(); s.add(1).add(2).add(1);", "[...s]", [1, 2]),
 ("const e = [1, 2, 3].entries ? 1 : 0;", "e", 1),
 ("const r = [1, 2, 3, 4].filter((v, i) => i % 2 === 0);", "r", [1, 3]),
 ("const x = Math.min(...[4, 2, 8]);", "x", 2),
 ("const x = [1, 2, 3].some(v => v > 2) && [1, 2].every(v => v > 0);", "x", True),
 ("const x = [[1], [2, [3]]].flat(Infinity);", "x", [1, 2, 3]),
 ("const x = Array.from(new Set([1, 1, 2]));", "x", [1, 2]),
 ("const x = Object.entries({a: 1}).map(([k, v]) => k + v);", "x", ["a1"]),
]


@pytest.mark.parametrize("pre,expr,want", CASES)
def test_semantics(pre, expr, want):
    assert _ev(pre, expr) == want
