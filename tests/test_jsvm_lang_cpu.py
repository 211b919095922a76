"""The module interpreter's JavaScript semantics: operator precedence, classes (extends, super, accessors, fields,
statics, subclassing a three.js object), object-literal accessors, function prototypes and labeled loops."""
import pytest

from phung5_b200.app import jsvm
from phung5_b200.app.jsvm import UNDEF


def _ev(expr, pre=""):
    src = ("export default function generate(THREE) { const g = new THREE.Group(); " + pre +
           " g.userData.v = " + expr + "; return g; }")
    r = jsvm.run_module(src, jsvm.Limits(steps=500_000, seconds=5))
    assert r.error is None, r.error
    return r.root.props["userData"].props["v"]


@pytest.mark.parametrize("expr,want", [
    ("2 + 1 * 100", 102), ("2 * 3 + 4 * 5", 26), ("1 + 2 * 3 + 4", 11), ("1 - 2 * 3 - 4", -9), ("10 - 2 - 3", 5),
    ("8 / 2 / 2", 2), ("7 % 4 * 2", 6), ("2 ** 3 * 2", 16), ("2 ** 3 ** 2", 512), ("1 + 2 * 3 ** 2 / 3 - 1", 6),
    ("(true ? 10 : 0) + 1 * 100", 110), ("1 << 2 + 1", 8), ("1 | 2 & 3 ^ 4", 7), ("3 > 2 > 1", False),
    ("1 + 2 < 4 && 5 > 3 || false", True), ("null ?? 5 + 1", 6), ("-2 * 3 + 1", -5), ('typeof 1 + "x"', "numberx"),
    ("0.5 * Math.PI * 2 - Math.PI", 0.0),
])
def test_operator_precedence(expr, want):
    assert _ev(expr) == want


def test_classes_extends_super_accessors_fields_and_statics():
    pre = """
      class A { constructor(x) { this.x = x; } f() { return this.x; } static make(x) { return new this(x); } }
      class B extends A {
        n = 2;
        static k = 7;
        constructor(x) { super(x + 1); this.y = this.n * 10; }
        f() { return super.f() * 100 + this.y; }
        get double() { return this.x * 2; }
        set double(v) { this.x = v / 2; }
      }
      const b = new B(1);
      b.double = 18;
    """
    assert _ev("b.f() + B.k", pre) == 927          # x 9 after the setter: 900 + 20 + 7
    assert _ev("[b instanceof B, b instanceof A, B.make(4) instanceof B, b.double]", pre).items == [True, True,
                                                                                                    True, 18.0]


def test_subclass_of_a_three_object_keeps_host_methods_and_overrides():
    pre = """
      class Tree extends THREE.Group {
        constructor(h) { super(); this.add(new THREE.Mesh(new THREE.CylinderGeometry(0.1, 0.1, h, 8),
                                                           new THREE.MeshStandardMaterial())); }
        add(o) { super.add(o); this.userData.n = (this.userData.n || 0) + 1; return this; }
        trunk() { return this.children[0]; }
      }
      const t = new Tree(2);
      t.add(new THREE.Mesh(new THREE.SphereGeometry(0.3), new THREE.MeshStandardMaterial()));
      g.add(t);
    """
    assert _ev("[t instanceof THREE.Group, t instanceof Tree, t.children.length, t.userData.n, !!t.trunk()]",
               pre).items == [True, True, 2.0, 2.0, True]


def test_object_accessors_prototypes_labels_and_errors():
    assert _ev("o.v", "const o = { _v: 1, get v() { return this._v * 2; }, set v(x) { this._v = x; } }; o.v = 3;") == 6
    assert _ev("q.get() + (q instanceof P ? 10 : 0)",
               "function P(x) { this.x = x; } P.prototype.get = function () { return this.x + 1; }; const q = new P(4);") == 15
    assert _ev("n", "let n = 0; outer: for (let i = 0; i < 5; i++) { for (let j = 0; j < 5; j++) "
                    "{ if (j == 3) continue outer; if (i == 4) break outer; n++; } }") == 12
    r = jsvm.run_module("export default function generate(THREE) { class A {} class B extends A "
                        "{ constructor() { this.x = 1; super(); } } new B(); }", jsvm.Limits(steps=10_000, seconds=2))
    assert "before accessing 'this'" in r.error
    r = jsvm.run_module("export default function generate(THREE) { class A {} A(); }", jsvm.Limits(steps=10_000, seconds=2))
    assert "without 'new'" in r.error


@pytest.mark.parametrize("expr,want", [
    ("-5 % 3", -2), ("5 % -3", 2), ("(0 - 1) % 4", -1), ("1 + '2'", "12"), ("'3' * '4'", 12),
    ("String(0.1 + 0.2)", "0.30000000000000004"), ("String(1e21)", "1e+21"), ("String(2e-7)", "2e-7"),
    ("(2.5).toFixed(0)", "3"), ("(-2.5).toFixed(0)", "-3"), ("(1.005).toFixed(2)", "1.00"), ("(-0.0001).toFixed(2)", "-0.00"),
    ("(255).toString(16)", "ff"), ("(25).toString(2)", "11001"), ("(0.5).toString(2)", "0.1"),
    ("'10' < '9'", True), ("null == undefined", True), ("typeof null", "object"), ("~~-3.7", -3), ("-1 >>> 0", 4294967295),
    ("1 << 31", -2147483648), ("Math.round(-2.5)", -2), ("[10, 9, 1].sort().join()", "1,10,9"),
    ("Object.keys({b: 1, 2: 1, a: 1, 1: 1}).join(',')", "1,2,b,a"), ("parseInt('0x1f')", 31), ("Number(' 12 ')", 12),
    ("'a,b,c'.split(',', 2).join('|')", "a|b"), ("String.fromCharCode(65, 66)", "AB"), ("'abc'.at(-1)", "c"),
    ("'abc'.substring(2, 0)", "ab"), ("'abcdef'.substr(1, 2)", "bc"), ("'7'.padStart(4, 'ab')", "aba7"),
    ("'b' + 'a' + + 'a' + 'a'", "baNaNa"), ("[null, undefined, 1].join('-')", "--1"), ("(function () { return arguments.length; })(1, 2, 3)", 3),
])
def test_js_semantics(expr, want):
    assert _ev(expr) == want


def test_object_quaternion_is_a_live_view_and_world_transforms():
    # the usual beam-between-two-points idiom: orient a cylinder with quaternion.setFromUnitVectors
    pre = """
      const a = new THREE.Vector3(0, 0, 0), b = new THREE.Vector3(0.3, 0.3, 0);
      const dir = b.clone().sub(a);
      const beam = new THREE.Mesh(new THREE.CylinderGeometry(0.02, 0.02, dir.length(), 8), new THREE.MeshStandardMaterial());
      beam.position.copy(a).add(b).multiplyScalar(0.5);
      beam.quaternion.setFromUnitVectors(new THREE.Vector3(0, 1, 0), dir.clone().normalize());
      const up = new THREE.Vector3(0, 1, 0).applyQuaternion(beam.quaternion);
      const parent = new THREE.Group(); parent.position.set(1, 0, 0); parent.add(beam);
      const w = beam.getWorldPosition(new THREE.Vector3());
      const child = new THREE.Mesh(new THREE.BoxGeometry(0.1, 0.1, 0.1), new THREE.MeshStandardMaterial());
      child.position.set(0.5, 0, 0); parent.add(child);
      g.attach(child);
      const q = new THREE.Quaternion().setFromAxisAngle(new THREE.Vector3(0, 0, 1), Math.PI / 2);
      const h = new THREE.Quaternion().slerp(q, 0.5);
      const m = new THREE.Matrix4().makeRotationZ(0.3).setPosition(1, 2, 3);
      const p = new THREE.Vector3(), qq = new THREE.Quaternion(), sc = new THREE.Vector3();
      m.clone().invert().invert().decompose(p, qq, sc);
    """
    got = _ev("[up.x, up.y, beam.rotation.z, w.x, child.position.x, child.parent === g, "
              "new THREE.Euler().setFromQuaternion(h).z, p.z, sc.x]", pre).items
    r2 = 1 / 2 ** 0.5
    assert got[0] == pytest.approx(r2) and got[1] == pytest.approx(r2)       # the rotation really changed
    assert got[2] == pytest.approx(-3.14159265 / 4)
    assert got[3] == pytest.approx(1.15) and got[4] == pytest.approx(1.5) and got[5] is True
    assert got[6] == pytest.approx(3.14159265 / 4) and got[7] == pytest.approx(3.0) and got[8] == pytest.approx(1.0)


def test_euler_order_is_honoured():
    pre = """
      const a = new THREE.Object3D(); a.rotation.order = 'YXZ'; a.rotation.set(0.3, 0.5, 0.2); a.updateMatrix();
      const b = new THREE.Object3D(); b.rotation.set(0.3, 0.5, 0.2); b.updateMatrix();
      const v1 = new THREE.Vector3(1, 2, 3).applyMatrix4(a.matrix), v2 = new THREE.Vector3(1, 2, 3).applyMatrix4(b.matrix);
      const q = new THREE.Quaternion().setFromEuler(a.rotation);
      const c = new THREE.Object3D(); c.rotation.order = 'YXZ'; c.quaternion.copy(q);
    """
    got = _ev("[v1.x, v2.x, c.rotation.x, c.rotation.y, c.rotation.z]", pre).items
    import math

    def rot(order, e, v):
        def R(ax, t):
            c_, s_ = math.cos(t), math.sin(t)
            return {"X": [[1, 0, 0], [0, c_, -s_], [0, s_, c_]], "Y": [[c_, 0, s_], [0, 1, 0], [-s_, 0, c_]],
                    "Z": [[c_, -s_, 0], [s_, c_, 0], [0, 0, 1]]}[ax]
        m = [[1, 0, 0], [0, 1, 0], [0, 0, 1]]
        for ax in order:
            r = R(ax, e["XYZ".index(ax)])
            m = [[sum(m[i][k] * r[k][j] for k in range(3)) for j in range(3)] for i in range(3)]
        return [sum(m[i][k] * v[k] for k in range(3)) for i in range(3)]
    assert got[0] == pytest.approx(rot("YXZ", (0.3, 0.5, 0.2), (1, 2, 3))[0])
    assert got[1] == pytest.approx(rot("XYZ", (0.3, 0.5, 0.2), (1, 2, 3))[0]) and got[0] != pytest.approx(got[1])
    assert got[2:] == pytest.approx([0.3, 0.5, 0.2])          # written back in the object's own order


def test_euler_order_travels_with_constructor_set_copy_and_object_clone():
    pre = """
      const e = new THREE.Euler(0.1, 0.2, 0.3, 'ZYX');
      const f = new THREE.Euler().copy(e), h = e.clone(), k = new THREE.Euler().set(1, 2, 3, 'YZX');
      const m = new THREE.Mesh(new THREE.BoxGeometry(0.2, 0.2, 0.2), new THREE.MeshBasicMaterial());
      m.rotation.order = 'ZXY'; m.rotation.set(0.3, 0.5, 0.7); m.position.set(0.1, 0.2, 0);
      m.userData.tag = {a: 1}; m.add(new THREE.Object3D());
      const c = m.clone(); c.position.x = 0.3;
      const d = new THREE.Mesh(); d.copy(m, false);
    """
    got = _ev("[e.order, f.order, h.order, k.order, c.rotation.order, c.quaternion.w - m.quaternion.w, m.position.x, "
              "c.geometry === m.geometry, c.userData.tag === m.userData.tag, c.userData.tag.a, c.children.length, "
              "d.rotation.order, d.position.y, d.children.length, d.material === m.material]", pre).items
    assert got[:5] == ["ZYX", "ZYX", "ZYX", "YZX", "ZXY"]
    assert got[5] == pytest.approx(0.0) and got[6] == pytest.approx(0.1)      # the clone owns its transform
    assert got[7] is True and got[8] is False and got[9] == 1 and got[10] == 1  # shared geometry, copied userData
    assert got[11:] == ["ZXY", pytest.approx(0.2), 0, True]                     # copy(source, recursive = false)


def test_class_flags_typed_arrays_and_shared_attribute_arrays():
    pre = """
      const m = new THREE.Mesh(new THREE.BoxGeometry(0.1, 0.1, 0.1), new THREE.MeshPhysicalMaterial());
      const im = new THREE.InstancedMesh(new THREE.BoxGeometry(0.1, 0.1, 0.1), new THREE.MeshBasicMaterial(), 2);
      const ls = new THREE.LineSegments(new THREE.BufferGeometry(), new THREE.LineDashedMaterial());
      const u = new Uint8Array([300, -1, 7.9]); const c = new Uint8ClampedArray([300, -5, 2.5]);
      const f = new Float32Array(4); f.set([1, 2], 1); f[9] = 5;
      const pos = new Float32Array([0, 0, 0, 1, 0, 0, 0, 1, 0]);
      const bg = new THREE.BufferGeometry(); bg.setAttribute('position', new THREE.BufferAttribute(pos, 3));
      pos[4] = 2;                                           // written after the attribute was made
      bg.attributes.position.array[6] = 3;                   // written through the attribute's own array
      bg.setIndex([0, 1, 2]); bg.computeVertexNormals();
      let threw = false; try { new THREE.BufferAttribute([0, 0, 0], 3); } catch (e) { threw = true; }
    """
    got = _ev("[m.isMesh, im.isMesh, im.isInstancedMesh, ls.isLine, ls instanceof THREE.Line, m.isGroup, "
              "m.material.isMeshStandardMaterial, ls.material.isLineBasicMaterial, u[0], u[1], u[2], c[0], c[1], c[2], "
              "f.length, f[1], f[9], Array.isArray(f), typeof f.push, new Float32Array([10, 9, 1]).sort().join(','), "
              "bg.attributes.position.getY(1), bg.attributes.position.getX(2), bg.index.count, "
              "bg.getAttribute('normal').getZ(0), threw, Math.fround(0.1) === 0.1]", pre).items
    assert got[:8] == [True, True, True, True, True, UNDEF, True, True]
    assert got[8:14] == [44, 255, 7, 255, 0, 2]            # modular bytes; clamped bytes round half to even
    assert got[14:20] == [4, 1, UNDEF, False, "undefined", "1,9,10"]
    assert got[20:] == [2, 3, 3, -1, True, False]          # (1, 2, 0) x (3, 1, 0) points to -z


def test_colors_live_in_linear_srgb_like_three_js():
    pre = """
      const a = new THREE.Color(0xff8000); const h = {}; a.getHSL(h); const hs = {}; a.getHSL(hs, THREE.SRGBColorSpace);
      const b = new THREE.Color(0.5, 0.5, 0.5); const d = new THREE.Color('#808080');
      const e = new THREE.Color().setRGB(0.5, 0.5, 0.5, THREE.SRGBColorSpace);
      const half = new THREE.Color(0xffffff).multiplyScalar(0.5);
    """
    got = _ev("[a.getHex(), a.r, a.g, h.h, hs.h, b.getHexString(), d.r, e.getHexString(), half.getHexString(), "
              "d.getStyle()]", pre).items
    assert got[0] == 0xFF8000 and got[1] == 1.0 and got[2] == pytest.approx(0.2158605, abs=1e-6)
    assert got[3] == pytest.approx(0.2158605 / 6, abs=1e-6) and got[4] == pytest.approx((128 / 255) / 6, abs=1e-6)
    assert got[5] == "bcbcbc" and got[6] == pytest.approx(0.2158605, abs=1e-6) and got[7] == "808080"
    assert got[8] == "bcbcbc" and got[9] == "rgb(128,128,128)"


def test_bounding_boxes_follow_set_from_object():
    pre = """
      const m = new THREE.Mesh(new THREE.SphereGeometry(0.5, 32, 16), new THREE.MeshBasicMaterial());
      m.rotation.y = Math.PI / 4; g.add(m);
      const loose = new THREE.Box3().setFromObject(g), tight = new THREE.Box3().setFromObject(g, true);
      const hidden = new THREE.Mesh(new THREE.BoxGeometry(4, 0.1, 0.1), new THREE.MeshBasicMaterial());
      hidden.visible = false; const g2 = new THREE.Group(); g2.add(hidden);
      const hb = new THREE.Box3().setFromObject(g2);
      const im = new THREE.InstancedMesh(new THREE.BoxGeometry(0.1, 0.1, 0.1), new THREE.MeshBasicMaterial(), 2);
      im.setMatrixAt(1, new THREE.Matrix4().makeTranslation(1, 0, 0));
      const ib = new THREE.Box3().setFromObject(im);
      const fixed = new THREE.Object3D(); fixed.matrixAutoUpdate = false; fixed.position.set(5, 0, 0);
      fixed.add(new THREE.Mesh(new THREE.BoxGeometry(1, 1, 1), new THREE.MeshBasicMaterial()));
      const fb = new THREE.Box3().setFromObject(fixed);
    """
    got = _ev("[loose.max.x, tight.max.x, hb.max.x, ib.min.x, ib.max.x, fb.max.x]", pre).items
    assert got[0] == pytest.approx(0.5 * 2 ** 0.5, abs=1e-6)        # the box around the rotated box
    assert got[1] == pytest.approx(0.5, abs=1e-3)                    # every vertex
    assert got[2] == pytest.approx(2.0)                               # invisible objects count
    assert got[3:5] == [pytest.approx(-0.05), pytest.approx(1.05)]    # instances: identity until set
    assert got[5] == pytest.approx(0.5)                               # matrixAutoUpdate = false keeps its matrix


def test_curves_space_points_by_arc_length_and_give_tangents():
    pre = """
      const c = new THREE.LineCurve3(new THREE.Vector3(0, 0, 0), new THREE.Vector3(2, 0, 0));
      const q = new THREE.QuadraticBezierCurve3(new THREE.Vector3(0, 0, 0), new THREE.Vector3(1, 2, 0), new THREE.Vector3(3, 0, 0));
      const sp = q.getSpacedPoints(4).map(p => p.x);
    """
    got = _ev("[c.getTangent(0.5).x, c.getLength(), c.getPoints().length, q.getPoints().length, q.getTangentAt(0).y > 0, "
              "q.getPointAt(0.5).x, q.getPoint(0.5).x, sp.length]", pre).items
    assert got[:5] == [pytest.approx(1.0), pytest.approx(2.0), 6, 6, True]       # getPoints(divisions = 5)
    # the arc-length midpoint of this asymmetric arc differs from its parameter midpoint
    assert got[6] == pytest.approx(1.25) and abs(got[5] - got[6]) > 0.01 and got[7] == 5


def test_shapes_sample_their_curves_by_divisions():
    pre = """
      const c = new THREE.Shape(); c.absarc(0, 0, 0.3, 0, Math.PI * 2, false);
      const q = new THREE.Shape(); q.moveTo(0, 0); q.quadraticCurveTo(1, 1, 2, 0); q.closePath();
      const e = new THREE.ExtrudeGeometry(c, {depth: 0.1, bevelEnabled: false, curveSegments: 6});
      const f = new THREE.ShapeGeometry(c, 4);
      const s = new THREE.Shape(); s.moveTo(0, 0); s.lineTo(1, 0); s.lineTo(1, 1); s.closePath();
    """
    got = _ev("[c.getPoints().length, c.getPoints(6).length, q.getPoints().length, q.getPoints(3).length, "
              "e.attributes.position.count, f.attributes.position.count, s.getPoints().length, "
              "s.currentPoint.x, c.extractPoints(2).shape.length]", pre).items
    # a full circle: 2 x divisions + 1 points with the last equal to the first; a quadratic: divisions + 1, closed
    assert got[:4] == [25, 13, 14, 5]
    # extrude: 12 outline points, caps of 12 + sides of 2 rings x 12, non-indexed: 3 per triangle
    assert got[4] == 3 * (2 * 10 + 2 * 12) and got[5] == 8          # flat shape: one vertex per outline point
    assert got[6:] == [4, 0, 5]
