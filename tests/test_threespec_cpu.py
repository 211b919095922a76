"""The checker follows the output specification's name tables (app/threespec.py), and the interpreter implements
every THREE member the specification allows."""
import numpy as np
import pytest

from phung5_b200.app import jsvm, threespec
from phung5_b200.app.jscheck import JSChecker

TAIL = " g.add(new THREE.Mesh(new THREE.BoxGeometry(1, 1, 1), new THREE.MeshStandardMaterial())); return g; }"


def _check(body, **kw):
    return JSChecker(_inline=True).check("export default function generate(THREE) { const g = new THREE.Group(); "
                                         + body + TAIL)


def _rules(body):
    return {f["rule"] for f in _check(body).failures}


def test_every_allowed_member_is_implemented():
    three = jsvm.make_three(jsvm.Interp())
    assert sorted(n for n in threespec.THREE_ALLOWED if n not in three.props) == []


@pytest.mark.parametrize("body,rule", [
    ("const m = new THREE.MeshPhongMaterial();", "FORBIDDEN_THREE_API"),
    ("const m = new THREE.MeshLambertMaterial();", "FORBIDDEN_THREE_API"),
    ("const t = new THREE.CanvasTexture();", "FORBIDDEN_THREE_API"),
    ("const l = new THREE.LineLoop();", "UNKNOWN_THREE_API"),
    ("const r = THREE.MathUtils.seededRandom();", "FORBIDDEN_THREE_API"),
    ("const k = 'sin'; const v = Math[k](1);", "COMPUTED_PROPERTY_ACCESS"),
    ("const o = {}; const p = o.__proto__;", "FORBIDDEN_PROPERTY_ACCESS"),
    ("const d = Date.now();", "FORBIDDEN_IDENTIFIER"),
    ("const f = async () => 1;", "ASYNC_NOT_ALLOWED"),
    ("class A { async m() {} }", "ASYNC_NOT_ALLOWED"),
])
def test_specification_rejections(body, rule):
    assert rule in _rules(body)


def test_console_is_not_a_global_and_its_statements_are_repaired_away():
    off = JSChecker(_inline=True)
    off.s.failure_repair = False
    src = "export default function generate(THREE) { const g = new THREE.Group(); console.log('x', 1);" + TAIL
    assert "IDENTIFIER_NOT_ALLOWED" in {f["rule"] for f in off.check(src).failures}
    res = JSChecker(_inline=True).check(src)
    assert res.ok and "console: console" in res.repaired and "console" not in res.code


def test_spec_globals_json_map_set_and_prototype_access():
    res = _check("""
      const o = JSON.parse(JSON.stringify({a: [1, 2], b: {c: 'x'}}));
      const m = new Map([['k', 2]]); m.set('j', 3);
      const s = new Set([1, 2, 2, 3]);
      let sum = 0; for (const [k, v] of m) sum += v; for (const v of s) sum += v;
      function F() {} F.prototype.w = 5;
      g.userData.v = [o.a[1], o.b.c, m.size, s.size, sum, new F().w, Number.parseInt('12'), JSON.stringify([1, 'a'])];
    """)
    assert res.ok, res.summary()


def _run(body):
    r = jsvm.run_module("export default function generate(THREE) { const g = new THREE.Group(); " + body + TAIL,
                        jsvm.Limits(steps=2_000_000, seconds=10))
    assert r.error is None, r.error
    return r.root.props["userData"].props


def _arr(v):
    return [float(x) for x in v.items]


def test_edges_wireframe_and_polyhedron_geometries():
    ud = _run("""
      const box = new THREE.BoxGeometry(1, 1, 1);
      g.userData.edges = new THREE.EdgesGeometry(box).attributes.position.count;
      g.userData.wire = new THREE.WireframeGeometry(box).attributes.position.count;
      const tet = new THREE.PolyhedronGeometry([1, 1, 1, -1, -1, 1, -1, 1, -1, 1, -1, -1], [2, 1, 0, 0, 3, 2, 1, 3, 0, 2, 3, 1], 2, 1);
      const p = tet.attributes.position;
      g.userData.tet = [p.count, Math.hypot(p.getX(0), p.getY(0), p.getZ(0))];
      g.add(new THREE.LineSegments(new THREE.EdgesGeometry(box), new THREE.LineBasicMaterial()));
    """)
    assert ud["edges"] == 24            # a cube's 12 edges, two points each; the diagonals are flat
    assert ud["wire"] == 36             # 18 distinct triangle edges
    assert _arr(ud["tet"])[0] == 24 and _arr(ud["tet"])[1] == pytest.approx(2.0)


def test_math_helpers_and_curves():
    ud = _run("""
      const sp = new THREE.Spherical().setFromVector3(new THREE.Vector3(1, 2, 3));
      const back = new THREE.Vector3().setFromSpherical(sp);
      g.userData.sph = [back.x, back.y, back.z];
      const cyl = new THREE.Vector3().setFromCylindricalCoords(2, Math.PI / 2, 5);
      g.userData.cyl = [cyl.x, cyl.y, cyl.z];
      const pl = new THREE.Plane().setFromNormalAndCoplanarPoint(new THREE.Vector3(0, 1, 0), new THREE.Vector3(0, 2, 0));
      g.userData.pl = [pl.distanceToPoint(new THREE.Vector3(5, 7, 1))];
      const tri = new THREE.Triangle(new THREE.Vector3(0, 0, 0), new THREE.Vector3(2, 0, 0), new THREE.Vector3(0, 2, 0));
      g.userData.tri = [tri.getArea()];
      const m3 = new THREE.Matrix3().set(2, 0, 0, 0, 3, 0, 0, 0, 4).invert();
      g.userData.m3 = [m3.determinant()];
      const arc = new THREE.EllipseCurve(0, 0, 2, 1, 0, Math.PI, false, 0).getPoints(4);
      g.userData.arc = [arc.length, arc[2].x, arc[2].y, arc[4].x];
      const path = new THREE.CurvePath();
      path.add(new THREE.LineCurve(new THREE.Vector2(0, 0), new THREE.Vector2(1, 0)));
      path.add(new THREE.LineCurve(new THREE.Vector2(1, 0), new THREE.Vector2(1, 1)));
      const mid = path.getPoint(0.75);
      g.userData.path = [mid.x, mid.y];
      class Helix extends THREE.Curve {
        getPoint(t, target = new THREE.Vector3()) { return target.set(Math.cos(6 * t), t, Math.sin(6 * t)); }
      }
      const tube = new THREE.TubeGeometry(new Helix(), 32, 0.05, 6, false);
      g.add(new THREE.Mesh(tube, new THREE.MeshStandardMaterial()));
      const q = new THREE.Quaternion().setFromAxisAngle(new THREE.Vector3(0, 0, 1), Math.PI / 2);
      const v = new THREE.Vector3(1, 0, 0).applyQuaternion(q).addScaledVector(new THREE.Vector3(0, 0, 1), 2);
      g.userData.q = [v.x, v.y, v.z];
    """)
    np.testing.assert_allclose(_arr(ud["sph"]), [1, 2, 3], atol=1e-9)
    np.testing.assert_allclose(_arr(ud["cyl"]), [2, 5, 0], atol=1e-9)
    assert _arr(ud["pl"]) == [5.0] and _arr(ud["tri"]) == [2.0]
    assert _arr(ud["m3"])[0] == pytest.approx(1 / 24)
    np.testing.assert_allclose(_arr(ud["arc"]), [5, 0, 1, -2], atol=1e-9)
    np.testing.assert_allclose(_arr(ud["path"]), [1, 0.5], atol=1e-9)
    np.testing.assert_allclose(_arr(ud["q"]), [0, 1, 2], atol=1e-9)


@pytest.mark.parametrize("pre,body,ok,rule", [
    ("function leg(THREE, h) { return new THREE.Mesh(new THREE.BoxGeometry(0.1, h, 0.1), "
     "new THREE.MeshStandardMaterial()); }\n", "g.add(leg(THREE, 0.5));", True, None),
    ("function leg(T, h) { return new T.Mesh(); }\n", "g.add(leg(THREE, 0.5));", False, "THREE_ALIAS_FORBIDDEN"),
    ("", "const { Mesh, BoxGeometry } = THREE; g.add(new Mesh(new BoxGeometry(0.2, 0.2, 0.2)));", True, None),
    ("", "const make = ({ Mesh, SphereGeometry }) => new Mesh(new SphereGeometry(0.1)); g.add(make(THREE));", True, None),
    ("", "const { ShaderMaterial } = THREE;", False, "FORBIDDEN_THREE_API"),
    ("", "const { MathUtils: { seededRandom } } = THREE;", False, "FORBIDDEN_THREE_API"),
    ("", "const T = THREE;", False, "THREE_ALIAS_FORBIDDEN"),
    ("", "const o = { ...THREE };", False, "THREE_ALIAS_FORBIDDEN"),
    ("", "g.userData.t = [THREE];", False, "THREE_ALIAS_FORBIDDEN"),
    ("", "const m = new THREE.Mesh(THREE);", False, "THREE_ALIAS_FORBIDDEN"),
    ("", "const x = Math.random();", False, "FORBIDDEN_IDENTIFIER"),
])
def test_three_flow_and_math_random(pre, body, ok, rule):
    c = JSChecker(_inline=True)
    c.s.failure_repair = False
    res = c.check(pre + "export default function generate(THREE) { const g = new THREE.Group(); " + body + TAIL)
    assert res.ok == ok, res.summary()
    if rule:
        assert rule in {f["rule"] for f in res.failures}


def test_math_random_is_repaired_with_a_seeded_generator():
    src = ("export default function generate(THREE) { const g = new THREE.Group(); "
           "for (let i = 0; i < 3; i++) { const m = new THREE.Mesh(new THREE.BoxGeometry(0.1, 0.1, 0.1), "
           "new THREE.MeshStandardMaterial()); m.position.x = Math.random() * 0.5 - 0.25; g.add(m); }" + TAIL)
    a, b = JSChecker(_inline=True).check(src), JSChecker(_inline=True).check(src)
    assert a.ok and "random" in a.repaired and "Math.random" not in a.code
    mats = [[c["matrix"] for c in r.scene["object"]["children"]] for r in (a, b)]
    assert mats[0] == mats[1] and len({m[12] for m in mats[0]}) > 1      # deterministic, and the draws differ


@pytest.mark.parametrize("gtype,params,lo,hi", [
    ("SphereGeometry", {"radius": 1.0, "thetaLength": np.pi / 2}, [-1, 0, -1], [1, 1, 1]),          # dome
    ("SphereGeometry", {"radius": 1.0, "phiLength": np.pi}, [-1, -1, 0], [1, 1, 1]),                # half, z >= 0
    ("CylinderGeometry", {"radiusTop": 1.0, "radiusBottom": 1.0, "height": 1.0, "thetaLength": np.pi,
                          "openEnded": True}, [0, -0.5, -1], [1, 0.5, 1]),
    ("ConeGeometry", {"radius": 0.5, "height": 2.0, "thetaStart": np.pi / 2, "thetaLength": np.pi},
     [-0.5, -1, -0.5], [0.5, 1, 0]),
    ("TorusGeometry", {"radius": 1.0, "tube": 0.2, "arc": np.pi}, [-1.2, 0, -0.2], [1.2, 1.2, 0.2]),
    ("IcosahedronGeometry", {"radius": 1.0, "detail": 0.0}, [-0.851] * 3, [0.851] * 3),
])
def test_partial_primitives_follow_their_angle_parameters(gtype, params, lo, hi):
    v, f = jsvm.geometry_mesh(jsvm.Geometry(gtype, params))
    np.testing.assert_allclose(v.min(0).values.numpy(), lo, atol=2e-3)
    np.testing.assert_allclose(v.max(0).values.numpy(), hi, atol=2e-3)
    assert f.shape[0] > 0 and int(f.max()) < v.shape[0]


def _cap_area(v, f):
    import torch
    tri = v[f]
    n = torch.cross(tri[:, 1] - tri[:, 0], tri[:, 2] - tri[:, 0], dim=1)
    top = tri[:, :, 2].min(1).values > float(v[:, 2].max()) - 1e-6
    return float(n[top].norm(dim=1).sum() / 2)


def test_extrude_holes_and_default_bevel():
    r = jsvm.run_module("""export default function generate(THREE) {
      const g = new THREE.Group();
      const s = new THREE.Shape(); s.moveTo(-1, -1); s.lineTo(1, -1); s.lineTo(1, 1); s.lineTo(-1, 1); s.lineTo(-1, -1);
      const h = new THREE.Path(); h.absellipse(0, 0, 0.5, 0.5, 0, Math.PI * 2, false, 0); s.holes.push(h);
      g.userData.n = s.holes.length;
      g.add(new THREE.Mesh(new THREE.ExtrudeGeometry(s)));                                   // three.js's defaults
      g.add(new THREE.Mesh(new THREE.ExtrudeGeometry(s, { depth: 0.5, bevelEnabled: false })));
      g.add(new THREE.Mesh(new THREE.ShapeGeometry(s)));
      return g; }""", jsvm.Limits(steps=2_000_000, seconds=10))
    assert r.error is None, r.error
    meshes = r.root.props["children"].items
    bev, flat_ext, flat = (jsvm.geometry_mesh(m.props["geometry"]) for m in meshes)
    # the default bevel: 0.1 wider in x / y, 0.2 thicker on both sides of the unit depth
    np.testing.assert_allclose(bev[0].min(0).values.numpy(), [-1.1, -1.1, -0.2], atol=1e-5)
    np.testing.assert_allclose(bev[0].max(0).values.numpy(), [1.1, 1.1, 1.2], atol=1e-5)
    np.testing.assert_allclose(flat_ext[0].max(0).values.numpy(), [1, 1, 0.5], atol=1e-6)
    hole = np.pi * 0.25
    for v, f in (bev, flat_ext, flat):
        assert _cap_area(v, f) == pytest.approx(4 - hole, rel=0.01)      # the hole is cut out of both caps
    assert float(r.root.props["userData"].props["n"]) == 1


def test_vertex_counts_follow_three_js():
    from phung5_b200.app.jscheck import declared_vertices
    G = jsvm.Geometry
    assert declared_vertices(G("ConeGeometry", {"radius": 1.0})) == 33 * 2 + 65          # one cap
    assert declared_vertices(G("CylinderGeometry", {"openEnded": True})) == 33 * 2       # no caps
    assert declared_vertices(G("CylinderGeometry", {})) == 33 * 2 + 2 * 65
    assert declared_vertices(G("IcosahedronGeometry", {"detail": 2.0})) == 60 * 9        # non-indexed
    c = JSChecker(_inline=True)
    src = ("export default function generate(THREE) { const g = new THREE.Group(); g.add(new THREE.Mesh("
           "new THREE.IcosahedronGeometry(0.5, %d), new THREE.MeshStandardMaterial())); return g; }")
    assert c.check(src % 60).ok                                    # 223,260 vertices
    assert "VERTEX_LIMIT_EXCEEDED" in {f["rule"] for f in c.check(src % 70).failures}   # 302,460


def test_material_arrays_follow_geometry_groups_and_vertex_colours_render():
    import torch

    from phung5_b200.render import scene as S
    src = """export default function generate(THREE) { const g = new THREE.Group();
      const cols = [0xff0000, 0x00ff00, 0x0000ff, 0xffff00, 0xff00ff, 0x00ffff];
      g.add(new THREE.Mesh(new THREE.BoxGeometry(0.5, 0.5, 0.5), cols.map(c => new THREE.MeshStandardMaterial({color: c}))));
      const q = new THREE.BufferGeometry();
      q.setAttribute('position', new THREE.Float32BufferAttribute([0, 0, 0.3, 0.2, 0, 0.3, 0, 0.2, 0.3,
                                                                   0, 0, 0.4, 0.2, 0, 0.4, 0, 0.2, 0.4], 3));
      q.setAttribute('color', new THREE.Float32BufferAttribute([0, 1, 0, 0, 1, 0, 0, 1, 0, 0, 0, 1, 0, 0, 1, 0, 0, 1], 3));
      q.addGroup(0, 3, 1); q.addGroup(3, 3, 0);
      g.add(new THREE.Mesh(q, [new THREE.MeshBasicMaterial({vertexColors: true}), new THREE.MeshBasicMaterial({color: 0xff0000})]));
      return g; }"""
    res = JSChecker(_inline=True).check(src)
    assert res.ok, res.summary()
    t, col = S.scene_triangles(res.scene)
    n = torch.linalg.cross(t[:, 1] - t[:, 0], t[:, 2] - t[:, 0])
    c = t.mean(1)
    px = (n[:, 0].abs() > 1e-6) & (c[:, 0] > 0.2)
    ny = (n[:, 1].abs() > 1e-6) & (c[:, 1] < -0.2)
    assert torch.allclose(col[px], torch.tensor([1.0, 0.0, 0.0]))         # group 0: +x
    assert torch.allclose(col[ny], torch.tensor([1.0, 1.0, 0.0]))         # group 3: -y
    z3 = (c[:, 2] - 0.3).abs() < 1e-6
    z4 = (c[:, 2] - 0.4).abs() < 1e-6
    assert torch.allclose(col[z3], torch.tensor([1.0, 0.0, 0.0]))         # group -> material 1 (plain red)
    assert torch.allclose(col[z4], torch.tensor([0.0, 0.0, 1.0]))         # material 0: its vertex colours


def test_data_texture_tints_the_render_by_its_mean_colour():
    from phung5_b200.render import scene as S
    src = """export default function generate(THREE) { const g = new THREE.Group();
      const n = 4; const data = new Uint8Array(n * n * 4);
      for (let i = 0; i < n * n; i++) { data[4 * i] = i % 2 ? 255 : 0; data[4 * i + 1] = 128; data[4 * i + 3] = 255; }
      const t = new THREE.DataTexture(data, n, n, THREE.RGBAFormat);          // NoColorSpace: texels are linear
      g.add(new THREE.Mesh(new THREE.BoxGeometry(0.5, 0.5, 0.5), new THREE.MeshStandardMaterial({map: t, color: 0xffffff})));
      return g; }"""
    res = JSChecker(_inline=True).check(src)
    assert res.ok, res.summary()
    _, col = S.scene_triangles(res.scene)
    np.testing.assert_allclose(col[0].numpy(), [0.5, 128 / 255, 0.0], atol=1e-4)


def test_post_validation_counts_like_the_reference_validator():
    # an InstancedMesh draws its geometry once: vertices are counted once, instances separately
    res = _check("const im = new THREE.InstancedMesh(new THREE.SphereGeometry(0.01, 64, 32), "
                 "new THREE.MeshStandardMaterial(), 400); g.add(im);")
    assert res.ok, res.summary()
    # DataTextures count by byteLength, once each, from the map slots only
    tex = ("const data = new Float32Array(512 * 512 * 4); const t = new THREE.DataTexture(data, 512, 512, "
           "THREE.RGBAFormat, THREE.FloatType); ")
    res = _check(tex + "g.add(new THREE.Mesh(new THREE.BoxGeometry(0.1, 0.1, 0.1), new THREE.MeshStandardMaterial({map: t})));")
    assert "TEXTURE_DATA_EXCEEDED" not in {f["rule"] for f in res.failures}
    assert res.stats["textureBytes"] == 512 * 512 * 16
    res = _check(tex + "const t2 = new THREE.DataTexture(new Float32Array(4), 1, 1); "
                       "const mat = new THREE.MeshStandardMaterial({map: t, roughnessMap: t2}); "
                       "g.add(new THREE.Mesh(new THREE.BoxGeometry(0.1, 0.1, 0.1), mat)); "
                       "g.add(new THREE.Mesh(new THREE.BoxGeometry(0.1, 0.1, 0.1), mat)); "
                       "g.add(new THREE.Mesh(new THREE.BoxGeometry(0.1, 0.1, 0.1), new THREE.MeshStandardMaterial({map: t})));")
    assert res.stats["textureBytes"] == 512 * 512 * 16 + 16
    res = _check(tex + "const t2 = new THREE.DataTexture(new Float32Array(512 * 512 * 4), 512, 512); "
                       "g.add(new THREE.Mesh(new THREE.BoxGeometry(0.1, 0.1, 0.1), "
                       "new THREE.MeshStandardMaterial({map: t, emissiveMap: t2})));")
    assert "TEXTURE_DATA_EXCEEDED" in {f["rule"] for f in res.failures}
    # only a Group, Mesh, LineSegments or Points may be returned
    res = JSChecker(_inline=True).check("export default function generate(THREE) { const o = new THREE.Object3D(); "
                                        "o.add(new THREE.Mesh(new THREE.BoxGeometry(0.1, 0.1, 0.1), "
                                        "new THREE.MeshBasicMaterial())); return o; }")
    assert [f["rule"] for f in res.failures] == ["INVALID_RETURN_TYPE"]


def test_instance_colours_multiply_the_material_colour():
    src = """export default function generate(THREE) { const g = new THREE.Group();
      const im = new THREE.InstancedMesh(new THREE.BoxGeometry(0.1, 0.1, 0.1), new THREE.MeshStandardMaterial({color: 0xffffff}), 3);
      const d = new THREE.Object3D();
      for (let i = 0; i < 3; i++) { d.position.set(0.2 * i - 0.2, 0, 0); d.updateMatrix(); im.setMatrixAt(i, d.matrix); }
      im.setColorAt(0, new THREE.Color(0xff0000)); im.setColorAt(2, new THREE.Color(0x00ff00));
      im.instanceMatrix.needsUpdate = true; im.instanceColor.needsUpdate = true;
      const c = new THREE.Color(); im.getColorAt(2, c); g.userData.c = c.getHex();
      g.add(im); return g; }"""
    res = JSChecker(_inline=True).check(src)
    assert res.ok, res.summary()
    mats = {m["uuid"]: m for m in res.scene["materials"]}
    kids = res.scene["object"]["children"][0]["children"]
    assert [mats[k["material"]]["color"] for k in kids] == [0xFF0000, 0xFFFFFF, 0x00FF00]
