"""Context-aware repair of unknown three.js constants (app/threefix.py) and its place in the checker."""
import numpy as np

from phung5_b200.app import threefix
from phung5_b200.app.jscheck import CheckerSettings, JSChecker

MODULE = """export default function generate(THREE) {
  const g = new THREE.Group();
  const data = new Uint8Array(4 * 4 * 4);
  const tex = new THREE.DataTexture(data, 4, 4, THREE.RGBA8, THREE.UnsignedByteTypeFormat);
  tex.wrapS = THREE.RepeatWrap;
  tex.wrapT = THREE.RepeatWrap;
  tex.minFilter = THREE.LinearMipMapLinear;
  tex.colorSpace = THREE.sRGBEncoding;
  const geo = new THREE.BufferGeometry();
  const pos = new THREE.Float32BufferAttribute([-0.5, -0.5, 0, 0.5, -0.5, 0, 0, 0.5, 0], 3);
  pos.setUsage(THREE.DynamicDraw);
  geo.setAttribute("position", pos);
  const mat = new THREE.MeshStandardMaterial({ color: 0x884422, map: tex, side: THREE.BothSides,
                                               blending: THREE.Normal });
  g.add(new THREE.Mesh(geo, mat));
  return g;
}
"""


def _inline(**kw):
    s = CheckerSettings()
    for k, v in kw.items():
        setattr(s, k, v)
    return JSChecker(s, _inline=True)


def test_rewrite_picks_each_constant_from_its_context():
    names = ["RGBA8", "UnsignedByteTypeFormat", "RepeatWrap", "LinearMipMapLinear", "sRGBEncoding", "DynamicDraw",
             "BothSides", "Normal"]
    code, fixes = threefix.rewrite(MODULE, names)
    assert "THREE.DataTexture(data, 4, 4, THREE.RGBAFormat, THREE.UnsignedByteType)" in code
    assert code.count("THREE.RepeatWrapping") == 2
    assert "tex.minFilter = THREE.LinearMipmapLinearFilter" in code
    assert "tex.colorSpace = THREE.SRGBColorSpace" in code
    assert "setUsage(THREE.DynamicDrawUsage)" in code
    assert "side: THREE.DoubleSide" in code
    # `Normal` alone would be ambiguous; the `blending:` key makes it NormalBlending
    assert "blending: THREE.NormalBlending" in code
    assert any("(filter)" in f for f in fixes) and any("(blending)" in f for f in fixes)


def test_checker_repairs_a_draft_that_only_misnames_constants():
    off = _inline(constant_repair=False).check(MODULE)
    assert not off.ok and {f["rule"] for f in off.failures} == {"UNKNOWN_THREE_API"}
    on = _inline().check(MODULE)
    assert on.ok, on.summary()
    assert any("RepeatWrap -> THREE.RepeatWrapping" in f for f in on.repaired)
    assert "THREE.RepeatWrap;" not in on.code and on.scene is not None


def test_no_rewrite_when_another_rule_fails_or_the_name_is_a_class():
    # another failure besides the unknown constant: the plan refuses
    fails = [{"rule": "UNKNOWN_THREE_API", "detail": "THREE.RepeatWrap is not a supported three.js member"},
             {"rule": "FORBIDDEN_IDENTIFIER", "detail": "`eval` is not allowed"}]
    assert threefix.plan(fails) is None
    # constructor, call and member-chain uses are never rewritten
    assert threefix.rewrite("const m = new THREE.MeshStandardMat();", ["MeshStandardMat"]) is None
    assert threefix.rewrite("const v = THREE.Vec3(1, 2, 3);", ["Vec3"]) is None
    assert threefix.rewrite("const d = THREE.MathUtil.degToRad(3);", ["MathUtil"]) is None
    # no context and no word in common with any constant: left alone
    assert threefix.rewrite("const q = THREE.Banana;", ["Banana"]) is None
    src = MODULE.replace("THREE.RepeatWrap;\n  tex.wrapT", "THREE.RepeatWrap;\n  eval('1');\n  tex.wrapT")
    res = _inline().check(src)
    assert not res.ok and not any("->" in f and "RepeatWrap" in f for f in res.repaired)


def test_three_namespace_parameter_name_is_followed():
    src = MODULE.replace("generate(THREE)", "generate(T)").replace("THREE.", "T.")
    res = _inline().check(src)
    assert res.ok, res.summary()
    assert "T.RepeatWrapping" in res.code


def _user_data(root):
    m = root.props["children"].items[0]
    return {k: float(v) for k, v in m.props["userData"].props.items()}


def _run(src):
    from phung5_b200.app import jsvm
    r = jsvm.run_module(src, jsvm.Limits(steps=2_000_000, seconds=10))
    assert r.error is None, r.error
    return jsvm, r


def test_primitive_vertex_edits_are_baked_and_serialised():
    # the usual terrain idiom: displace a segmented plane's vertices through its position attribute
    jsvm, r = _run("""export default function generate(THREE) {
      const geo = new THREE.PlaneGeometry(2, 2, 4, 4);
      const p = geo.attributes.position;
      for (let i = 0; i < p.count; i++) p.setZ(i, 0.25 * p.getX(i));
      p.needsUpdate = true;
      geo.computeVertexNormals();
      const g = new THREE.Group();
      const m = new THREE.Mesh(geo, new THREE.MeshStandardMaterial());
      m.userData.count = p.count;
      m.userData.uvs = geo.getAttribute("uv").count;
      m.userData.tris = geo.index.count / 3;
      g.add(m);
      return g;
    }""")
    scene = jsvm.to_scene_json(r.root)
    mesh = scene["object"]["children"][0]
    assert _user_data(r.root) == {"count": 25, "uvs": 25, "tris": 32}
    geo = next(x for x in scene["geometries"] if x["uuid"] == mesh["geometry"])
    pos = np.asarray(geo["data"]["attributes"]["position"]["array"], dtype=np.float32).reshape(-1, 3)
    assert pos.shape == (25, 3)
    np.testing.assert_allclose(pos[:, 2], 0.25 * pos[:, 0], atol=1e-6)      # the edit reached the scene
    assert pos[:, 0].min() == -1 and pos[:, 1].max() == 1                   # top-left vertex first


def test_buffer_transforms_apply_to_the_vertices_at_once():
    jsvm, r = _run("""export default function generate(THREE) {
      const geo = new THREE.BufferGeometry();
      geo.setAttribute("position", new THREE.Float32BufferAttribute([0, 0, 0, 1, 0, 0, 0, 1, 0], 3));
      geo.translate(0, 2, 0);
      const box = new THREE.BoxGeometry(1, 1, 1);
      box.translate(3, 0, 0);                     // parametric: kept as a transform until baked
      const bx = box.attributes.position.getX(0); // bake: the translation is in the vertices now
      box.scale(2, 2, 2);                         // baked: moves the vertices
      const m = new THREE.Mesh(geo, new THREE.MeshBasicMaterial());
      m.userData.y = geo.attributes.position.getY(0);
      m.userData.bx = bx;
      m.userData.bx2 = box.attributes.position.getX(0);
      const g = new THREE.Group();
      g.add(m);
      g.add(new THREE.Mesh(box, new THREE.MeshBasicMaterial()));
      return g;
    }""")
    ud = _user_data(r.root)
    assert ud["y"] == 2
    assert ud["bx"] in (2.5, 3.5) and ud["bx2"] == 2 * ud["bx"]
