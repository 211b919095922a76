"""Scene JSON -> triangles -> rasterizer (CPU restatement): geometry, camera and shading sanity."""
import torch

from phung5_b200.render.scene import normalise, render, render_views, scene_triangles, view_projection

SCENE = {"geometries": [{"uuid": "g1", "type": "BoxGeometry", "w": 1, "h": 1, "d": 1},
                        {"uuid": "g2", "type": "SphereGeometry", "radius": 0.5}],
         "materials": [{"uuid": "m1", "color": 0xFF0000}, {"uuid": "m2", "color": 0x00FF00}],
         "object": {"matrix": [1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1],
                    "children": [{"geometry": "g1", "material": "m1"},
                                 {"geometry": "g2", "material": "m2",
                                  "matrix": [1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1, 0, 1.5, 0, 0, 1]}]}}


def test_scene_triangles_and_transform():
    tris, cols = scene_triangles(SCENE)
    assert tris.shape[1:] == (3, 3) and cols.shape == (tris.shape[0], 3)
    assert 12 < tris.shape[0]
    # the sphere is translated by +1.5 on x
    assert tris[12:, :, 0].mean() > 1.0


def test_render_front_view_colours():
    tris, cols = scene_triangles(SCENE)
    img = render(normalise(tris), cols, view_projection(0, 0), 128)
    assert img.shape == (128, 128, 4) and img.dtype == torch.uint8
    bg = img[0, 0, :3]
    assert (bg == 255).all()                         # white background
    red = ((img[..., 0] > 100) & (img[..., 1] < 60)).sum().item()
    green = ((img[..., 1] > 100) & (img[..., 0] < 60)).sum().item()
    assert red > 300 and green > 300                 # both objects visible and shaded


def test_depth_order_nearer_wins():
    # two parallel quads, the nearer (z = 0.5) red, the farther blue; camera on +z looks at them
    quad = lambda z: torch.tensor([[[-0.5, -0.5, z], [0.5, -0.5, z], [0.5, 0.5, z]],
                                   [[-0.5, -0.5, z], [0.5, 0.5, z], [-0.5, 0.5, z]]])
    tris = torch.cat([quad(-0.2), quad(0.3)])
    cols = torch.tensor([[0, 0, 1.0]] * 2 + [[1.0, 0, 0]] * 2)
    img = render(tris, cols, view_projection(0, 0), 64)
    c = img[32, 32]
    assert c[0] > 150 and c[2] < 50


def test_views():
    imgs = render_views(SCENE, "front4", size=64)
    assert len(imgs) == 4 and all(i.shape == (64, 64, 4) for i in imgs)


def _sphere(metal, rough, col=0xCC8844):
    return {"geometries": [{"uuid": "s", "type": "SphereGeometry", "radius": 0.5, "widthSegments": 48,
                            "heightSegments": 24}],
            "materials": [{"uuid": "m", "type": "MeshStandardMaterial", "color": col, "roughness": rough,
                           "metalness": metal}],
            "object": {"children": [{"geometry": "s", "material": "m"}]}}


def test_standard_material_shading_responds_to_material_and_lights():
    from phung5_b200.render.scene import render_pbr
    out = {}
    for name, (metal, rough) in {"rough": (0.0, 1.0), "glossy": (0.0, 0.2), "metal": (1.0, 0.3)}.items():
        tris, cols, mats = scene_triangles(_sphere(metal, rough), with_materials=True)
        assert mats.shape == (tris.shape[0], 2) and float(mats[0, 1]) == metal
        out[name] = {rig: render_pbr(normalise(tris), cols, mats, 0, 10, 96, rig, background=(0, 0, 0)).float()
                     for rig in ("studio", "neutral", "follow")}
    for rig in ("studio", "neutral", "follow"):
        img = out["rough"][rig]
        assert (img[0, 0, :3] == 0).all()                                 # background
        assert img[48, 48, :3].max() < 250                                # lit, not blown out
    # a glossy surface has a highlight the rough one lacks; a metal takes its albedo's colour in reflections
    assert out["glossy"]["studio"][..., :3].amax() > out["rough"]["studio"][..., :3].amax()
    assert (out["metal"]["studio"] - out["rough"]["studio"]).abs().mean() > 3
    # hemisphere environment: the top of the sphere (sky side) is brighter than the bottom (ground side)
    img = out["rough"]["neutral"]
    top, bottom = img[26:32, 44:52, :3].mean(), img[64:70, 44:52, :3].mean()
    assert top > bottom + 5, (top, bottom)
    # camera-follow lighting: the view-facing centre is the brightest part of a rough sphere from any side
    tris, cols, mats = scene_triangles(_sphere(0.0, 1.0), with_materials=True)
    for az in (0, 90, 200):
        img = render_pbr(normalise(tris), cols, mats, az, 0, 96, "follow", background=(0, 0, 0)).float()[..., :3].mean(-1)
        ring = img[30:66, 30:66]
        assert img[44:52, 44:52].mean() >= ring[ring > 0].mean()


def test_jsvm_exports_standard_material_parameters():
    from phung5_b200.app import jsvm
    r = jsvm.run_module("""export default function generate(THREE) {
      return new THREE.Mesh(new THREE.BoxGeometry(1, 1, 1),
                            new THREE.MeshStandardMaterial({ color: 0x336699, roughness: 0.25, metalness: 0.8 }));
    }""")
    sc = jsvm.to_scene_json(r.root)
    m = sc["materials"][0]
    assert m["roughness"] == 0.25 and m["metalness"] == 0.8
    _, _, mats = scene_triangles(sc, with_materials=True)
    assert torch.allclose(mats[0], torch.tensor([0.25, 0.8]))
