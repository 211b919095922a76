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
