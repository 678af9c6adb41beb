"""The callers on either side of the path (CPU): COLMAP ingestion without pycolmap, the point-cloud
initialisation of the model, and checkpoints in the reference's format.

* A synthetic reconstruction written in COLMAP's binary and text formats loads into the same
  cameras (poses, rescaled intrinsics, name order, test split), point cloud and extent, matching
  values computed here from the written records; unsupported camera models and images whose aspect
  ratio disagrees with their camera are rejected as in the reference (utils/dataset.py:66-92).
* init_from_point_cloud equals the reference's GaussianModel.__init__ on the same cloud
  (tests/golden/model_init.npz, written by tests/golden/make_golden.py from the reference).
* Checkpoints round-trip, and a file in the reference's save_checkpoint layout (main.py:77-94) loads
  under this package's parameter names.
"""
import struct

import numpy as np
import pytest
import torch

from hds_b200 import checkpoint, colmap

MODELS = {"SIMPLE_PINHOLE": 0, "PINHOLE": 1, "OPENCV": 4}


def random_pose(rng):
    q = rng.standard_normal(4)
    q /= np.linalg.norm(q)
    return q, rng.standard_normal(3)


def make_scene(root, fmt, rng, model="PINHOLE", bad_aspect=False):
    """Writes <root>/sparse/0 (binary or text) and <root>/images: 2 cameras, 9 images, 40 points."""
    from PIL import Image

    sparse = root / "sparse" / "0"
    sparse.mkdir(parents=True)
    (root / "images").mkdir()
    cams = {1: (model, 80, 60, [70.0, 72.0, 40.0, 30.0] if model == "PINHOLE" else
                ([65.0, 40.0, 30.0] if model == "SIMPLE_PINHOLE" else [70.0, 72.0, 40.0, 30.0, 0, 0, 0, 0])),
            2: ("SIMPLE_PINHOLE", 120, 90, [100.0, 60.0, 45.0])}
    images = {}
    for k, name in enumerate(["f.png", "a.png", "c.png", "i.png", "b.png", "e.png", "d.png", "h.png", "g.png"]):
        q, t = random_pose(rng)
        cam_id = 1 if k % 2 == 0 else 2
        images[10 + k] = (q, t, cam_id, name)
        w, h = cams[cam_id][1] * 2, cams[cam_id][2] * 2  # files stored at twice the SfM resolution
        if bad_aspect and k == 0:
            h += 20
        Image.fromarray(rng.integers(0, 256, (h, w, 3), dtype=np.uint8)).save(root / "images" / name)
    points = {100 + i: (rng.standard_normal(3) * 2, rng.integers(0, 256, 3)) for i in range(40)}
    if fmt == "bin":
        with open(sparse / "cameras.bin", "wb") as f:
            f.write(struct.pack("<Q", len(cams)))
            for cid, (m, w, h, params) in cams.items():
                f.write(struct.pack("<iiQQ", cid, MODELS[m], w, h) + struct.pack(f"<{len(params)}d", *params))
        with open(sparse / "images.bin", "wb") as f:
            f.write(struct.pack("<Q", len(images)))
            for iid, (q, t, cid, name) in images.items():
                f.write(struct.pack("<I7dI", iid, *q, *t, cid) + name.encode() + b"\x00")
                f.write(struct.pack("<Q", 2) + struct.pack("<ddq", 1.0, 2.0, 100) + struct.pack("<ddq", 3.0, 4.0, -1))
        with open(sparse / "points3D.bin", "wb") as f:
            f.write(struct.pack("<Q", len(points)))
            for pid, (xyz, rgb) in points.items():
                f.write(struct.pack("<Q3d3BdQ", pid, *xyz, *[int(c) for c in rgb], 0.5, 1) + struct.pack("<II", 10, 0))
    else:
        with open(sparse / "cameras.txt", "w") as f:
            f.write("# Camera list\n")
            for cid, (m, w, h, params) in cams.items():
                f.write(f"{cid} {m} {w} {h} " + " ".join(repr(p) for p in params) + "\n")
        with open(sparse / "images.txt", "w") as f:
            f.write("# Image list\n")
            for iid, (q, t, cid, name) in images.items():
                f.write(f"{iid} " + " ".join(repr(float(x)) for x in (*q, *t)) + f" {cid} {name}\n")
                f.write("1.0 2.0 100 3.0 4.0 -1\n")
        with open(sparse / "points3D.txt", "w") as f:
            f.write("# 3D point list\n")
            for pid, (xyz, rgb) in points.items():
                f.write(f"{pid} " + " ".join(repr(float(x)) for x in xyz) + " " + " ".join(str(int(c)) for c in rgb)
                        + " 0.5 10 0\n")
    return cams, images, points


@pytest.mark.parametrize("fmt", ["bin", "txt"])
def test_colmap_scene_loads_like_the_reference(tmp_path, fmt):
    rng = np.random.default_rng(0)
    cams, images, points = make_scene(tmp_path, fmt, rng)
    ds = colmap.ColmapDataset(tmp_path, max_width=150, test_every=4, device="cpu")
    names = sorted(v[3] for v in images.values())
    assert [c.name for c in ds.test_cameras] == names[::4]
    assert [c.name for c in ds.train_cameras] == [n for i, n in enumerate(names) if i % 4]
    by_name = {v[3]: (iid, v) for iid, v in images.items()}
    for cam in ds.train_cameras + ds.test_cameras:
        iid, (q, t, cid, _) = by_name[cam.name]
        model, w0, h0, params = cams[cid]
        fx, fy, cx, cy = (params[0], params[0], params[1], params[2]) if model == "SIMPLE_PINHOLE" else params[:4]
        width = min(2 * w0, 150)
        height = round(2 * h0 * width / (2 * w0))
        sx, sy = width / w0, height / h0
        assert cam.image_id == iid and (cam.width, cam.height) == (width, height)
        assert cam.image.shape == (height, width, 3) and cam.image.dtype == torch.uint8
        np.testing.assert_allclose([cam.fx, cam.fy, cam.cx, cam.cy], [fx * sx, fy * sy, cx * sx, cy * sy], rtol=1e-12)
        R = colmap.qvec_to_rotmat(q)
        np.testing.assert_allclose(cam.world_to_camera[:3, :3].numpy(), R, atol=1e-6)
        np.testing.assert_allclose(cam.world_to_camera[:3, 3].numpy(), t, atol=1e-6)
        np.testing.assert_allclose(cam.center.numpy(), -R.T @ t, atol=1e-5)
    pts = np.array([p[0] for p in points.values()], np.float32)
    cols = np.array([p[1] for p in points.values()], np.float32) / 255.0
    np.testing.assert_array_equal(ds.point_cloud.points, pts)
    np.testing.assert_array_equal(ds.point_cloud.colors, cols)
    centers = torch.stack([c.center for c in ds.train_cameras])
    assert ds.extent == pytest.approx(1.1 * (centers - centers.mean(0)).norm(dim=1).max().item())


def test_binary_and_text_agree(tmp_path):
    loaded = []
    for fmt in ("bin", "txt"):
        make_scene(tmp_path / fmt, fmt, np.random.default_rng(5))
        loaded.append(colmap.ColmapDataset(tmp_path / fmt, max_width=None, device="cpu"))
    a, b = loaded
    for ca, cb in zip(a.train_cameras + a.test_cameras, b.train_cameras + b.test_cameras):
        assert ca.name == cb.name and torch.allclose(ca.world_to_camera, cb.world_to_camera)
        assert (ca.fx, ca.fy, ca.cx, ca.cy, ca.width, ca.height) == (cb.fx, cb.fy, cb.cx, cb.cy, cb.width, cb.height)
    np.testing.assert_array_equal(a.point_cloud.points, b.point_cloud.points)


def test_unsupported_model_and_aspect_are_rejected(tmp_path):
    make_scene(tmp_path / "distorted", "bin", np.random.default_rng(1), model="OPENCV")
    with pytest.raises(ValueError, match="undistort the scene first"):
        colmap.ColmapDataset(tmp_path / "distorted", device="cpu")
    make_scene(tmp_path / "aspect", "txt", np.random.default_rng(2), bad_aspect=True)
    with pytest.raises(ValueError, match="aspect ratio"):
        colmap.ColmapDataset(tmp_path / "aspect", device="cpu")


def test_point_cloud_initialisation_matches_the_reference(golden):
    g = golden("model_init.npz")
    params = colmap.init_from_point_cloud(colmap.PointCloud(g["points"], g["colors"]))
    names = {"means": "means", "log_scales": "scales", "quats": "quats", "opacity_logits": "opacities",
             "sh_dc": "sh_dc", "sh_rest": "sh_rest"}
    for ours, ref in names.items():
        np.testing.assert_allclose(params[ours].numpy(), g[f"param_{ref}"], rtol=1e-6, atol=1e-7, err_msg=ours)


def test_checkpoint_round_trip_and_reference_layout(tmp_path):
    rng = np.random.default_rng(3)
    n = 50
    params = {"means": torch.randn(n, 3), "log_scales": torch.randn(n, 3), "quats": torch.randn(n, 4),
              "opacity_logits": torch.randn(n, 1), "sh_dc": torch.randn(n, 1, 3), "sh_rest": torch.randn(n, 15, 3)}
    path = checkpoint.save_checkpoint(tmp_path / "run", params, active_sh_degree=2, iteration=700, test_psnr=21.5)
    back = checkpoint.load_checkpoint(tmp_path / "run")
    assert back["active_sh_degree"] == 2 and back["iteration"] == 700 and back["test_psnr"] == 21.5
    for k, v in params.items():
        assert torch.equal(back["params"][k], v)
    # The reference's own layout: main.py's save_checkpoint writes these keys and names.
    ref = {"params": {"means": params["means"], "scales": params["log_scales"], "quats": params["quats"],
                      "opacities": params["opacity_logits"], "sh_dc": params["sh_dc"], "sh_rest": params["sh_rest"]},
           "active_sh_degree": 3, "iteration": 30000, "test_psnr": float(rng.random())}
    torch.save(ref, tmp_path / "model.pt")
    got = checkpoint.load_checkpoint(tmp_path / "model.pt")
    assert torch.equal(got["params"]["log_scales"], params["log_scales"])
    assert torch.equal(got["params"]["opacity_logits"], params["opacity_logits"])
    assert path.name == "model.pt"
    bad = dict(ref, params={k: v for k, v in ref["params"].items() if k != "quats"})
    torch.save(bad, tmp_path / "bad.pt")
    with pytest.raises(ValueError, match="missing"):
        checkpoint.load_checkpoint(tmp_path / "bad.pt")
