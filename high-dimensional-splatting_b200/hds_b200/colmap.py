"""COLMAP scene ingestion without pycolmap: the reference's ColmapDataset (utils/dataset.py) and the
point-cloud initialisation of its GaussianModel (utils/gaussian.py:22-60).

The reference reads <root>/sparse/0 through pycolmap.Reconstruction, which is not installed here.
This module parses COLMAP's own reconstruction files -- cameras, images and points3D, in the binary
(.bin) or text (.txt) form, as COLMAP documents them -- and builds the same objects: cameras sorted
by image name with every test_every-th held out, intrinsics rescaled to the loaded image size
(images wider than max_width downscaled), world_to_camera from the image's cam_from_world pose, the
point cloud with colours in [0, 1], and the scene extent.  Only undistorted pinhole models are
accepted, as in the reference.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

# COLMAP camera model ids and their parameter counts (COLMAP's src/colmap/sensor/models.h).
CAMERA_MODELS = {0: ("SIMPLE_PINHOLE", 3), 1: ("PINHOLE", 4), 2: ("SIMPLE_RADIAL", 4), 3: ("RADIAL", 5),
                 4: ("OPENCV", 8), 5: ("OPENCV_FISHEYE", 8), 6: ("FULL_OPENCV", 12), 7: ("FOV", 5),
                 8: ("SIMPLE_RADIAL_FISHEYE", 4), 9: ("RADIAL_FISHEYE", 5), 10: ("THIN_PRISM_FISHEYE", 12)}
MODEL_IDS = {name: (i, n) for i, (name, n) in CAMERA_MODELS.items()}


@dataclass
class ColmapCamera:
    camera_id: int
    model: str
    width: int
    height: int
    params: np.ndarray  # float64, the model's parameter vector


@dataclass
class ColmapImage:
    image_id: int
    qvec: np.ndarray  # (w, x, y, z): rotation of cam_from_world
    tvec: np.ndarray  # translation of cam_from_world
    camera_id: int
    name: str


@dataclass
class ColmapPoint:
    point_id: int
    xyz: np.ndarray
    rgb: np.ndarray  # uint8


def _read(f, fmt):
    size = struct.calcsize(fmt)
    data = f.read(size)
    if len(data) != size:
        raise ValueError("truncated COLMAP file")
    return struct.unpack(fmt, data)


def read_cameras_binary(path) -> dict[int, ColmapCamera]:
    cams = {}
    with open(path, "rb") as f:
        (count,) = _read(f, "<Q")
        for _ in range(count):
            cam_id, model_id, width, height = _read(f, "<iiQQ")
            name, n = CAMERA_MODELS[model_id]
            params = np.array(_read(f, f"<{n}d"), dtype=np.float64)
            cams[cam_id] = ColmapCamera(cam_id, name, int(width), int(height), params)
    return cams


def read_images_binary(path) -> dict[int, ColmapImage]:
    images = {}
    with open(path, "rb") as f:
        (count,) = _read(f, "<Q")
        for _ in range(count):
            image_id, qw, qx, qy, qz, tx, ty, tz, cam_id = _read(f, "<I7dI")
            name = bytearray()
            while True:
                ch = f.read(1)
                if ch in (b"\x00", b""):
                    break
                name += ch
            (n2d,) = _read(f, "<Q")
            f.seek(24 * n2d, 1)  # x, y (double), point3D_id (int64) per observation
            images[image_id] = ColmapImage(image_id, np.array([qw, qx, qy, qz]), np.array([tx, ty, tz]), cam_id,
                                           name.decode())
    return images


def read_points3d_binary(path) -> dict[int, ColmapPoint]:
    points = {}
    with open(path, "rb") as f:
        (count,) = _read(f, "<Q")
        for _ in range(count):
            pid, x, y, z, r, g, b, _err, track = _read(f, "<Q3d3BdQ")
            f.seek(8 * track, 1)  # image_id, point2D_idx (uint32 each) per track element
            points[pid] = ColmapPoint(pid, np.array([x, y, z]), np.array([r, g, b], dtype=np.uint8))
    return points


def _text_lines(path):
    with open(path) as f:
        for line in f:
            line = line.strip()
            if line and not line.startswith("#"):
                yield line


def read_cameras_text(path) -> dict[int, ColmapCamera]:
    cams = {}
    for line in _text_lines(path):
        parts = line.split()
        cam_id, model, width, height = int(parts[0]), parts[1], int(parts[2]), int(parts[3])
        cams[cam_id] = ColmapCamera(cam_id, model, width, height, np.array([float(x) for x in parts[4:]]))
    return cams


def read_images_text(path) -> dict[int, ColmapImage]:
    images = {}
    with open(path) as f:
        rows = [ln.rstrip("\n") for ln in f if not ln.startswith("#")]
    # Two lines per image: the pose line, then its observations (possibly empty).
    i = 0
    while i < len(rows):
        if not rows[i].strip():
            i += 1
            continue
        parts = rows[i].split()
        image_id = int(parts[0])
        q = np.array([float(x) for x in parts[1:5]])
        t = np.array([float(x) for x in parts[5:8]])
        images[image_id] = ColmapImage(image_id, q, t, int(parts[8]), " ".join(parts[9:]))
        i += 2
    return images


def read_points3d_text(path) -> dict[int, ColmapPoint]:
    points = {}
    for line in _text_lines(path):
        parts = line.split()
        pid = int(parts[0])
        points[pid] = ColmapPoint(pid, np.array([float(x) for x in parts[1:4]]),
                                  np.array([int(x) for x in parts[4:7]], dtype=np.uint8))
    return points


def read_reconstruction(sparse_dir):
    """(cameras, images, points) of a COLMAP reconstruction folder, binary files preferred."""
    d = Path(sparse_dir)
    if (d / "cameras.bin").exists():
        return (read_cameras_binary(d / "cameras.bin"), read_images_binary(d / "images.bin"),
                read_points3d_binary(d / "points3D.bin"))
    if (d / "cameras.txt").exists():
        return (read_cameras_text(d / "cameras.txt"), read_images_text(d / "images.txt"),
                read_points3d_text(d / "points3D.txt"))
    raise FileNotFoundError(f"{d}: no cameras.bin or cameras.txt")


def qvec_to_rotmat(q: np.ndarray) -> np.ndarray:
    """Rotation matrix of a unit quaternion (w, x, y, z), normalised first (COLMAP stores unit
    quaternions; pycolmap's Rigid3d normalises on construction)."""
    w, x, y, z = q / np.linalg.norm(q)
    return np.array([[1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)],
                     [2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)],
                     [2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)]])


@dataclass
class Camera:
    """One view as the reference's Camera (utils/dataset.py:11-24)."""

    image_id: int
    name: str
    world_to_camera: torch.Tensor  # [4, 4] float32
    center: torch.Tensor  # [3]
    fx: float
    fy: float
    cx: float
    cy: float
    width: int
    height: int
    image: torch.Tensor  # [H, W, 3] uint8


@dataclass
class PointCloud:
    points: np.ndarray  # [N, 3] float32
    colors: np.ndarray  # [N, 3] float32 in [0, 1]


class ColmapDataset:
    """<root>/images and <root>/sparse/0 as the reference's ColmapDataset (utils/dataset.py:31-120):
    train_cameras, test_cameras (every test_every-th image by name), point_cloud and extent."""

    def __init__(self, data_path, max_width: int | None = 1600, test_every: int = 8, device: str = "cuda"):
        root = Path(data_path)
        self.cameras_by_id, images, points = read_reconstruction(root / "sparse" / "0")
        records = sorted(images.values(), key=lambda im: im.name)
        cams = [self._load_camera(im, root / "images", max_width, device) for im in records]
        self.train_cameras = [c for i, c in enumerate(cams) if i % test_every != 0]
        self.test_cameras = [c for i, c in enumerate(cams) if i % test_every == 0]
        pts = list(points.values())
        self.point_cloud = PointCloud(points=np.array([p.xyz for p in pts], dtype=np.float32).reshape(-1, 3),
                                      colors=np.array([p.rgb for p in pts], dtype=np.float32).reshape(-1, 3) / 255.0)
        centers = torch.stack([c.center for c in self.train_cameras])
        self.extent: float = 1.1 * (centers - centers.mean(dim=0)).norm(dim=1).max().item()

    def _load_camera(self, im: ColmapImage, images_dir: Path, max_width, device) -> Camera:
        from PIL import Image

        cam = self.cameras_by_id[im.camera_id]
        if cam.model not in ("SIMPLE_PINHOLE", "PINHOLE"):
            raise ValueError(f"{im.name}: camera model {cam.model} is unsupported, undistort the scene first")
        if cam.model == "SIMPLE_PINHOLE":
            f, cx, cy = cam.params
            fx = fy = f
        else:
            fx, fy, cx, cy = cam.params
        pil = Image.open(images_dir / im.name)
        width, height = pil.size
        if abs((width / height) / (cam.width / cam.height) - 1) > 0.01:
            raise ValueError(f"{im.name} is {pil.size}, not the aspect ratio of its COLMAP camera "
                             f"{(cam.width, cam.height)}")
        if max_width is not None and width > max_width:
            width, height = max_width, round(height * max_width / width)
        sx, sy = width / cam.width, height / cam.height
        pil.draft("RGB", (width, height))
        pil = pil.convert("RGB").resize((width, height))
        w2c = torch.eye(4)
        w2c[:3, :3] = torch.from_numpy(qvec_to_rotmat(im.qvec)).float()
        w2c[:3, 3] = torch.from_numpy(im.tvec).float()
        return Camera(image_id=im.image_id, name=im.name, world_to_camera=w2c.to(device),
                      center=w2c.inverse()[:3, 3].to(device), fx=float(fx) * sx, fy=float(fy) * sy,
                      cx=float(cx) * sx, cy=float(cy) * sy, width=width, height=height,
                      image=torch.from_numpy(np.array(pil)).to(device))


SH_C0 = 0.28209479177387814


def init_from_point_cloud(point_cloud: PointCloud, max_sh_degree: int = 3, device="cpu") -> dict:
    """The raw parameters of the reference's GaussianModel.__init__ (utils/gaussian.py:22-60): one
    gaussian per point; isotropic log-scale log(sqrt(mean squared distance to the 3 nearest
    neighbours)), clamped at 1e-7 before the root; identity quaternions; opacity logit of 0.1; SH DC
    from the point colour ((rgb - 0.5) / C0), higher degrees zero.  Names as the fused projection
    takes them (log_scales, opacity_logits)."""
    from scipy.spatial import KDTree

    pts = np.asarray(point_cloud.points, dtype=np.float32)
    n = len(pts)
    dists, _ = KDTree(pts).query(pts, k=4)
    dist2 = torch.from_numpy((dists[:, 1:] ** 2).mean(axis=1)).float().clamp_min(1e-7)
    log_scales = torch.log(torch.sqrt(dist2)).unsqueeze(-1).repeat(1, 3)
    coeffs = (max_sh_degree + 1) ** 2
    sh = torch.zeros(n, coeffs, 3)
    sh[:, 0] = (torch.from_numpy(np.asarray(point_cloud.colors, dtype=np.float32)) - 0.5) / SH_C0
    params = {"means": torch.from_numpy(pts), "log_scales": log_scales,
              "quats": torch.tensor([1.0, 0.0, 0.0, 0.0]).repeat(n, 1),
              "opacity_logits": torch.logit(torch.full((n, 1), 0.1)),
              "sh_dc": sh[:, :1], "sh_rest": sh[:, 1:]}
    return {k: v.contiguous().to(device) for k, v in params.items()}
