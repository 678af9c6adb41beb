"""Seeded synthetic workloads standing in for the reference's Truck scene.

The reference measures on the Tanks and Temples Truck scene (~1.18M gaussians, one 979x546 view),
which is not available here.  These generators draw gaussians with the shapes and value
distributions of the benchmark configurations instead (configs 0-4 of the build's baseline), plus
the distribution of the reference's own test scenes (tests/scenes.py:15-33 of the reference).

Every draw uses a seeded CPU torch.Generator, so a scene is identical on every machine; tensors
are moved to the requested device afterwards.  Cameras follow the COLMAP convention the
reference uses (x right, y down, z forward; world_to_camera maps world points into that frame).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch


@dataclass
class Camera:
    """A pinhole view: world_to_camera [4, 4], intrinsics in pixels and the image size."""

    world_to_camera: torch.Tensor
    fx: float
    fy: float
    cx: float
    cy: float
    width: int
    height: int

    @property
    def center(self) -> torch.Tensor:
        r = self.world_to_camera[:3, :3]
        t = self.world_to_camera[:3, 3]
        return -(r.T @ t)

    def to(self, device) -> "Camera":
        return Camera(self.world_to_camera.to(device), self.fx, self.fy, self.cx, self.cy, self.width, self.height)


@dataclass
class Scene:
    """Activated gaussian parameters (scales positive, unit quats, opacities in (0, 1)) and views."""

    means: torch.Tensor
    scales: torch.Tensor
    quats: torch.Tensor
    opacities: torch.Tensor
    sh_dc: torch.Tensor
    sh_rest: torch.Tensor
    features: torch.Tensor | None
    cameras: list[Camera] = field(default_factory=list)

    @property
    def n(self) -> int:
        return self.means.shape[0]

    def to(self, device) -> "Scene":
        move = lambda t: None if t is None else t.to(device).contiguous()
        return Scene(move(self.means), move(self.scales), move(self.quats), move(self.opacities), move(self.sh_dc),
                     move(self.sh_rest), move(self.features), [c.to(device) for c in self.cameras])


def look_at(center, target=(0.0, 0.0, 0.0), up=(0.0, -1.0, 0.0)) -> torch.Tensor:
    """world_to_camera for a camera at `center` looking at `target`, y down in the image."""
    c = torch.tensor(center, dtype=torch.float64)
    f = torch.tensor(target, dtype=torch.float64) - c
    f = f / f.norm()
    right = torch.linalg.cross(f, torch.tensor(up, dtype=torch.float64))
    right = right / right.norm()
    down = torch.linalg.cross(f, right)
    r = torch.stack([right, down, f])
    w2c = torch.eye(4, dtype=torch.float64)
    w2c[:3, :3] = r
    w2c[:3, 3] = -(r @ c)
    return w2c.float()


def orbit_camera(radius: float, elevation_deg: float, azimuth_deg: float, width: int, height: int,
                 focal_scale: float = 1.1) -> Camera:
    el, az = math.radians(elevation_deg), math.radians(azimuth_deg)
    # y is down, so a camera above the plane has negative y.
    center = (radius * math.cos(el) * math.sin(az), -radius * math.sin(el), -radius * math.cos(el) * math.cos(az))
    f = focal_scale * width
    return Camera(look_at(center), f, f, width / 2.0, height / 2.0, width, height)


def _normal(g, *shape, mean=0.0, std=1.0):
    return torch.randn(*shape, generator=g) * std + mean


def _activated(g, n, log_scale_mean, log_scale_std, opacity_logit_mean, opacity_logit_std, channels):
    scales = torch.exp(_normal(g, n, 3, mean=log_scale_mean, std=log_scale_std))
    quats = torch.nn.functional.normalize(torch.randn(n, 4, generator=g), dim=-1)
    opacities = torch.sigmoid(_normal(g, n, 1, mean=opacity_logit_mean, std=opacity_logit_std))
    sh_dc = _normal(g, n, 1, 3, std=0.5)
    sh_rest = _normal(g, n, 15, 3, std=0.1)
    features = torch.randn(n, channels, generator=g) if channels else None
    return scales, quats, opacities, sh_dc, sh_rest, features


def plane_and_clusters(g, n, plane_share=0.7, clusters=50, cluster_sigma=0.4):
    """70% on a noisy plane y ~ N(0, 0.05) over x, z in [-5, 5], the rest in isotropic clusters."""
    n_plane = int(round(plane_share * n))
    plane = torch.empty(n_plane, 3)
    plane[:, 0] = torch.rand(n_plane, generator=g) * 10 - 5
    plane[:, 2] = torch.rand(n_plane, generator=g) * 10 - 5
    plane[:, 1] = _normal(g, n_plane, std=0.05)
    centers = torch.empty(clusters, 3)
    centers[:, 0] = torch.rand(clusters, generator=g) * 8 - 4
    centers[:, 2] = torch.rand(clusters, generator=g) * 8 - 4
    centers[:, 1] = -torch.rand(clusters, generator=g) * 2.0
    pick = torch.randint(clusters, (n - n_plane,), generator=g)
    blobs = centers[pick] + _normal(g, n - n_plane, 3, std=cluster_sigma)
    return torch.cat([plane, blobs])


def config0(seed: int = 0, channels: int = 32) -> Scene:
    """4,096 gaussians, 128x96, camera at (0, 0, -6) looking at the origin, fx = fy = 120."""
    g = torch.Generator().manual_seed(seed)
    n = 4096
    means = torch.rand(n, 3, generator=g) * 4 - 2
    rest = _activated(g, n, -3.5, 0.6, 0.0, 1.5, channels)
    cam = Camera(look_at((0.0, 0.0, -6.0)), 120.0, 120.0, 64.0, 48.0, 128, 96)
    return Scene(means, *rest, cameras=[cam])


def config1(seed: int = 0, n: int = 100_000, channels: int = 32, width: int = 979, height: int = 546) -> Scene:
    """Plane + 50 clusters, log-scales N(-4.5, 0.8); one view at radius 8, elevation 15 deg, f = 1.1 W."""
    g = torch.Generator().manual_seed(seed)
    means = plane_and_clusters(g, n)
    rest = _activated(g, n, -4.5, 0.8, 0.0, 1.5, channels)
    return Scene(means, *rest, cameras=[orbit_camera(8.0, 15.0, 30.0, width, height)])


def config2(seed: int = 0, channels: int = 512) -> Scene:
    """Config-1 distribution at 1.18M gaussians (the Truck-sized channel sweep)."""
    return config1(seed, n=1_180_000, channels=channels)


def orbit(n_views: int, width: int = 979, height: int = 546, radius: float = 8.0,
          elevation=(10.0, 30.0)) -> list[Camera]:
    """Views evenly spaced in azimuth, elevation swept between the two bounds."""
    cams = []
    for i in range(n_views):
        el = elevation[0] + (elevation[1] - elevation[0]) * (0.5 - 0.5 * math.cos(2 * math.pi * i / n_views))
        cams.append(orbit_camera(radius, el, 360.0 * i / n_views, width, height))
    return cams


def config3(seed: int = 0, channels: int = 128, n_views: int = 64, n: int = 1_180_000) -> Scene:
    """1.18M gaussians, C = 128, 64 orbit views at 979x546 (data-parallel multi-view batch)."""
    s = config1(seed, n=n, channels=channels)
    s.cameras = orbit(n_views)
    return s


def config4(seed: int = 0, channels: int = 512, n: int = 4_000_000) -> Scene:
    """4M gaussians, 80% from 200 dense clusters (sigma 0.2), one 1920x1080 view."""
    g = torch.Generator().manual_seed(seed)
    n_cl = int(round(0.8 * n))
    centers = torch.rand(200, 3, generator=g) * 6 - 3
    centers[:, 1] = -torch.rand(200, generator=g) * 2.0
    pick = torch.randint(200, (n_cl,), generator=g)
    clustered = centers[pick] + _normal(g, n_cl, 3, std=0.2)
    means = torch.cat([clustered, plane_and_clusters(g, n - n_cl)])
    rest = _activated(g, n, -4.0, 0.6, 1.0, 1.0, channels)
    return Scene(means, *rest, cameras=[orbit_camera(8.0, 20.0, 45.0, 1920, 1080)])


def reference_test_scene(seed: int, n: int, channels: int = 3) -> dict[str, torch.Tensor]:
    """The distribution of the reference's tests/scenes.py:15-33: a box in front of an identity
    camera, scales exp(U[-4.5, -1.5]), opacities U[0.04, 0.99], colours U[0, 1)."""
    g = torch.Generator().manual_seed(seed)
    means = torch.rand(n, 3, generator=g) * torch.tensor([4.0, 3.0, 4.0]) + torch.tensor([-2.0, -1.5, 1.0])
    scales = torch.exp(torch.rand(n, 3, generator=g) * 3 - 4.5)
    quats = torch.nn.functional.normalize(torch.randn(n, 4, generator=g), dim=-1)
    opacities = torch.rand(n, 1, generator=g) * 0.95 + 0.04
    colors = torch.rand(n, channels, generator=g)
    return {"means": means, "scales": scales, "quats": quats, "opacities": opacities, "colors": colors}


def identity_camera(width: int, height: int) -> Camera:
    """The reference tests' camera: identity pose, focal 0.8 W, principal point at the centre."""
    f = 0.8 * width
    return Camera(torch.eye(4), f, f, width / 2.0, height / 2.0, width, height)
