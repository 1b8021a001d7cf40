"""Seeded synthetic point clouds with the shapes of the five workload configs.

The reference measures on SemanticKITTI LiDAR frames; these generators stand
in for them (no dataset is redistributed or reproduced).  Every generator is a
pure function of its seed and returns a C-contiguous float32 (N, 3) array.

  c1  10,000 N(0,1) points, K=1,000, range [-4,4]^3 16x16x16
  c2  one 64-beam x 1,920-step LiDAR scan (122,880 pts), K=16,384,
      range x,y in [-80,80], z in [-3,3], 32x32x8
  c3  32 clouds of 16,384 pts in [0,1]^3 (20% on 3 sphere surfaces), K=4,096,
      range [0,1]^3 16x16x16
  c4  1,048,576 pts: 90% in 50 anisotropic Gaussian clusters, 10% uniform,
      K=65,536, range [-100,100]^3 64x64x32
  c5  256 scans generated as c2 with seeds base+i, K=16,384 each
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Tuple

import numpy as np


@dataclass(frozen=True)
class Config:
    name: str
    n: int
    k: int
    rng: Tuple[float, float, float, float, float, float]
    blocks: Tuple[int, int, int]
    clouds: int = 1


CONFIGS = {
    "c1": Config("c1", 10_000, 1_000, (-4, 4, -4, 4, -4, 4), (16, 16, 16)),
    "c2": Config("c2", 122_880, 16_384, (-80, 80, -80, 80, -3, 3), (32, 32, 8)),
    "c3": Config("c3", 16_384, 4_096, (0, 1, 0, 1, 0, 1), (16, 16, 16), clouds=32),
    "c4": Config("c4", 1_048_576, 65_536, (-100, 100, -100, 100, -100, 100), (64, 64, 32)),
    "c5": Config("c5", 122_880, 16_384, (-80, 80, -80, 80, -3, 3), (32, 32, 8), clouds=256),
}


def gaussian_cloud(n: int = 10_000, seed: int = 0) -> np.ndarray:
    """c1: i.i.d. standard normal xyz."""
    r = np.random.default_rng(seed)
    return np.ascontiguousarray(r.standard_normal((n, 3)).astype(np.float32))


def lidar_scan(seed: int = 0, beams: int = 64, steps: int = 1920,
               sensor_height: float = 1.73, box_fraction: float = 0.3,
               n_boxes: int = 48, noise: float = 0.02) -> np.ndarray:
    """c2: synthetic 64-beam spinning-LiDAR scan.

    Elevation is spread evenly over [-25, +3] degrees per beam and azimuth is
    uniform in [0, 2*pi).  A ray's range is its ground-plane hit from
    ``sensor_height`` clipped to [2, 80] m (upward beams read 80 m).
    ``box_fraction`` of the rays are aimed at one of ``n_boxes`` random
    axis-aligned boxes (edges 1-5 m, centres 5-60 m away, standing on the
    ground) and take the nearer of the box hit and the ground hit.  Gaussian
    range noise of ``noise`` metres is added.
    """
    r = np.random.default_rng(seed)
    el = np.deg2rad(np.linspace(-25.0, 3.0, beams, dtype=np.float64))[:, None]
    el = np.broadcast_to(el, (beams, steps)).copy()
    az = r.uniform(0.0, 2.0 * math.pi, (beams, steps))

    sin_el = np.sin(el)
    with np.errstate(divide="ignore"):
        rg = np.where(sin_el < 0, sensor_height / np.maximum(-sin_el, 1e-12), 80.0)
    rg = np.clip(rg, 2.0, 80.0)

    # boxes: centre distance, azimuth, edge lengths
    bd = r.uniform(5.0, 60.0, n_boxes)
    bphi = r.uniform(0.0, 2.0 * math.pi, n_boxes)
    bsz = r.uniform(1.0, 5.0, (n_boxes, 3))
    bc = np.stack([bd * np.cos(bphi), bd * np.sin(bphi),
                   -sensor_height + bsz[:, 2] / 2.0], axis=1)
    lo = bc - bsz / 2.0
    hi = bc + bsz / 2.0

    hit_mask = r.random((beams, steps)) < box_fraction
    which = r.integers(0, n_boxes, (beams, steps))
    # aim the selected rays into their box's angular extent
    half = np.arctan2(np.maximum(bsz[:, 0], bsz[:, 1]) / 2.0, bd)
    aim = bphi[which] + r.uniform(-1.0, 1.0, (beams, steps)) * half[which]
    az = np.where(hit_mask, aim, az)

    dx = np.cos(el) * np.cos(az)
    dy = np.cos(el) * np.sin(az)
    dz = np.sin(el)
    # slab intersection of each selected ray with its box (origin at sensor)
    with np.errstate(divide="ignore", invalid="ignore"):
        d = np.stack([dx, dy, dz], axis=-1)
        inv = 1.0 / np.where(np.abs(d) < 1e-12, 1e-12, d)
        t0 = (lo[which] - 0.0) * inv
        t1 = (hi[which] - 0.0) * inv
        tmin = np.max(np.minimum(t0, t1), axis=-1)
        tmax = np.min(np.maximum(t0, t1), axis=-1)
    box_hit = hit_mask & (tmax >= np.maximum(tmin, 0.0)) & (tmin > 0.0)
    rng_m = np.where(box_hit, np.minimum(rg, tmin), rg)
    rng_m = rng_m + r.normal(0.0, noise, (beams, steps))

    pts = np.stack([rng_m * dx, rng_m * dy, rng_m * dz], axis=-1).reshape(-1, 3)
    return np.ascontiguousarray(pts.astype(np.float32))


def kitti_records(seed: int = 0, beams: int = 64, steps: int = 1948,
                  below: int = 24) -> np.ndarray:
    """A synthetic stand-in for one SemanticKITTI velodyne frame, as the
    file's records: (N, 4) float32 x, y, z, remission.

    The points are a ``lidar_scan`` of ``beams`` x ``steps`` rays (124,672 by
    default, about a real frame's 124.7k); ``below`` random records are moved
    below z = -5 m (the reference benchmark drops those,
    eval/src_cpu/compare_cpu_test_kitti.cpp:202-216) and one record sits at
    exactly z = -5 m (kept).  Remission is uniform on 0.00 .. 0.99 in steps of
    0.01.  No dataset record is reproduced.
    """
    r = np.random.default_rng(10_000 + seed)
    pts = lidar_scan(seed, beams=beams, steps=steps)
    n = pts.shape[0]
    idx = r.choice(n, below + 1, replace=False)
    pts[idx[:below], 2] = r.uniform(-12.0, -5.001, below).astype(np.float32)
    pts[idx[below], 2] = np.float32(-5.0)
    rem = (r.integers(0, 100, n) / 100.0).astype(np.float32)
    return np.ascontiguousarray(np.concatenate([pts, rem[:, None]], axis=1), dtype=np.float32)


def sphere_cube_cloud(n: int = 16_384, seed: int = 0, sphere_fraction: float = 0.2,
                      n_spheres: int = 3) -> np.ndarray:
    """c3: uniform in [0,1]^3 with ``sphere_fraction`` of the points resampled
    onto the surfaces of ``n_spheres`` spheres of radius 0.1-0.3."""
    r = np.random.default_rng(seed)
    pts = r.random((n, 3))
    centres = r.uniform(0.3, 0.7, (n_spheres, 3))
    radii = r.uniform(0.1, 0.3, n_spheres)
    sel = r.random(n) < sphere_fraction
    m = int(sel.sum())
    which = r.integers(0, n_spheres, m)
    v = r.standard_normal((m, 3))
    v /= np.linalg.norm(v, axis=1, keepdims=True)
    pts[sel] = centres[which] + v * radii[which, None]
    return np.ascontiguousarray(pts.astype(np.float32))


def cluster_cloud(n: int = 1_048_576, seed: int = 0, n_clusters: int = 50,
                  background: float = 0.1, extent: float = 100.0) -> np.ndarray:
    """c4: 90% of the points from ``n_clusters`` anisotropic Gaussians (means
    uniform in [-extent, extent]^3, per-axis sigma log-uniform in [0.5, 10]),
    10% uniform background over the same cube."""
    r = np.random.default_rng(seed)
    nb = int(round(n * background))
    nc = n - nb
    mu = r.uniform(-extent, extent, (n_clusters, 3))
    sig = np.exp(r.uniform(math.log(0.5), math.log(10.0), (n_clusters, 3)))
    which = r.integers(0, n_clusters, nc)
    cl = mu[which] + r.standard_normal((nc, 3)) * sig[which]
    bg = r.uniform(-extent, extent, (nb, 3))
    pts = np.concatenate([cl, bg], axis=0)
    pts = pts[r.permutation(n)]
    return np.ascontiguousarray(pts.astype(np.float32))


def make(config: str, seed: int = 0, count: int | None = None) -> List[np.ndarray]:
    """Clouds of a named config ('c1'..'c5').  ``count`` limits batched configs."""
    c = CONFIGS[config]
    nclouds = c.clouds if count is None else min(count, c.clouds)
    if config == "c1":
        return [gaussian_cloud(c.n, seed)]
    if config == "c2":
        return [lidar_scan(seed)]
    if config == "c3":
        return [sphere_cube_cloud(c.n, seed + i) for i in range(nclouds)]
    if config == "c4":
        return [cluster_cloud(c.n, seed)]
    if config == "c5":
        return [lidar_scan(seed + i) for i in range(nclouds)]
    raise KeyError(config)
