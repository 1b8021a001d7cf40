"""Grouping after sampling on the GPU: the ball query, the gather of sampled
points and the relative grouping equal the brute-force oracle
(oracle/nsfps_oracle.c nsfps_oracle_ball_query) exactly, on the sampler's own
outputs (FPS centres) and on edge cases: non-finite points and centres, a
centre far outside the cloud, duplicates, flat and line-like clouds (one axis
at the per-axis cell cap), radius 0 / negative / NaN / infinite, nsample 1 and
the largest nsample, empty clouds in a batch."""
import numpy as np
import pytest

import oracle
from ns_fps_b200 import synthetic
from tests import capi

pytestmark = pytest.mark.gpu


def _check(pts, centers, radius, nsample):
    idx, hits = capi.ball_query(pts, centers, radius, nsample)
    ridx, rhits = oracle.ball_query(pts, centers, radius, nsample)
    np.testing.assert_array_equal(hits, rhits)
    np.testing.assert_array_equal(idx, ridx)
    return idx, hits


def test_ball_query_on_fps_centres_c1():
    c = synthetic.CONFIGS["c1"]
    pts = synthetic.make("c1", seed=0)[0]
    s = capi.fps(pts, c.k, c.rng, c.blocks)
    centers = pts[s.astype(np.int64)]
    for radius, nsample in [(0.5, 32), (0.2, 16), (1.5, 64), (0.05, 8)]:
        idx, hits = _check(pts, centers, radius, nsample)
        assert hits.min() >= 1  # every centre is a point of the cloud


def test_ball_query_on_fps_centres_lidar():
    pts = synthetic.lidar_scan(seed=3)
    s = capi.fps(pts, 4096, (-80, 80, -80, 80, -3, 3), (32, 32, 8))
    centers = pts[s.astype(np.int64)]
    for radius, nsample in [(0.5, 32), (2.0, 64)]:
        _check(pts, centers, radius, nsample)


def test_ball_query_clusters_and_large_nsample():
    pts = synthetic.cluster_cloud(60_000, seed=5)
    rs = np.random.default_rng(5)
    centers = pts[rs.integers(0, len(pts), 700)]
    _check(pts, centers, 3.0, 1024)
    _check(pts, centers, 1.0, 1)
    _check(pts, centers, 0.7, 100)


def test_ball_query_edge_cases():
    rs = np.random.default_rng(9)
    base = rs.normal(size=(20_000, 3)).astype(np.float32)
    centers = np.concatenate([base[rs.integers(0, len(base), 300)],
                              rs.normal(scale=4.0, size=(20, 3)).astype(np.float32),
                              np.array([[np.nan, 0, 0], [np.inf, 0, 0], [1e38, -1e38, 0],
                                        [0, 0, 1e6]], dtype=np.float32)])
    bad = base.copy()
    bad[rs.integers(0, len(bad), 50), 0] = np.nan
    bad[rs.integers(0, len(bad), 50), 1] = np.inf
    bad[rs.integers(0, len(bad), 50), 2] = -np.inf
    dup = np.repeat(base[:3], 4000, axis=0)
    flat = base.copy()
    flat[:, 2] = 1.0
    line = np.zeros((200_000, 3), dtype=np.float32)
    line[:, 0] = rs.uniform(0, 1e4, 200_000).astype(np.float32)
    line_c = line[rs.integers(0, len(line), 500)]
    huge = (base * np.float32(1e30)).astype(np.float32)
    for radius, nsample in [(0.4, 32), (-0.4, 16), (0.0, 8), (float("nan"), 8),
                            (float("inf"), 8), (1e-4, 4)]:
        _check(base, centers, radius, nsample)
        _check(bad, centers, radius, nsample)
    _check(dup, centers, 0.3, 64)
    _check(dup, dup[::997], 1e-6, 128)
    _check(flat, centers, 0.25, 32)
    _check(line, line_c, 0.5, 16)   # 20,000 cells of width 0.5 -> capped at 4096
    _check(line, line_c, 3.0, 48)
    _check(huge, huge[::50], 3e29, 16)
    _check(base[:1], base[:5], 1.0, 4)


def test_ball_query_batched_device_and_group_ops():
    import torch
    from ns_fps_b200 import group
    clouds = [synthetic.sphere_cube_cloud(16_384, seed=40 + i) for i in range(6)]
    pts = torch.from_numpy(np.stack(clouds)).cuda()
    m, S, radius = 512, 24, 0.08
    from ns_fps_b200 import torch_fps
    sidx = torch_fps.fps(pts, m)
    sidx = torch.stack(sidx)
    centers = group.gather_points(pts, sidx)
    idx, hits = group.ball_query(pts, centers, radius, S)
    torch.cuda.synchronize()
    grouped = group.group_points(pts, centers, idx)
    for b, cl in enumerate(clouds):
        c_np = cl[sidx[b].cpu().numpy()]
        np.testing.assert_array_equal(centers[b].cpu().numpy(), c_np)
        ridx, rhits = oracle.ball_query(cl, c_np, radius, S)
        np.testing.assert_array_equal(idx[b].cpu().numpy(), ridx)
        np.testing.assert_array_equal(hits[b].cpu().numpy().astype(np.uint32), rhits)
        ref_g = cl[ridx] - c_np[:, None, :]
        np.testing.assert_array_equal(grouped[b].cpu().numpy(), ref_g)


def test_ball_query_batch_with_empty_cloud():
    import torch
    rs = np.random.default_rng(12)
    sizes = [3000, 0, 5000, 1]
    clouds = [rs.normal(size=(n, 3)).astype(np.float32) for n in sizes]
    centers = [rs.normal(size=(64, 3)).astype(np.float32) for _ in sizes]
    poff = np.concatenate([[0], np.cumsum(sizes)])
    coff = np.arange(len(sizes) + 1) * 64
    d_pts = torch.from_numpy(np.concatenate(clouds)).cuda()
    d_ctr = torch.from_numpy(np.concatenate(centers)).cuda()
    S = 16
    d_idx = torch.full((len(sizes) * 64, S), -7, dtype=torch.int64, device="cuda")
    d_hits = torch.zeros(len(sizes) * 64, dtype=torch.int32, device="cuda")
    capi.ball_query_device(d_pts.data_ptr(), poff, d_ctr.data_ptr(), coff, 0.5, S,
                           d_idx.data_ptr(), d_hits.data_ptr(),
                           torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    for b in range(len(sizes)):
        ridx, rhits = oracle.ball_query(clouds[b], centers[b], 0.5, S)
        np.testing.assert_array_equal(d_idx[b * 64:(b + 1) * 64].cpu().numpy(), ridx)
        np.testing.assert_array_equal(d_hits[b * 64:(b + 1) * 64].cpu().numpy(), rhits)


def test_gather_rejects_out_of_range_index():
    import torch
    from ns_fps_b200 import group
    pts = torch.randn(100, 3, device="cuda")
    bad = torch.tensor([0, 5, 100], dtype=torch.int64, device="cuda")
    with pytest.raises(RuntimeError, match="outside its cloud"):
        group.gather_points(pts, bad)
    ok = torch.tensor([0, 5, 99], dtype=torch.int64, device="cuda")
    np.testing.assert_array_equal(group.gather_points(pts, ok).cpu().numpy(),
                                  pts[ok].cpu().numpy())
