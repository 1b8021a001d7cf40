"""Parity cases shared by the golden generator and the tests.

Each case is a point cloud, a sample count and a SpaceRange (bounds + blocks,
or bounds=None for the reference's compute_bbox path).  Inputs are rebuilt
from seeds; only the small hand-made edge cases store their points.

Families:
  * cfg_*      the five workload configs (ns_fps_b200.synthetic; c3/c5 use a
               few clouds of the batch)
  * ref_*      shaped like the reference's test.py checks (randn clouds from
               numpy's legacy RandomState(42)/(123), python-side bounding boxes
               with a 1% margin, the granularity sweep, manual ranges that
               clip the data)
  * edge_*     duplicates, exact ties, clamped outliers, non-power-of-two
               grids (bucket collisions), tiny clouds, degenerate ranges
  * kitti_*    the reference KITTI benchmark's setting
               (eval/src_cpu/compare_cpu_test_kitti.cpp:202-245): records
               filtered to z >= -5, the bounding box +- 1e-6 with 128 x 128 x 2
               blocks, on synthetic frames (ns_fps_b200.synthetic.kitti_records)
  * wide_*     power-of-two grids with more than 64 blocks on an axis
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np

from ns_fps_b200 import synthetic as S

HEAD = 2048  # entries kept for cases pinned by hash


@dataclass
class Case:
    name: str
    make: Callable[[], np.ndarray]
    k: int
    bounds: Optional[Tuple[float, ...]]
    blocks: Tuple[int, int, int]
    stored: str = "full"        # "full" indices or "head" + hash
    store_points: bool = False  # points saved in golden.npz
    large: bool = False         # slow on the CPU oracle

    def points(self) -> np.ndarray:
        return np.ascontiguousarray(np.asarray(self.make(), dtype=np.float32))


def bbox_python(points, margin=0.01):
    """Bounding box with a 1% margin + 1e-4, like the reference test.py
    compute_bbox_python (test.py:10-28)."""
    lo = points.min(axis=0)
    hi = points.max(axis=0)
    pad = (hi - lo) * margin + 1e-4
    return (float(lo[0] - pad[0]), float(hi[0] + pad[0]), float(lo[1] - pad[1]),
            float(hi[1] + pad[1]), float(lo[2] - pad[2]), float(hi[2] + pad[2]))


def _cfg(name: str, seed: int = 0, idx: int = 0):
    def f():
        return S.make(name, seed=seed, count=idx + 1)[idx]
    return f


def _ref_correctness() -> List[Case]:
    # test.py:88-104: np.random.seed(42), then four clouds in this order
    rs = np.random.RandomState(42)
    clouds = [
        ("ref_small_100_10", rs.randn(100, 3).astype(np.float32), 10),
        ("ref_medium_1k_100", rs.randn(1000, 3).astype(np.float32), 100),
        ("ref_large_10k_1k", rs.randn(10000, 3).astype(np.float32), 1000),
        ("ref_nonuniform_5k_500",
         (rs.randn(5000, 3).astype(np.float32) * np.array([10, 1, 0.1])).astype(np.float32), 500),
    ]
    out = []
    for name, pts, k in clouds:
        out.append(Case(name, (lambda p=pts: p), k, bbox_python(pts), (16, 16, 16)))
    return out


def _ref_granularity() -> List[Case]:
    # test.py:157-217: seed 42, randn(5000, 3) * 100, 500 samples, 7 grids
    pts = (np.random.RandomState(42).randn(5000, 3).astype(np.float32) * 100).astype(np.float32)
    grids = [(8, 8, 8), (16, 16, 16), (32, 32, 32), (64, 64, 64), (16, 8, 4), (4, 16, 64),
             (32, 16, 8)]
    return [Case(f"ref_gran_{a}x{b}x{c}", (lambda p=pts: p), 500, bbox_python(pts), (a, b, c))
            for a, b, c in grids]


def _ref_manual() -> List[Case]:
    # test.py:220-273: seed 123, anisotropic cloud, ranges that clip the data
    pts = np.random.RandomState(123).randn(3000, 3).astype(np.float32)
    pts[:, 0] = pts[:, 0] * 50 + 100
    pts[:, 1] = pts[:, 1] * 20 - 30
    pts[:, 2] = pts[:, 2] * 5 + 10
    rngs = [
        ("ref_manual_bbox", bbox_python(pts)),
        ("ref_manual_all", (0, 200, -100, 0, 0, 20)),
        ("ref_manual_y_tight", (0, 200, -40, -20, 0, 20)),
        ("ref_manual_z_tight", (0, 200, -100, 0, 10, 15)),
    ]
    return [Case(n, (lambda p=pts: p), 300, r, (16, 16, 8)) for n, r in rngs]


def _edge() -> List[Case]:
    cases = []
    r = np.random.RandomState(7)
    # all points identical -> stops after the first sample
    cases.append(Case("edge_all_same", lambda: np.full((257, 3), 1.5, np.float32), 50,
                      (0, 4, 0, 4, 0, 4), (16, 16, 16), store_points=True))
    # few distinct locations, many duplicates -> early stop at #distinct
    base = r.rand(5, 3).astype(np.float32)
    dup = base[r.randint(0, 5, 300)]
    cases.append(Case("edge_duplicates", lambda d=dup: d, 100, (0, 1, 0, 1, 0, 1), (4, 4, 4),
                      store_points=True))
    # integer lattice: many exactly equal distances -> tie-break order
    g = np.stack(np.meshgrid(np.arange(12), np.arange(12), np.arange(6), indexing="ij"),
                 -1).reshape(-1, 3).astype(np.float32)
    g = g[r.permutation(len(g))]
    cases.append(Case("edge_lattice_ties", lambda g=g: g, 400, (-0.5, 12, -0.5, 12, -0.5, 6),
                      (8, 8, 4), store_points=True))
    # outliers outside the range are clamped into border cells (a spread much
    # wider than this makes the reference reserve gigabytes for its cube list)
    o = r.randn(2000, 3).astype(np.float32)
    o[::7] *= 4
    cases.append(Case("edge_clamped_outliers", lambda o=o: o, 600, (-2, 2, -2, 2, -2, 2),
                      (16, 16, 16), store_points=True))
    # non-power-of-two grids: Morton codes collide modulo total_blocks
    q = (r.rand(3000, 3) * [3, 5, 7]).astype(np.float32)
    for bl in [(3, 5, 7), (5, 3, 1), (1, 2, 1), (6, 10, 12), (100, 3, 2)]:
        cases.append(Case(f"edge_hashed_{bl[0]}x{bl[1]}x{bl[2]}", lambda q=q: q, 700,
                          (0, 3, 0, 5, 0, 7), bl, store_points=True))
    # 1x1x1 grid: a single bucket
    cases.append(Case("edge_single_bucket", lambda q=q: q, 300, (0, 3, 0, 5, 0, 7), (1, 1, 1),
                      store_points=True))
    # tiny clouds and k around n
    t = r.randn(9, 3).astype(np.float32)
    for k in (1, 2, 8, 9, 20):
        cases.append(Case(f"edge_tiny_k{k}", lambda t=t: t, k, (-3, 3, -3, 3, -3, 3), (2, 2, 2),
                          store_points=True))
    cases.append(Case("edge_two_points", lambda: np.array([[0, 0, 0], [1, 1, 1]], np.float32), 2,
                      (-1, 2, -1, 2, -1, 2), (4, 4, 4), store_points=True))
    # compute_bbox path (range=None in fps): bounds from the reference's bbox
    b = (r.rand(4000, 3) * [30, 10, 2] - [15, 5, 1]).astype(np.float32)
    cases.append(Case("edge_bbox_default", lambda b=b: b, 800, None, (16, 16, 16),
                      store_points=True))
    cases.append(Case("edge_bbox_32x16x4", lambda b=b: b, 800, None, (32, 16, 4),
                      store_points=True))
    # flat cloud at a large offset through the bbox: the z extent collapses
    f = r.rand(1500, 3).astype(np.float32) * 10
    f[:, 2] = 80.0
    cases.append(Case("edge_flat_z80_bbox", lambda f=f: f, 200, None, (8, 8, 8),
                      store_points=True))
    # zero-width manual range (inverted ranges make the reference throw; they
    # are rejected up front, see tests/test_host.py)
    cases.append(Case("edge_zero_width_x", lambda f=f: f, 200, (3, 3, 0, 10, 79, 81), (8, 8, 8),
                      store_points=True))
    # large coordinates: squared distances far beyond 1e30
    big = (r.randn(1000, 3) * 1e17).astype(np.float32)
    cases.append(Case("edge_huge_coords", lambda b=big: b, 100, (-1e18, 1e18, -1e18, 1e18,
                                                                  -1e18, 1e18), (8, 8, 8),
                      store_points=True))
    return cases


def _kitti_like(seed: int, every: int = 1):
    from ns_fps_b200 import kitti

    def f():
        return kitti.filter_records(S.kitti_records(seed)[::every])
    return f


def _wide() -> List[Case]:
    out = [
        # a whole frame: one cloud of >= 98,304 points (the grid-wide loop)
        Case("kitti_like_f0_128x128x2", _kitti_like(0), 16384, None, (128, 128, 2)),
        # every 6th record: ~20.8k points (the round loop in one cluster)
        Case("kitti_like_f1_sub6_128x128x2", _kitti_like(1, 6), 4096, None, (128, 128, 2)),
    ]
    # (the reference's cube list reserve() takes (2nx+1)(2ny+1)(2nz+1) entries
    # in int, src/yuezu_fps.cpp:574, so the other axes' blocks stay wide)
    r = np.random.RandomState(77)
    w = (r.rand(20000, 3) * 1000.0).astype(np.float32)
    out.append(Case("wide_1024x2x2", lambda w=w: w, 3000, (0, 1000, 0, 1000, 0, 1000),
                    (1024, 2, 2), store_points=True))
    out.append(Case("wide_2x256x4_100k", lambda: (np.random.RandomState(78).rand(100_000, 3)
                                                   * 1000.0).astype(np.float32),
                    3000, (0, 1000, 0, 1000, 0, 1000), (2, 256, 4)))
    return out


def config_cases(include_large: bool) -> List[Case]:
    out = [
        Case("cfg_c1", _cfg("c1"), 1000, S.CONFIGS["c1"].rng, S.CONFIGS["c1"].blocks),
        Case("cfg_c3_cloud0", _cfg("c3", 0, 0), 4096, S.CONFIGS["c3"].rng, S.CONFIGS["c3"].blocks),
        Case("cfg_c3_cloud1", _cfg("c3", 0, 1), 4096, S.CONFIGS["c3"].rng, S.CONFIGS["c3"].blocks),
        Case("cfg_c2", _cfg("c2"), 16384, S.CONFIGS["c2"].rng, S.CONFIGS["c2"].blocks),
        Case("cfg_c5_scan7", _cfg("c5", 0, 7), 16384, S.CONFIGS["c5"].rng,
             S.CONFIGS["c5"].blocks, stored="head"),
    ]
    if include_large:
        out.append(Case("cfg_c4", _cfg("c4"), 65536, S.CONFIGS["c4"].rng, S.CONFIGS["c4"].blocks,
                        stored="head", large=True))
    return out


def all_cases(include_large: bool = False) -> List[Case]:
    return (config_cases(include_large) + _ref_correctness() + _ref_granularity() +
            _ref_manual() + _edge() + _wide())


def by_name(include_large: bool = True):
    return {c.name: c for c in all_cases(include_large)}
