"""GPU parity of the large-cloud layouts of the round loop against the CPU
oracle: bit-exact indices.

* The grid-wide loop (one cloud of at least 4,096 points over 64 or 128
  co-resident CTAs, 320 or 512 published candidates per round) on seeded
  random clouds: the golden vectors pin it on the c2 and c4 configs only;
  these cases add exact distance ties (quantised coordinates), clamped
  outliers (ranges narrower than the data), clustered and flat clouds and
  several direct (power-of-two) grids, and check that it is what ran.
* A batch of LiDAR scans, one cluster per scan with ~6 leaves per worker
  thread: slots dealt over the worker warps, samples queued with slot masks.
"""
import numpy as np
import pytest

import oracle
from tests import capi

pytestmark = pytest.mark.gpu

MODE_GRID = 3  # nsfps_profile.mode of the grid-wide round loop


def _cloud(rs, n, kind):
    if kind == 0:    # quantised: many exact ties among distances
        return (np.round(rs.randn(n, 3) * 8) / 4).astype(np.float32)
    if kind == 1:    # clustered
        c = rs.randn(24, 3) * 40
        return (c[rs.randint(0, 24, n)] + rs.randn(n, 3) * rs.uniform(0.5, 3)).astype(np.float32)
    if kind == 2:    # flat, scan-like
        p = rs.rand(n, 3) * [120, 120, 4]
        return p.astype(np.float32)
    return rs.randn(n, 3).astype(np.float32)


@pytest.mark.parametrize("seed", range(6))
def test_grid_loop_random_clouds_match_oracle(seed):
    rs = np.random.RandomState(7000 + seed)
    n = int(rs.choice([100_000, 160_000, 260_000]))
    pts = _cloud(rs, n, seed % 4)
    blocks = tuple(int(v) for v in rs.choice([8, 16, 32, 64], 3))
    lo, hi = pts.min(0), pts.max(0)
    shrink = rs.uniform(0.75, 1.05)  # below 1: points outside the range are clamped
    mid, half = (lo + hi) / 2, (hi - lo) / 2 * shrink + 1e-3
    bounds = (mid[0] - half[0], mid[0] + half[0], mid[1] - half[1], mid[1] + half[1],
              mid[2] - half[2], mid[2] + half[2])
    k = int(rs.choice([2_000, 6_000]))
    exp = oracle.fps(pts, k, bounds, blocks)
    capi.set_profiling(True)
    try:
        got = capi.fps(pts, k, bounds, blocks)
        prof = capi.last_profile()
    finally:
        capi.set_profiling(False)
    assert prof.mode == MODE_GRID, f"expected the grid-wide loop, ran mode {prof.mode}"
    assert prof.ctas_per_cloud in (64, 128)
    assert np.array_equal(got, exp), (
        f"n={n} k={k} blocks={blocks}: first mismatch at "
        f"{np.nonzero(got[:len(exp)] != exp[:len(got)])[0][:5]}")


def test_grid_loop_work_counter_equals_reference_work():
    """On a c2 scan (the grid-wide loop over 64 CTAs) the kernel's count of
    points in the buckets the reference updates equals the oracle's."""
    from ns_fps_b200 import synthetic as S
    cfg = S.CONFIGS["c2"]
    pts = S.make("c2", seed=11, count=1)[0]
    capi.set_profiling(True)
    try:
        idx = capi.fps(pts, cfg.k, cfg.rng, cfg.blocks)
        prof = capi.last_profile()
    finally:
        capi.set_profiling(False)
    exp, sum_u, _ = oracle.fps(pts, cfg.k, cfg.rng, cfg.blocks, stats=True)
    assert prof.mode == MODE_GRID and prof.ctas_per_cloud == 64
    assert np.array_equal(idx, exp)
    assert prof.ref_points_updated == sum_u
    assert prof.points_evaluated <= prof.ref_points_updated


MODE_CLUSTER_ROUNDS = 2  # nsfps_profile.mode of the round loop in one cluster per cloud


def test_batched_scans_large_parts_match_oracle():
    """A batch of LiDAR scans (c5's generator) runs one cluster of 16 CTAs per
    scan with about 6 leaves per worker thread: the layout whose slots are
    dealt over the worker warps and whose samples carry a slot mask."""
    from ns_fps_b200 import synthetic as S
    cfg = S.CONFIGS["c5"]
    clouds = S.make("c5", seed=300, count=3)
    k = 4000
    capi.set_profiling(True)
    try:
        got = capi.fps_batched(clouds, k, cfg.rng, cfg.blocks)
        prof = capi.last_profile()
    finally:
        capi.set_profiling(False)
    assert prof.mode == MODE_CLUSTER_ROUNDS and prof.ctas_per_cloud == 16, (prof.mode, prof.ctas_per_cloud)
    for i, cl in enumerate(clouds):
        exp = oracle.fps(cl, k, cfg.rng, cfg.blocks)
        assert np.array_equal(got[i], exp), f"scan {i}"


def _batch_profiled(clouds, k, rng, blocks, force=None):
    import os
    old = os.environ.get("NSFPS_BATCH_GROUP_CTAS")
    if force is not None:
        os.environ["NSFPS_BATCH_GROUP_CTAS"] = str(force)
    capi.set_profiling(True)
    try:
        got = capi.fps_batched(clouds, k, rng, blocks)
        return got, capi.last_profile()
    finally:
        capi.set_profiling(False)
        if force is not None:
            if old is None:
                os.environ.pop("NSFPS_BATCH_GROUP_CTAS", None)
            else:
                os.environ["NSFPS_BATCH_GROUP_CTAS"] = old


def test_batch_of_scans_runs_on_cta_groups():
    """More scans than the device holds clusters of 16 CTAs (7 on B200): the
    batch runs on groups of 16 co-resident CTAs, each group sampling its
    scans one after the other, with lists through global memory."""
    from ns_fps_b200 import synthetic as S
    cfg = S.CONFIGS["c5"]
    clouds = S.make("c5", seed=500, count=12)
    k = 3000
    got, prof = _batch_profiled(clouds, k, cfg.rng, cfg.blocks)
    assert prof.mode == MODE_GRID and prof.ctas_per_cloud == 16, (prof.mode, prof.ctas_per_cloud)
    for i in (0, 1, 9, 10, 11):  # groups 0..2 take two scans each
        assert np.array_equal(got[i], oracle.fps(clouds[i], k, cfg.rng, cfg.blocks)), f"scan {i}"


def test_cta_groups_loop_over_many_clouds_of_mixed_sizes_and_ranges():
    """Forced groups of 4 CTAs over 44 clouds (more than the 37 groups the
    device holds): groups take several clouds in turn, each with its own
    range and size."""
    rs = np.random.RandomState(61)
    clouds, bounds, blocks = [], [], []
    for i in range(44):
        n = int(rs.choice([701, 800, 5000, 16384]))
        p = (rs.rand(n, 3) * rs.uniform(1, 50, 3)).astype(np.float32)
        clouds.append(p)
        lo, hi = p.min(0) - 1e-3, p.max(0) + 1e-3
        bounds.append((lo[0], hi[0], lo[1], hi[1], lo[2], hi[2]))
        blocks.append(tuple(int(v) for v in rs.choice([4, 8, 16, 32], 3)))
    k = 700
    import os
    os.environ["NSFPS_BATCH_GROUP_CTAS"] = "4"
    capi.set_profiling(True)
    try:
        got = capi.fps_batched(clouds, k, bounds, blocks, per_cloud=True)
        prof = capi.last_profile()
    finally:
        capi.set_profiling(False)
        os.environ.pop("NSFPS_BATCH_GROUP_CTAS", None)
    assert prof.mode == MODE_GRID and prof.ctas_per_cloud == 4
    for i, cl in enumerate(clouds):
        assert np.array_equal(got[i], oracle.fps(cl, k, bounds[i], blocks[i])), f"cloud {i} n={len(cl)}"
