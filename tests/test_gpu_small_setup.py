"""GPU parity of the fused setup of small clouds against the CPU oracle.

Clouds of at most 24,576 points (every cloud of the call, with at most 2^17
buckets per range) are binned, sorted, cut into leaves and planned by one CTA
per cloud in one launch (a single cloud) or two (a batch) instead of the ~25
of the multi-launch pipeline.  Both must give the reference's bucket order,
so the samples are compared index for index with the oracle, and the launch
count shows which setup ran: sizes on both sides of each register-round step
(4 / 8 / 10 / 16 / 24 x 1024 points; up to 10 x 1024 the cloud is staged in
shared memory) and of the limit, exact distance ties, one bucket holding a
whole cloud (runs cut every 16 points), hashed grids (leaves with several
cells) and a grid over the bucket limit.
"""
import numpy as np
import pytest

import oracle
from tests import capi

pytestmark = pytest.mark.gpu

FUSED_MAX = 24576


def _run(fn):
    capi.set_profiling(True)
    try:
        out = fn()
        return out, capi.last_profile()
    finally:
        capi.set_profiling(False)


def _cloud(rs, n, kind):
    if kind == 0:  # quantised: exact ties
        return (np.round(rs.randn(n, 3) * 6) / 4).astype(np.float32)
    if kind == 1:  # clustered
        c = rs.randn(12, 3) * 3
        return (c[rs.randint(0, 12, n)] + rs.randn(n, 3) * 0.4).astype(np.float32)
    return (rs.rand(n, 3) * 8 - 4).astype(np.float32)


@pytest.mark.parametrize("n", [17, 1000, 4096, 4097, 8192, 8193, 10000, 10240, 10241, 16384,
                               16385, FUSED_MAX, FUSED_MAX + 1])
def test_single_cloud_matches_oracle(n):
    rs = np.random.RandomState(n)
    pts = _cloud(rs, n, n % 3)
    blocks = (16, 16, 16) if n % 2 else (32, 32, 8)
    bounds = (-4, 4, -4, 4, -4, 4)
    k = min(n - 1, 2000)
    exp = oracle.fps(pts, k, bounds, blocks)
    got, prof = _run(lambda: capi.fps(pts, k, bounds, blocks))
    np.testing.assert_array_equal(got, exp)
    if n <= FUSED_MAX:
        assert prof.launches <= 6, f"fused setup expected, {prof.launches} launches"
    else:
        assert prof.launches >= 12, f"multi-launch setup expected, {prof.launches} launches"


def test_one_bucket_cloud_matches_oracle():
    """Every point in one cell: a single run cut into 16-point leaves."""
    rs = np.random.RandomState(5)
    pts = (rs.rand(3000, 3) * 0.2).astype(np.float32)
    bounds, blocks = (0, 4, 0, 4, 0, 4), (8, 8, 8)
    exp = oracle.fps(pts, 500, bounds, blocks)
    got, prof = _run(lambda: capi.fps(pts, 500, bounds, blocks))
    np.testing.assert_array_equal(got, exp)
    assert prof.launches <= 6


def test_mixed_batch_with_hashed_ranges_matches_oracle():
    """Per-cloud ranges: direct grids and hashed ones (several cells per
    bucket), cloud sizes from 2 to the fused limit."""
    rs = np.random.RandomState(11)
    sizes = [2, 40, 700, 5000, 12000, FUSED_MAX, 3000, 9000]
    clouds = [_cloud(rs, n, i % 3) for i, n in enumerate(sizes)]
    bounds = [(-4, 4, -4, 4, -4, 4)] * len(sizes)
    blocks = [(16, 16, 16), (100, 3, 2), (32, 32, 8), (20, 20, 20), (16, 16, 16), (64, 8, 8),
              (7, 9, 11), (16, 16, 16)]
    k = 1500
    got, prof = _run(lambda: capi.fps_batched(clouds, k, bounds, blocks, per_cloud=True))
    assert prof.launches <= 6, f"fused setup expected, {prof.launches} launches"
    for i, c in enumerate(clouds):
        np.testing.assert_array_equal(got[i], oracle.fps(c, k, bounds[i], blocks[i]),
                                      err_msg=f"cloud {i} ({sizes[i]} points, {blocks[i]})")


def test_grid_over_bucket_limit_uses_pipeline():
    rs = np.random.RandomState(12)
    pts = _cloud(rs, 8000, 2)
    bounds, blocks = (-4, 4, -4, 4, -4, 4), (64, 64, 64)  # 262,144 buckets > 2^17
    exp = oracle.fps(pts, 1000, bounds, blocks)
    got, prof = _run(lambda: capi.fps(pts, 1000, bounds, blocks))
    np.testing.assert_array_equal(got, exp)
    assert prof.launches >= 12


@pytest.mark.parametrize("n", [4096, 10000, 12288, 12289])
def test_small_single_cloud_on_the_grid_loop(n):
    """A single cloud of 4,096 points or more runs the 64-CTA grid-wide loop.
    Up to 12,288 points it is launched right behind its setup with the
    worst-case plan (every leaf a single point still leaves one leaf per
    worker thread); above, after the plan's round trip.  Both exact."""
    rs = np.random.RandomState(100 + n)
    pts = _cloud(rs, n, n % 3)
    bounds, blocks = (-4, 4, -4, 4, -4, 4), (16, 16, 16)
    k = n // 8
    exp = oracle.fps(pts, k, bounds, blocks)
    for _ in range(2):  # the second call replays the cached setup graph
        got, prof = _run(lambda: capi.fps(pts, k, bounds, blocks))
        np.testing.assert_array_equal(got, exp)
        assert prof.mode == 3 and prof.ctas_per_cloud == 64, (prof.mode, prof.ctas_per_cloud)
