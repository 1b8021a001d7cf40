"""The reference's own checks, run through the reference's import name.

A user of satreeby/ns_fps imports ``yuezu_fps.yuezu_fps_module`` (setup.py:6,
test.py:3).  These tests import the engine under exactly that name and run
the checks of the reference's test.py -- verify_correctness (test.py:88-152),
verify_granularity (:157-217), verify_manual_range (:220-273) and
verify_step_by_step (:276-305) -- on the same inputs (numpy's legacy global
seed, the same clouds in the same order, compute_bbox_python's 1% margin).

The reference only compares distance sequences with a brute-force FPS
(|diff| < 1e-3, lengths within 1).  That check is kept, and every sample
index is also compared with the CPU oracle: integer work, exact equality.
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def yf():
    import yuezu_fps.yuezu_fps_module as m
    return m


def compute_bbox_python(yf, points, xb=16, yb=16, zb=16, margin=0.01):
    """test.py:10-28: bounds with a 1% margin + 1e-4, made by make_range."""
    mn, mx = points.min(axis=0), points.max(axis=0)
    pad = (mx - mn) * margin + 1e-4
    return yf.make_range(float(mn[0] - pad[0]), float(mx[0] + pad[0]),
                         float(mn[1] - pad[1]), float(mx[1] + pad[1]),
                         float(mn[2] - pad[2]), float(mx[2] + pad[2]), xb, yb, zb)


def fps_numpy(points, n_samples):
    """test.py:35-63: brute-force FPS (max distance per step)."""
    n = len(points)
    if n_samples >= n:
        return np.arange(n), np.zeros(n)
    idx = np.zeros(n_samples, dtype=np.int64)
    mind = np.full(n, np.inf, dtype=np.float32)
    p = points.astype(np.float32)
    md = np.zeros(n_samples, dtype=np.float32)
    md[0] = np.inf
    for i in range(1, n_samples):
        d = np.sum((p - p[idx[i - 1]]) ** 2, axis=1)
        mind = np.minimum(mind, d)
        md[i] = np.max(mind)
        idx[i] = np.argmax(mind)
        if md[i] == 0:
            return idx[:i], md[:i]
    return idx, md


def distance_sequence(points, indices):
    """test.py:66-81."""
    p = points.astype(np.float32)
    mind = np.full(len(points), np.inf, dtype=np.float32)
    md = np.zeros(len(indices), dtype=np.float32)
    md[0] = np.inf
    for i in range(1, len(indices)):
        mind = np.minimum(mind, np.sum((p - p[indices[i - 1]]) ** 2, axis=1))
        md[i] = np.max(mind)
    return md


def _range_tuple(r):
    return ((r.min_x, r.max_x, r.min_y, r.max_y, r.min_z, r.max_z),
            (r.x_blocks, r.y_blocks, r.z_blocks))


def _check(yf, points, k, r, dist_check=True):
    got = yf.fps(points, k, r)
    assert got.dtype == np.uint64
    bounds, blocks = _range_tuple(r)
    np.testing.assert_array_equal(got, oracle.fps(points, k, bounds, blocks))
    if dist_check:
        _, py_d = fps_numpy(points, k)
        cpp_d = distance_sequence(points, got.astype(np.int64))
        m = min(len(py_d), len(cpp_d))
        assert abs(len(py_d) - len(cpp_d)) <= 1
        assert np.max(np.abs(py_d[1:m] - cpp_d[1:m]), initial=0.0) < 1e-3
    return got


def test_import_name_is_the_engine(yf):
    import ns_fps_b200.yuezu_fps_module as m
    assert yf is m
    assert (yf.MORTON_BLOCK_SIZE, yf.CACHE_BLOCK_SIZE) == (16, 16)


def test_verify_correctness(yf):
    np.random.seed(42)
    cases = [
        (np.random.randn(100, 3).astype(np.float32), 10),
        (np.random.randn(1000, 3).astype(np.float32), 100),
        (np.random.randn(10000, 3).astype(np.float32), 1000),
        (np.random.randn(5000, 3).astype(np.float32) * [10, 1, 0.1], 500),
    ]
    for points, k in cases:
        points = np.asarray(points)  # the last case is float64, as in test.py
        _check(yf, points.astype(np.float32), k, compute_bbox_python(yf, points))
        # float64 input is converted like the reference's array_t<float>
        np.testing.assert_array_equal(yf.fps(points, k, compute_bbox_python(yf, points)),
                                      yf.fps(points.astype(np.float32), k,
                                             compute_bbox_python(yf, points)))


def test_verify_granularity(yf):
    np.random.seed(42)
    points = np.random.randn(5000, 3).astype(np.float32) * 100
    for xb, yb, zb in [(8, 8, 8), (16, 16, 16), (32, 32, 32), (64, 64, 64), (16, 8, 4),
                       (4, 16, 64), (32, 16, 8)]:
        _check(yf, points, 500, compute_bbox_python(yf, points, xb, yb, zb))


def test_verify_manual_range(yf):
    np.random.seed(123)
    points = np.random.randn(3000, 3).astype(np.float32)
    points[:, 0] = points[:, 0] * 50 + 100
    points[:, 1] = points[:, 1] * 20 - 30
    points[:, 2] = points[:, 2] * 5 + 10
    ranges = [compute_bbox_python(yf, points, 16, 16, 8),
              yf.make_range(0, 200, -100, 0, 0, 20, 16, 16, 8),
              yf.make_range(0, 200, -40, -20, 0, 20, 16, 16, 8),
              yf.make_range(0, 200, -100, 0, 10, 15, 16, 16, 8)]
    for r in ranges:
        # clipped ranges change which points the cube reaches, so the
        # brute-force distance check does not apply; the indices must still
        # be the reference's
        _check(yf, points, 300, r, dist_check=False)


def test_verify_step_by_step(yf):
    np.random.seed(123)
    points = np.random.randn(100, 3).astype(np.float32)
    got = _check(yf, points, 20, compute_bbox_python(yf, points))
    py_idx, _ = fps_numpy(points, 20)
    np.testing.assert_array_equal(got.astype(np.int64), py_idx)
