"""Grouping after sampling, host side (no GPU): the C restatement of the ball
query (oracle/nsfps_oracle.c) agrees with an independent numpy restatement of
the PointNet++ definition, including the edge cases the device tests use, and
the C ABI rejects bad arguments before touching a device."""
import ctypes

import numpy as np
import pytest

import oracle
from tests import capi


def _edge_clouds():
    rs = np.random.default_rng(7)
    base = rs.normal(size=(600, 3)).astype(np.float32)
    dup = np.repeat(np.array([[0.5, -0.25, 2.0]], dtype=np.float32), 300, axis=0)
    flat = base.copy()
    flat[:, 2] = 0.0
    bad = base.copy()
    bad[5] = [np.nan, 0, 0]
    bad[17] = [np.inf, 1, 1]
    bad[33] = [0, -np.inf, 0]
    huge = (base * np.float32(1e30)).astype(np.float32)
    return {"gauss": base, "dup": dup, "flat": flat, "nonfinite": bad, "huge": huge}


@pytest.mark.parametrize("name", ["gauss", "dup", "flat", "nonfinite", "huge"])
@pytest.mark.parametrize("radius,nsample", [(0.3, 16), (1.0, 64), (-0.5, 8), (0.0, 4),
                                            (float("inf"), 8), (float("nan"), 4), (1e-3, 1)])
def test_c_oracle_matches_numpy_restatement(name, radius, nsample):
    pts = _edge_clouds()[name]
    rs = np.random.default_rng(11)
    centers = np.concatenate([pts[rs.integers(0, len(pts), 40)],
                              rs.normal(scale=3.0, size=(8, 3)).astype(np.float32),
                              np.array([[np.nan, 0, 0], [1e38, 0, 0]], dtype=np.float32)])
    if name == "huge":
        radius = radius * 1e30
    i1, h1 = oracle.ball_query(pts, centers, radius, nsample)
    i2, h2 = oracle.ball_query_numpy(pts, centers, radius, nsample)
    np.testing.assert_array_equal(h1, h2)
    np.testing.assert_array_equal(i1, i2)


def test_oracle_semantics_small_case():
    pts = np.array([[0, 0, 0], [1, 0, 0], [0.5, 0, 0], [3, 0, 0], [0.2, 0.1, 0]],
                   dtype=np.float32)
    centers = np.array([[0, 0, 0], [10, 0, 0], [3, 0, 0]], dtype=np.float32)
    idx, hits = oracle.ball_query(pts, centers, 0.6, 4)
    # centre 0: points 0, 2 (d2 0.25), 4 (d2 0.05) in index order, padded with 0
    assert idx[0].tolist() == [0, 2, 4, 0] and hits[0] == 3
    # centre 1: nothing within reach -> zeros
    assert idx[1].tolist() == [0, 0, 0, 0] and hits[1] == 0
    # centre 2: only point 3
    assert idx[2].tolist() == [3, 3, 3, 3] and hits[2] == 1
    # d2 < r2 is strict: point 1 at distance exactly 1 is no hit for r = 1
    idx, hits = oracle.ball_query(pts, centers[:1], 1.0, 8)
    assert 1 not in idx[0, :hits[0]].tolist()


def test_grouping_argument_errors():
    lib = capi.lib()
    pts = np.zeros((4, 3), dtype=np.float32)
    idx = np.zeros((4, 8), dtype=np.int64)
    f32 = pts.ctypes.data_as(capi._f32p)
    i64 = idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int64))
    assert lib.nsfps_ball_query(f32, ctypes.c_uint64(4), f32, ctypes.c_uint64(4),
                                ctypes.c_float(1.0), ctypes.c_uint32(0), i64, None, 0) == capi.ERR_ARG
    assert "nsample" in capi.last_error()
    assert lib.nsfps_ball_query(f32, ctypes.c_uint64(4), f32, ctypes.c_uint64(4),
                                ctypes.c_float(1.0), ctypes.c_uint32(2048), i64, None, 0) == capi.ERR_ARG
    assert lib.nsfps_ball_query(f32, ctypes.c_uint64(4), None, ctypes.c_uint64(4),
                                ctypes.c_float(1.0), ctypes.c_uint32(8), i64, None, 0) == capi.ERR_ARG
    offs_bad = (ctypes.c_uint64 * 3)(0, 5, 3)
    offs_ok = (ctypes.c_uint64 * 3)(0, 2, 4)
    assert lib.nsfps_ball_query_device(ctypes.c_void_p(1), offs_bad, ctypes.c_void_p(1), offs_ok,
                                       ctypes.c_uint64(2), ctypes.c_float(1.0),
                                       ctypes.c_uint32(8), ctypes.c_void_p(1), None,
                                       None) == capi.ERR_ARG
    assert "must not decrease" in capi.last_error()
    assert lib.nsfps_ball_query_device(ctypes.c_void_p(1), None, ctypes.c_void_p(1), offs_ok,
                                       ctypes.c_uint64(2), ctypes.c_float(1.0),
                                       ctypes.c_uint32(8), ctypes.c_void_p(1), None,
                                       None) == capi.ERR_ARG
    assert lib.nsfps_gather_points_device(ctypes.c_void_p(1), offs_ok, None, offs_ok,
                                          ctypes.c_uint64(2), ctypes.c_void_p(1),
                                          None) == capi.ERR_ARG
    assert lib.nsfps_group_points_device(ctypes.c_void_p(1), offs_ok, ctypes.c_void_p(1),
                                         offs_ok, ctypes.c_uint64(2), ctypes.c_uint32(0),
                                         ctypes.c_void_p(1), ctypes.c_void_p(1),
                                         None) == capi.ERR_ARG
    # nothing to do: no centres, no clouds
    assert lib.nsfps_ball_query(f32, ctypes.c_uint64(4), f32, ctypes.c_uint64(0),
                                ctypes.c_float(1.0), ctypes.c_uint32(8), i64, None, 0) == capi.OK
    assert lib.nsfps_ball_query_device(None, None, None, None, ctypes.c_uint64(0),
                                       ctypes.c_float(1.0), ctypes.c_uint32(8), None, None,
                                       None) == capi.OK
