"""Parity checkers for the ns_fps_b200 engine -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the cpu_baseline / reference
legs of ``bench.py`` may import this package.  The product (``libnsfps.so`` and
``ns_fps_b200.yuezu_fps_module``) never imports, links or calls anything here.

Three checkers, all CPU:

* ``fps`` -- our C restatement of the reference algorithm
  (``oracle/nsfps_oracle.c``; it follows satreeby/ns_fps
  ``src/yuezu_fps.cpp:7-730``, see the file header for the line map).
* ``ref_fps`` -- the reference's own ``src/yuezu_fps.cpp`` compiled in place
  with ``-ffp-contract=off`` into ``oracle/_ref/libnsfps_ref.so`` by
  ``oracle/Makefile`` (present wherever that build ran; the prebuilt file
  travels with the repository snapshot).
* ``ref_module`` -- the reference's pybind11 module built from its own binding
  source (``yuezu_fps/yuezu_fps_pybind.cpp``) for API-surface comparisons.
"""
from __future__ import annotations

import ctypes
import importlib.util
import os
from typing import Optional, Sequence, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(_HERE, "_build", "libnsfps_oracle.so")
REF_SO = os.path.join(_HERE, "_ref", "libnsfps_ref.so")
REF_FMA_SO = os.path.join(_HERE, "_ref", "libnsfps_ref_fma.so")
REF_PY_DIR = os.path.join(_HERE, "_ref", "refpy")

_u64p = ctypes.POINTER(ctypes.c_uint64)
_f32p = ctypes.POINTER(ctypes.c_float)
_u32p = ctypes.POINTER(ctypes.c_uint32)

_libs = {}


def _load(path: str) -> ctypes.CDLL:
    if path not in _libs:
        if not os.path.exists(path):
            raise FileNotFoundError(
                f"{path} is missing: run `make -C oracle` (or __graft_entry__.build())")
        _libs[path] = ctypes.CDLL(path)
    return _libs[path]


def have_ref() -> bool:
    return os.path.exists(REF_SO)


def _pts(points) -> np.ndarray:
    p = np.ascontiguousarray(np.asarray(points, dtype=np.float32))
    if p.ndim != 2 or p.shape[1] != 3:
        raise ValueError("points must have shape (N, 3)")
    return p


def _rng_blocks(rng: Sequence[float], blocks: Sequence[int]):
    r = (ctypes.c_float * 6)(*[float(v) for v in rng])
    b = (ctypes.c_uint32 * 3)(*[int(v) for v in blocks])
    return r, b


def fps(points, k: int, rng: Sequence[float], blocks: Sequence[int],
        stats: bool = False):
    """Restated reference FPS.  Returns uint64 indices (and, with stats=True,
    (indices, sum_u, u_per_iteration))."""
    lib = _load(ORACLE_SO)
    p = _pts(points)
    n = p.shape[0]
    cap = max(int(k), n, 1)
    out = np.zeros(cap, dtype=np.uint64)
    u_iter = np.zeros(cap, dtype=np.uint64)
    out_len = ctypes.c_uint64(0)
    sum_u = ctypes.c_uint64(0)
    r, b = _rng_blocks(rng, blocks)
    rc = lib.nsfps_oracle_fps(
        p.ctypes.data_as(_f32p), ctypes.c_uint64(n), ctypes.c_uint64(int(k)), r, b,
        out.ctypes.data_as(_u64p), ctypes.byref(out_len), ctypes.byref(sum_u),
        u_iter.ctypes.data_as(_u64p))
    if rc != 0:
        raise RuntimeError(f"oracle fps failed (code {rc})")
    m = out_len.value
    if stats:
        return out[:m].copy(), int(sum_u.value), u_iter[:m].copy()
    return out[:m].copy()


def bbox(points) -> Tuple[float, ...]:
    """Restated compute_bbox bounds (min_x, max_x, min_y, max_y, min_z, max_z)."""
    lib = _load(ORACLE_SO)
    p = _pts(points)
    out = (ctypes.c_float * 6)()
    lib.nsfps_oracle_bbox(p.ctypes.data_as(_f32p), ctypes.c_uint64(p.shape[0]), out)
    return tuple(float(v) for v in out)


def range_info(rng, blocks, luts: bool = False):
    """Restated SpaceRange derived fields: dict(inv_bs, block_size, bits,
    total_bits[, luts])."""
    lib = _load(ORACLE_SO)
    r, b = _rng_blocks(rng, blocks)
    f = (ctypes.c_float * 6)()
    u = (ctypes.c_uint32 * 4)()
    rc = lib.nsfps_oracle_range_info(r, b, f, u, None, None, None)
    if rc != 0:
        raise ValueError(f"invalid range (code {rc})")
    out = dict(inv_bs=tuple(f[0:3]), block_size=tuple(f[3:6]), bits=tuple(u[0:3]),
               total_bits=int(u[3]))
    if luts:
        arrs = [np.zeros(1 << u[a], dtype=np.uint32) for a in range(3)]
        lib.nsfps_oracle_range_info(r, b, f, u, *[a.ctypes.data_as(_u32p) for a in arrs])
        out["luts"] = arrs
    return out


def bin_points(points, rng, blocks):
    """Restated (cell xyz, bucket) of every point."""
    lib = _load(ORACLE_SO)
    p = _pts(points)
    n = p.shape[0]
    cells = np.zeros((n, 3), dtype=np.uint32)
    buckets = np.zeros(n, dtype=np.uint64)
    r, b = _rng_blocks(rng, blocks)
    rc = lib.nsfps_oracle_bin(p.ctypes.data_as(_f32p), ctypes.c_uint64(n), r, b,
                              cells.ctypes.data_as(_u32p), buckets.ctypes.data_as(_u64p))
    if rc != 0:
        raise ValueError(f"invalid range (code {rc})")
    return cells, buckets


def ball_query(points, centers, radius: float, nsample: int):
    """Restated PointNet++ ball query (brute force, ``nsfps_oracle_ball_query``):
    (idx int64 (M, nsample), hits uint32 (M,)).  Not part of the reference."""
    lib = _load(ORACLE_SO)
    p = _pts(points)
    c = _pts(centers)
    m = c.shape[0]
    idx = np.zeros((m, max(int(nsample), 1)), dtype=np.int64)
    hits = np.zeros(m, dtype=np.uint32)
    lib.nsfps_oracle_ball_query(p.ctypes.data_as(_f32p), ctypes.c_uint64(p.shape[0]),
                                c.ctypes.data_as(_f32p), ctypes.c_uint64(m),
                                ctypes.c_float(radius), ctypes.c_uint32(int(nsample)),
                                idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                                hits.ctypes.data_as(_u32p))
    return idx, hits


def ball_query_numpy(points, centers, radius: float, nsample: int):
    """The same definition vectorised in numpy float32 (each operation rounded
    separately, no FMA): an independent restatement for checking the C one."""
    p = _pts(points)
    c = _pts(centers)
    idx = np.zeros((c.shape[0], int(nsample)), dtype=np.int64)
    hits = np.zeros(c.shape[0], dtype=np.uint32)
    with np.errstate(invalid="ignore", over="ignore"):
        r2 = np.float32(radius) * np.float32(radius)
        for j in range(c.shape[0]):
            d = p - c[j]
            d2 = (d[:, 0] * d[:, 0] + d[:, 1] * d[:, 1]) + d[:, 2] * d[:, 2]
            h = np.nonzero(d2 < r2)[0][: int(nsample)]
            hits[j] = len(h)
            if len(h):
                idx[j, :] = h[0]
                idx[j, : len(h)] = h
    return idx, hits


# ---------------------------------------------------------------- reference

def ref_fps(points, k: int, rng: Optional[Sequence[float]], blocks: Sequence[int],
            fma: bool = False) -> np.ndarray:
    """The reference's yuezu_fps() compiled in place.  rng=None uses the
    reference's compute_bbox(points, *blocks)."""
    lib = _load(REF_FMA_SO if fma else REF_SO)
    p = _pts(points)
    n = p.shape[0]
    cap = max(int(k), n, 1)
    out = np.zeros(cap, dtype=np.uint64)
    out_len = ctypes.c_uint64(0)
    r, b = _rng_blocks(rng if rng is not None else (0, 1, 0, 1, 0, 1), blocks)
    rc = lib.ref_fps(p.ctypes.data_as(_f32p), ctypes.c_uint64(n), ctypes.c_uint64(int(k)),
                     r, b, ctypes.c_int(1 if rng is None else 0),
                     out.ctypes.data_as(_u64p), ctypes.byref(out_len))
    if rc != 0:
        raise RuntimeError("reference fps raised")
    return out[:out_len.value].copy()


def ref_bbox(points, blocks=(16, 16, 16)) -> Tuple[float, ...]:
    lib = _load(REF_SO)
    p = _pts(points)
    _, b = _rng_blocks((0, 1, 0, 1, 0, 1), blocks)
    out = (ctypes.c_float * 6)()
    lib.ref_bbox(p.ctypes.data_as(_f32p), ctypes.c_uint64(p.shape[0]), b, out)
    return tuple(float(v) for v in out)


def ref_range_info(rng, blocks, luts: bool = False):
    lib = _load(REF_SO)
    r, b = _rng_blocks(rng, blocks)
    f = (ctypes.c_float * 6)()
    u = (ctypes.c_uint32 * 5)()
    lib.ref_range_info(r, b, f, u, None, None, None)
    out = dict(inv_bs=tuple(f[0:3]), block_size=tuple(f[3:6]), bits=tuple(u[0:3]),
               total_bits=int(u[3]), total_blocks=int(u[4]))
    if luts:
        arrs = [np.zeros(1 << u[a], dtype=np.uint32) for a in range(3)]
        lib.ref_range_info(r, b, f, u, *[a.ctypes.data_as(_u32p) for a in arrs])
        out["luts"] = arrs
    return out


def ref_fps_many(clouds, k: int, rng, blocks, threads: int):
    """Reference yuezu_fps() over whole clouds on `threads` host threads.
    Returns (list of index arrays, wall seconds of the parallel part)."""
    lib = _load(REF_SO)
    cl = [_pts(c) for c in clouds]
    cnt = len(cl)
    ptrs = (_f32p * cnt)(*[c.ctypes.data_as(_f32p) for c in cl])
    ns = (ctypes.c_uint64 * cnt)(*[c.shape[0] for c in cl])
    outs = [np.zeros(max(int(k), c.shape[0], 1), dtype=np.uint64) for c in cl]
    optrs = (_u64p * cnt)(*[o.ctypes.data_as(_u64p) for o in outs])
    lens = (ctypes.c_uint64 * cnt)()
    secs = ctypes.c_double(0.0)
    r, b = _rng_blocks(rng, blocks)
    rc = lib.ref_fps_many(ptrs, ns, ctypes.c_uint64(cnt), ctypes.c_uint64(int(k)), r, b,
                          optrs, lens, ctypes.c_int(int(threads)), ctypes.byref(secs))
    if rc != 0:
        raise RuntimeError("reference fps raised in a worker thread")
    return [o[:lens[i]].copy() for i, o in enumerate(outs)], float(secs.value)


def ref_module():
    """The reference's pybind11 module (yuezu_fps_module) built from its own
    binding source, or None when that build is absent."""
    for f in (os.listdir(REF_PY_DIR) if os.path.isdir(REF_PY_DIR) else []):
        if f.startswith("yuezu_fps_module") and f.endswith(".so"):
            spec = importlib.util.spec_from_file_location(
                "nsfps_oracle_ref.yuezu_fps_module", os.path.join(REF_PY_DIR, f))
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            return mod
    return None
