"""ctypes binding of the engine's C ABI (include/nsfps.h).

This is the binding a Python integrator writes against libnsfps.so without
the pybind11 module; bench.py and the tests use it to call the engine through
its C ABI.  Every function raises RuntimeError with nsfps_last_error() when a
call fails.
"""
import ctypes
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(ROOT, "ns_fps_b200", "libnsfps.so")
HEADER = os.path.join(ROOT, "include", "nsfps.h")

_u64p = ctypes.POINTER(ctypes.c_uint64)
_f32p = ctypes.POINTER(ctypes.c_float)
_u32p = ctypes.POINTER(ctypes.c_uint32)


class Range(ctypes.Structure):
    _fields_ = [("min_x", ctypes.c_float), ("max_x", ctypes.c_float),
                ("min_y", ctypes.c_float), ("max_y", ctypes.c_float),
                ("min_z", ctypes.c_float), ("max_z", ctypes.c_float),
                ("x_blocks", ctypes.c_uint32), ("y_blocks", ctypes.c_uint32),
                ("z_blocks", ctypes.c_uint32)]


class RangeInfo(ctypes.Structure):
    _fields_ = [("inv_bs", ctypes.c_float * 3), ("block_size", ctypes.c_float * 3),
                ("bits", ctypes.c_uint32 * 3), ("total_bits", ctypes.c_uint32),
                ("total_blocks", ctypes.c_uint64)]


class Profile(ctypes.Structure):
    _fields_ = [("setup_ms", ctypes.c_float), ("loop_ms", ctypes.c_float),
                ("total_ms", ctypes.c_float), ("launches", ctypes.c_uint32),
                ("ctas_per_cloud", ctypes.c_uint32), ("mode", ctypes.c_uint32),
                ("leaves", ctypes.c_uint32), ("ref_points_updated", ctypes.c_uint64),
                ("points_evaluated", ctypes.c_uint64), ("iterations", ctypes.c_uint64)]


OK, ERR_ARG, ERR_CUDA, ERR_OOM, ERR_TIMEOUT, ERR_UNSUPPORTED = range(6)

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} missing: run `python -m ns_fps_b200.build`")
        _lib = ctypes.CDLL(LIB_PATH)
        _lib.nsfps_last_error.restype = ctypes.c_char_p
    return _lib


def last_error() -> str:
    return lib().nsfps_last_error().decode()


def rng(bounds, blocks) -> Range:
    return Range(*[float(v) for v in bounds], *[int(b) for b in blocks])


def fps(points, k, bounds=None, blocks=(16, 16, 16), device=0):
    """nsfps_fps.  bounds None: the cloud's bounding box (compute_bbox) with
    `blocks` -- nsfps_fps with a NULL range for 16^3 (fps(range=None)),
    nsfps_fps_with_bbox otherwise (fps_with_bbox)."""
    p = np.ascontiguousarray(np.asarray(points, dtype=np.float32))
    n = p.shape[0]
    out = np.empty(max(min(int(k), n), 1), dtype=np.uint64)  # the library fills [0, len)
    ln = ctypes.c_uint64(0)
    if bounds is None and tuple(int(b) for b in blocks) != (16, 16, 16):
        xb, yb, zb = (int(b) for b in blocks)
        rc = lib().nsfps_fps_with_bbox(p.ctypes.data_as(_f32p), ctypes.c_uint64(n),
                                       ctypes.c_uint64(int(k)), ctypes.c_uint32(xb),
                                       ctypes.c_uint32(yb), ctypes.c_uint32(zb),
                                       out.ctypes.data_as(_u64p), ctypes.byref(ln),
                                       ctypes.c_int(device))
        if rc != OK:
            raise RuntimeError(f"nsfps_fps_with_bbox rc={rc}: {last_error()}")
        return _trimmed(out, ln.value)
    r = rng(bounds, blocks) if bounds is not None else None
    rc = lib().nsfps_fps(p.ctypes.data_as(_f32p), ctypes.c_uint64(n), ctypes.c_uint64(int(k)),
                         ctypes.byref(r) if r is not None else None,
                         out.ctypes.data_as(_u64p), ctypes.byref(ln), ctypes.c_int(device))
    if rc != OK:
        raise RuntimeError(f"nsfps_fps rc={rc}: {last_error()}")
    return _trimmed(out, ln.value)


def _trimmed(out, n):
    """The first n entries: the array itself when full, else a compact copy."""
    return out if n == out.shape[0] else out[:n].copy()


def fps_batched(clouds, k, bounds, blocks, devices=(0,), per_cloud=False):
    cl = [np.ascontiguousarray(np.asarray(c, dtype=np.float32)) for c in clouds]
    cnt = len(cl)
    # pointer arrays from plain addresses (ctypes.data_as costs microseconds
    # per array)
    ptrs = (ctypes.c_void_p * cnt)(*[c.ctypes.data for c in cl])
    ns = (ctypes.c_uint64 * cnt)(*[c.shape[0] for c in cl])
    # one block for every cloud's samples (the library fills each one's head)
    caps = [max(min(int(k), c.shape[0]), 1) for c in cl]
    starts = np.concatenate([[0], np.cumsum(caps)]).astype(np.int64)
    block = np.empty(int(starts[-1]), dtype=np.uint64)
    outs = [block[starts[i]:starts[i + 1]] for i in range(cnt)]
    optrs = (ctypes.c_void_p * cnt)(*[o.ctypes.data for o in outs])
    lens = (ctypes.c_uint64 * cnt)()
    if per_cloud:
        rs = (Range * cnt)(*[rng(b, bl) for b, bl in zip(bounds, blocks)])
    else:
        rs = (Range * 1)(rng(bounds, blocks))
    devs = (ctypes.c_int * len(devices))(*devices)
    rc = lib().nsfps_fps_batched(ptrs, ns, ctypes.c_uint64(cnt), ctypes.c_uint64(int(k)), rs,
                                 ctypes.c_int(1 if per_cloud else 0), optrs, lens, devs,
                                 ctypes.c_int(len(devices)))
    if rc != OK:
        raise RuntimeError(f"nsfps_fps_batched rc={rc}: {last_error()}")
    return [o[:lens[i]] for i, o in enumerate(outs)]


class TestHooks(ctypes.Structure):
    _fields_ = [("wait_limit_ns", ctypes.c_uint64), ("withhold_cta", ctypes.c_int32),
                ("withhold_step", ctypes.c_uint32), ("fail_alloc_device", ctypes.c_int32),
                ("reserved", ctypes.c_int32)]


def set_test_hooks(wait_limit_ns: int = 0, withhold_cta: int = -1, withhold_step: int = 0,
                   fail_alloc_device: int = -1, reset: bool = False):
    """nsfps_set_test_hooks (test use only): the in-kernel wait limit, one CTA
    that withholds its list / proposals at one round / step, a one-shot
    failed workspace request.  reset=True restores the defaults."""
    h = None if reset else TestHooks(int(wait_limit_ns), int(withhold_cta), int(withhold_step),
                                      int(fail_alloc_device), 0)
    rc = lib().nsfps_set_test_hooks(ctypes.byref(h) if h is not None else None)
    if rc != OK:
        raise RuntimeError(f"nsfps_set_test_hooks rc={rc}: {last_error()}")


def set_profiling(on: bool):
    lib().nsfps_set_profiling(ctypes.c_int(1 if on else 0))


def last_profile() -> Profile:
    p = Profile()
    lib().nsfps_last_profile(ctypes.byref(p))
    return p


def header_functions():
    """Names of the functions include/nsfps.h declares."""
    import re
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"NSFPS_API\s+[^;()]*?\b(nsfps_\w+)\s*\(", txt)))


def fps_device(d_xyz_ptr: int, offsets, k: int, ranges, per_cloud: bool, d_out_ptr: int,
               stream_ptr: int = 0):
    """nsfps_fps_device: clouds already in device memory (packed float32 xyz at
    d_xyz_ptr, `offsets` = count + 1 point offsets), results to the device
    buffer at d_out_ptr (count * k uint64).  `ranges` is one (bounds, blocks)
    pair, a list of them, or None (each cloud's bounding box with 16^3
    blocks, computed on the device).  Returns the per-cloud sample counts."""
    count = len(offsets) - 1
    offs = (ctypes.c_uint64 * (count + 1))(*[int(o) for o in offsets])
    if ranges is None:  # compute_bbox(cloud, 16, 16, 16) per cloud, on the device
        rs = None
    elif per_cloud:
        rs = (Range * count)(*[rng(b, bl) for b, bl in ranges])
    else:
        rs = (Range * 1)(rng(*ranges))
    lens = (ctypes.c_uint64 * count)()
    rc = lib().nsfps_fps_device(ctypes.c_void_p(d_xyz_ptr), offs, ctypes.c_uint64(count),
                                ctypes.c_uint64(int(k)), rs, ctypes.c_int(1 if per_cloud else 0),
                                ctypes.c_void_p(d_out_ptr), lens, ctypes.c_void_p(stream_ptr))
    if rc != OK:
        raise RuntimeError(f"nsfps_fps_device rc={rc}: {last_error()}")
    return [int(v) for v in lens]


def fps_device_with_bbox(d_xyz_ptr: int, offsets, k: int, blocks, d_out_ptr: int,
                         stream_ptr: int = 0):
    """nsfps_fps_device_with_bbox: as fps_device with each cloud's bounding
    box (reduced on the device) and `blocks` blocks.  Returns the per-cloud
    sample counts."""
    count = len(offsets) - 1
    offs = (ctypes.c_uint64 * (count + 1))(*[int(o) for o in offsets])
    lens = (ctypes.c_uint64 * count)()
    xb, yb, zb = (int(b) for b in blocks)
    rc = lib().nsfps_fps_device_with_bbox(ctypes.c_void_p(d_xyz_ptr), offs, ctypes.c_uint64(count),
                                          ctypes.c_uint64(int(k)), ctypes.c_uint32(xb),
                                          ctypes.c_uint32(yb), ctypes.c_uint32(zb),
                                          ctypes.c_void_p(d_out_ptr), lens,
                                          ctypes.c_void_p(stream_ptr))
    if rc != OK:
        raise RuntimeError(f"nsfps_fps_device_with_bbox rc={rc}: {last_error()}")
    return [int(v) for v in lens]


def fps_device_static(d_xyz_ptr: int, n: int, k: int, bounds, blocks, d_out_ptr: int,
                      stream_ptr: int = 0) -> int:
    """nsfps_fps_device_static: one cloud of n points in device memory,
    sampled with no device allocation (fixed scratch array; n at most
    NSFPS_STATIC_MAX_POINTS).  Returns the sample count."""
    r = rng(bounds, blocks)
    ln = ctypes.c_uint64(0)
    rc = lib().nsfps_fps_device_static(ctypes.c_void_p(d_xyz_ptr), ctypes.c_uint64(int(n)),
                                       ctypes.c_uint64(int(k)), ctypes.byref(r),
                                       ctypes.c_void_p(d_out_ptr), ctypes.byref(ln),
                                       ctypes.c_void_p(stream_ptr))
    if rc != OK:
        raise RuntimeError(f"nsfps_fps_device_static rc={rc}: {last_error()}")
    return int(ln.value)


# ---------------------------------------------------------------- grouping

def _offsets(offsets):
    return (ctypes.c_uint64 * len(offsets))(*[int(o) for o in offsets])


def ball_query(points, centers, radius: float, nsample: int, device: int = 0):
    """nsfps_ball_query: one cloud and its centres in host memory.  Returns
    (idx int64 (M, nsample), hits uint32 (M,))."""
    p = np.ascontiguousarray(np.asarray(points, dtype=np.float32))
    c = np.ascontiguousarray(np.asarray(centers, dtype=np.float32))
    m = c.shape[0]
    idx = np.zeros((m, max(int(nsample), 1)), dtype=np.int64)
    hits = np.zeros(m, dtype=np.uint32)
    rc = lib().nsfps_ball_query(p.ctypes.data_as(_f32p), ctypes.c_uint64(p.shape[0]),
                                c.ctypes.data_as(_f32p), ctypes.c_uint64(m),
                                ctypes.c_float(radius), ctypes.c_uint32(int(nsample)),
                                idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                                hits.ctypes.data_as(_u32p), ctypes.c_int(device))
    if rc != OK:
        raise RuntimeError(f"nsfps_ball_query rc={rc}: {last_error()}")
    return idx, hits


def ball_query_device(d_xyz_ptr: int, point_offsets, d_centers_ptr: int, center_offsets,
                      radius: float, nsample: int, d_idx_ptr: int, d_hits_ptr: int = 0,
                      stream_ptr: int = 0):
    """nsfps_ball_query_device on packed device-resident clouds and centres."""
    count = len(point_offsets) - 1
    rc = lib().nsfps_ball_query_device(
        ctypes.c_void_p(d_xyz_ptr), _offsets(point_offsets), ctypes.c_void_p(d_centers_ptr),
        _offsets(center_offsets), ctypes.c_uint64(count), ctypes.c_float(radius),
        ctypes.c_uint32(int(nsample)), ctypes.c_void_p(d_idx_ptr),
        ctypes.c_void_p(d_hits_ptr or None), ctypes.c_void_p(stream_ptr))
    if rc != OK:
        raise RuntimeError(f"nsfps_ball_query_device rc={rc}: {last_error()}")


def gather_points_device(d_xyz_ptr: int, point_offsets, d_idx_ptr: int, idx_offsets,
                         d_out_ptr: int, stream_ptr: int = 0):
    """nsfps_gather_points_device."""
    count = len(point_offsets) - 1
    rc = lib().nsfps_gather_points_device(
        ctypes.c_void_p(d_xyz_ptr), _offsets(point_offsets), ctypes.c_void_p(d_idx_ptr),
        _offsets(idx_offsets), ctypes.c_uint64(count), ctypes.c_void_p(d_out_ptr),
        ctypes.c_void_p(stream_ptr))
    if rc != OK:
        raise RuntimeError(f"nsfps_gather_points_device rc={rc}: {last_error()}")


def group_points_device(d_xyz_ptr: int, point_offsets, d_centers_ptr: int, center_offsets,
                        nsample: int, d_idx_ptr: int, d_out_ptr: int, stream_ptr: int = 0):
    """nsfps_group_points_device."""
    count = len(point_offsets) - 1
    rc = lib().nsfps_group_points_device(
        ctypes.c_void_p(d_xyz_ptr), _offsets(point_offsets), ctypes.c_void_p(d_centers_ptr),
        _offsets(center_offsets), ctypes.c_uint64(count), ctypes.c_uint32(int(nsample)),
        ctypes.c_void_p(d_idx_ptr), ctypes.c_void_p(d_out_ptr), ctypes.c_void_p(stream_ptr))
    if rc != OK:
        raise RuntimeError(f"nsfps_group_points_device rc={rc}: {last_error()}")
