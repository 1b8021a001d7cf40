"""Host-side logic of the engine, no GPU needed: the C ABI exports, SpaceRange
arithmetic and bbox against the reference, argument validation, the
reference's early returns, and the drop-in module's surface."""
import ctypes
import math
import subprocess

import numpy as np
import pytest

import oracle
from tests import capi

needs_ref = pytest.mark.skipif(not oracle.have_ref(), reason="reference not compiled here")


def test_header_functions_are_exported():
    names = capi.header_functions()
    assert len(names) >= 14
    lib = capi.lib()
    for n in names:
        assert hasattr(lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", capi.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if ln.strip()}
    ours = {e for e in exported if e.startswith("nsfps_")}
    assert ours == set(names), "exports and header disagree"


def _info(bounds, blocks):
    r = capi.rng(bounds, blocks)
    info = capi.RangeInfo()
    rc = capi.lib().nsfps_range_get_info(ctypes.byref(r), ctypes.byref(info))
    assert rc == capi.OK, capi.last_error()
    return info


@needs_ref
def test_range_info_matches_reference():
    rs = np.random.RandomState(11)
    for _ in range(80):
        lo = rs.uniform(-1e3, 1e3, 3).astype(np.float32)
        hi = (lo + rs.uniform(1e-3, 2e3, 3)).astype(np.float32)
        bounds = (lo[0], hi[0], lo[1], hi[1], lo[2], hi[2])
        blocks = tuple(int(b) for b in rs.choice([1, 2, 3, 4, 6, 8, 16, 33, 64, 512, 1024], 3))
        info = _info(bounds, blocks)
        ref = oracle.ref_range_info(bounds, blocks, luts=True)
        assert np.array_equal(np.float32(list(info.inv_bs)), np.float32(ref["inv_bs"]))
        assert np.array_equal(np.float32(list(info.block_size)), np.float32(ref["block_size"]))
        assert tuple(info.bits) == tuple(ref["bits"])
        assert info.total_bits == ref["total_bits"]
        assert info.total_blocks == blocks[0] * blocks[1] * blocks[2]
        for a in range(3):
            ln = ctypes.c_uint64(0)
            buf = np.zeros(1 << ref["bits"][a], dtype=np.uint32)
            rc = capi.lib().nsfps_range_get_lut(ctypes.byref(capi.rng(bounds, blocks)), a,
                                                buf.ctypes.data_as(capi._u32p),
                                                ctypes.c_uint64(buf.size), ctypes.byref(ln))
            assert rc == capi.OK
            assert ln.value == buf.size
            assert np.array_equal(buf, ref["luts"][a])


@needs_ref
def test_compute_bbox_matches_reference():
    rs = np.random.RandomState(12)
    for n in (0, 1, 5, 999):
        pts = (rs.randn(n, 3) * 70 - 5).astype(np.float32)
        r = capi.Range()
        rc = capi.lib().nsfps_compute_bbox(pts.ctypes.data_as(capi._f32p), ctypes.c_uint64(n), 32,
                                           16, 8, ctypes.byref(r))
        assert rc == capi.OK
        ref = oracle.ref_bbox(pts, (32, 16, 8))
        got = (r.min_x, r.max_x, r.min_y, r.max_y, r.min_z, r.max_z)
        assert np.array_equal(np.float32(got), np.float32(ref))
        if n == 0:
            assert (r.x_blocks, r.y_blocks, r.z_blocks) == (1, 1, 1)
        else:
            assert (r.x_blocks, r.y_blocks, r.z_blocks) == (32, 16, 8)


def test_reference_early_returns_need_no_gpu():
    # yuezu_fps: n == 0 or k == 0 -> [], k >= n -> 0..n-1 (src/yuezu_fps.cpp:678-688)
    pts = np.random.RandomState(0).randn(7, 3).astype(np.float32)
    assert len(capi.fps(pts, 0, (-5, 5, -5, 5, -5, 5), (4, 4, 4))) == 0
    assert len(capi.fps(np.zeros((0, 3), np.float32), 5, (-5, 5, -5, 5, -5, 5), (4, 4, 4))) == 0
    assert np.array_equal(capi.fps(pts, 7, (-5, 5, -5, 5, -5, 5), (4, 4, 4)), np.arange(7))
    assert np.array_equal(capi.fps(pts, 100, None), np.arange(7))


def test_batched_wrapper_returns_each_clouds_samples_without_gpu():
    """The batched wrapper hands the library one output block and returns a
    view per cloud; clouds the reference answers without sampling (k >= n,
    n == 0) exercise it on the host."""
    rs = np.random.RandomState(1)
    clouds = [rs.randn(n, 3).astype(np.float32) for n in (3, 0, 12, 1)]
    got = capi.fps_batched(clouds, 12, (-5, 5, -5, 5, -5, 5), (4, 4, 4))
    assert [len(g) for g in got] == [3, 0, 12, 1]
    for g, c in zip(got, clouds):
        assert g.dtype == np.uint64
        np.testing.assert_array_equal(g, np.arange(c.shape[0]))
    # the views do not overlap: writing one leaves the others intact
    got[0][:] = 7
    np.testing.assert_array_equal(got[2], np.arange(12))
    # the single-cloud wrapper returns the full array itself, or a compact copy
    full = capi.fps(clouds[2], 12, (-5, 5, -5, 5, -5, 5), (4, 4, 4))
    assert full.flags.owndata and len(full) == 12


def _rc_of_fps(pts, k, bounds, blocks):
    p = np.ascontiguousarray(pts, dtype=np.float32)
    out = np.zeros(max(k, 1), dtype=np.uint64)
    ln = ctypes.c_uint64(0)
    r = capi.rng(bounds, blocks)
    return capi.lib().nsfps_fps(p.ctypes.data_as(capi._f32p), ctypes.c_uint64(len(p)),
                                ctypes.c_uint64(k), ctypes.byref(r),
                                out.ctypes.data_as(capi._u64p), ctypes.byref(ln), 0)


def test_argument_errors():
    pts = np.random.RandomState(1).randn(50, 3).astype(np.float32)
    assert _rc_of_fps(pts, 10, (-5, 5, -5, 5, -5, 5), (0, 4, 4)) == capi.ERR_ARG
    assert "block counts" in capi.last_error()
    assert _rc_of_fps(pts, 10, (-5, 5, -5, 5, -5, 5), (2048, 4, 4)) == capi.ERR_UNSUPPORTED
    # an inverted range makes the reference throw on its first sampling step
    assert _rc_of_fps(pts, 10, (-5, 5, 5, -5, -5, 5), (4, 4, 4)) == capi.ERR_ARG
    assert "max must not be below min" in capi.last_error()
    ln = ctypes.c_uint64(0)
    assert capi.lib().nsfps_fps(None, ctypes.c_uint64(5), ctypes.c_uint64(2), None, None,
                                ctypes.byref(ln), 0) == capi.ERR_ARG
    assert capi.lib().nsfps_range_get_info(None, None) == capi.ERR_ARG


def test_version_and_device_count_calls():
    assert capi.lib().nsfps_version() >= 100
    c = ctypes.c_int(-1)
    capi.lib().nsfps_device_count(ctypes.byref(c))
    assert c.value >= 0


# ----------------------------------------------------------- drop-in module

def test_module_surface_matches_reference(yf):
    ref = oracle.ref_module()
    if ref is None:
        pytest.skip("reference module not built here")
    pub = {n for n in dir(ref) if not n.startswith("_")}
    ours = {n for n in dir(yf) if not n.startswith("_")}
    assert pub <= ours, pub - ours
    rs = {n for n in dir(ref.SpaceRange) if not n.startswith("_")}
    os_ = {n for n in dir(yf.SpaceRange) if not n.startswith("_")}
    assert rs <= os_, rs - os_
    for c in ("DEFAULT_X_BLOCKS", "DEFAULT_Y_BLOCKS", "DEFAULT_Z_BLOCKS", "MORTON_BLOCK_SIZE",
              "CACHE_BLOCK_SIZE"):
        assert getattr(yf, c) == getattr(ref, c)


def test_spacerange_methods_match_reference(yf):
    ref = oracle.ref_module()
    if ref is None:
        pytest.skip("reference module not built here")
    rs = np.random.RandomState(2)
    for _ in range(30):
        lo = rs.uniform(-50, 50, 3)
        hi = lo + rs.uniform(0.1, 100, 3)
        b = [int(v) for v in rs.choice([1, 2, 3, 8, 16, 100], 3)]
        args = (float(lo[0]), float(hi[0]), float(lo[1]), float(hi[1]), float(lo[2]),
                float(hi[2]), *b)
        a, r = yf.make_range(*args), ref.make_range(*args)
        for m in ("block_size_x", "block_size_y", "block_size_z", "x_bits", "y_bits", "z_bits",
                  "total_bits", "total_blocks"):
            assert np.float32(getattr(a, m)()) == np.float32(getattr(r, m)()), m
        for f in ("min_x", "max_x", "min_y", "max_y", "min_z", "max_z", "x_blocks", "y_blocks",
                  "z_blocks"):
            assert getattr(a, f) == getattr(r, f)
        u, v = yf.make_uniform_range(*args[:6], b[0]), ref.make_uniform_range(*args[:6], b[0])
        assert (u.x_blocks, u.y_blocks, u.z_blocks) == (v.x_blocks, v.y_blocks, v.z_blocks)
    d = yf.SpaceRange()
    assert d.x_blocks == 0 and d.min_x == 0.0


def test_module_shape_error_and_early_returns(yf):
    with pytest.raises(RuntimeError, match=r"Expected 2D array with shape \(N, 3\)"):
        yf.fps(np.zeros((5, 2), np.float32), 3)
    with pytest.raises(RuntimeError, match=r"Expected 2D array with shape \(N, 3\)"):
        yf.fps(np.zeros(9, np.float32), 3)
    pts = np.random.RandomState(5).randn(6, 3)  # float64 is converted like the reference
    out = yf.fps(pts, 6)
    assert out.dtype == np.uint64 and np.array_equal(out, np.arange(6))
    assert len(yf.fps(pts, 0)) == 0
    assert np.array_equal(yf.fps(pts, n_samples=10), np.arange(6))
    assert np.array_equal(yf.fps_with_bbox(pts, 9, 4, 4, 4), np.arange(6))
    with pytest.raises(TypeError):
        yf.fps(pts, 3, n_samples=3)
    with pytest.raises(RuntimeError):
        yf.fps(np.random.randn(50, 3), 5, yf.make_range(-1, 1, -1, 1, -1, 1, 0, 4, 4))


def test_cube_threshold_idea_is_exact():
    """The loop kernel reads the cube half-width ceil(sqrt(D) / bs) from
    thresholds: T[n] = the largest float32 D with ceil(sqrt(D)/bs) <= n.  Check
    the idea in float32 arithmetic (numpy's sqrt and divide are correctly
    rounded) against the direct formula on random D."""
    rs = np.random.RandomState(9)
    f32 = np.float32
    for bs in (f32(0.25), f32(5.0), f32(6.25), f32(160 / 32), f32(1 / 3)):
        blocks = 40

        def ratio(D):
            return f32(np.sqrt(f32(D))) / bs

        tab = []
        for n in range(blocks - 1):
            lo, hi = 0, 0x7F7FFFFF
            while hi - lo > 1:
                mid = (lo + hi) // 2
                d = np.array([mid], np.uint32).view(np.float32)[0]
                if ratio(d) <= n:
                    lo = mid
                else:
                    hi = mid
            tab.append(np.array([lo], np.uint32).view(np.float32)[0])
        tab = np.array(tab, np.float32)
        D = (rs.uniform(0, (blocks * float(bs)) ** 2, 4000)).astype(np.float32)
        D = np.concatenate([D, tab, np.nextafter(tab, np.float32(np.inf))])
        for d in D:
            direct = min(int(math.ceil(ratio(d))), blocks - 1)
            via_tab = int(np.sum(tab < d))
            assert direct == via_tab, (float(bs), float(d))


def test_reference_import_name_resolves_to_the_engine():
    """`import yuezu_fps.yuezu_fps_module as yf` (the reference's name,
    setup.py:6, test.py:3) gives this engine's module object."""
    import yuezu_fps.yuezu_fps_module as yf
    import ns_fps_b200.yuezu_fps_module as m
    assert yf is m
    r = yf.make_range(-1, 1, -2, 2, -3, 3, 128, 128, 2)
    assert (r.x_blocks, r.y_blocks, r.z_blocks) == (128, 128, 2)


def test_test_hooks_set_and_reset_without_gpu():
    capi.set_test_hooks(wait_limit_ns=1_000_000, withhold_cta=3, withhold_step=2,
                        fail_alloc_device=0)
    capi.set_test_hooks(reset=True)
    with pytest.raises(RuntimeError, match="rc=1"):
        capi.set_test_hooks(wait_limit_ns=10 ** 12)
    capi.set_test_hooks(reset=True)
