"""GPU parity on grids with more than 64 blocks on an axis, and on the
reference KITTI benchmark's setting.

The round loops hold an axis's cube thresholds across the replay warp's lanes
only when every axis has at most 64 of them; wider axes take the table walk in
shared memory.  The reference's KITTI harness uses exactly such a grid: the
bounding box +- 1e-6 with 128 x 128 x 2 blocks on frames filtered to z >= -5
(eval/src_cpu/compare_cpu_test_kitti.cpp:202-245).  These tests run that path
in both round loops -- the grid-wide loop (a single cloud) and the loop in
thread-block clusters (a batch of ~20k-point clouds, one cluster each) -- and
check which ran:

* goldens made by the compiled reference (tests/golden: kitti_like_*,
  wide_*), including the path through the .bin reader straight into device
  memory and the device-side bounding box;
* seeded clouds on grids with 128, 256 and 1024 blocks on one axis, against
  the CPU oracle.

Sample indices are integers: exact equality.
"""
import json
import os

import numpy as np
import pytest

import oracle
from ns_fps_b200 import kitti, synthetic
from tests import capi
from tests.golden import cases as C

pytestmark = pytest.mark.gpu

MODE_ROUNDS, MODE_GRID = 2, 3
GOLD_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
GOLD = json.load(open(os.path.join(GOLD_DIR, "golden.json")))
GOLD_NPZ = np.load(os.path.join(GOLD_DIR, "golden.npz"))
CASES = C.by_name(include_large=False)


def _profiled(fn):
    capi.set_profiling(True)
    try:
        return fn(), capi.last_profile()
    finally:
        capi.set_profiling(False)


def _points(name):
    if (name + "/points") in GOLD_NPZ.files:
        return GOLD_NPZ[name + "/points"]
    return CASES[name].points()


@pytest.mark.parametrize("name", ["kitti_like_f0_128x128x2", "kitti_like_f1_sub6_128x128x2",
                                  "wide_1024x2x2", "wide_2x256x4_100k"])
def test_wide_axis_goldens_run_the_round_loops(name):
    case = CASES[name]
    pts = _points(name)
    got, prof = _profiled(lambda: capi.fps(pts, case.k, case.bounds, case.blocks))
    assert prof.mode == MODE_GRID, f"{name}: expected the grid-wide loop, ran {prof.mode}"
    assert max(case.blocks) > 64
    exp = GOLD_NPZ[name + "/indices"].astype(np.uint64)
    assert GOLD[name]["stored"] == "full" and len(got) == GOLD[name]["len"]
    np.testing.assert_array_equal(got, exp)


@pytest.mark.parametrize("name", ["kitti_like_f1_sub6_128x128x2", "wide_1024x2x2"])
def test_wide_axis_goldens_in_clusters(name):
    """The same golden cloud twice in one device batch: a cluster per cloud
    (each cloud's bounding box reduced on the device when the case has none)."""
    import torch
    case = CASES[name]
    pts = _points(name)
    n = pts.shape[0]
    d = torch.from_numpy(np.concatenate([pts, pts])).cuda()
    out = torch.empty(2 * case.k, dtype=torch.int64, device="cuda")
    offs = np.array([0, n, 2 * n], np.int64)
    if case.bounds is None:
        run = lambda: capi.fps_device_with_bbox(d.data_ptr(), offs, case.k, case.blocks,
                                                out.data_ptr())
    else:
        run = lambda: capi.fps_device(d.data_ptr(), offs, case.k, (case.bounds, case.blocks),
                                      False, out.data_ptr())
    lens, prof = _profiled(run)
    assert prof.mode == MODE_ROUNDS, f"{name}: expected the cluster loop, ran {prof.mode}"
    exp = GOLD_NPZ[name + "/indices"].astype(np.uint64)
    got = out.cpu().numpy().astype(np.uint64).reshape(2, case.k)
    for c in range(2):
        assert lens[c] == len(exp)
        np.testing.assert_array_equal(got[c][:len(exp)], exp)


def test_kitti_bin_straight_to_device_matches_reference_golden(tmp_path):
    """A frame written as .bin records, read by kitti.load_bin straight into
    a CUDA tensor, sampled by the device entry with the box reduced on the
    device at 128 x 128 x 2: the compiled reference's golden indices, mapped
    to record numbers as the reference's Point3D index does."""
    import torch
    from ns_fps_b200 import torch_fps
    name = "kitti_like_f0_128x128x2"
    case = CASES[name]
    rec = synthetic.kitti_records(0)
    f = tmp_path / "frame.bin"
    rec.astype("<f4").tofile(f)
    t, recno = kitti.load_bin(f, device="cuda:0", return_index=True)
    assert t.is_cuda and t.shape == (GOLD[name]["n"], 3)
    idx = torch_fps.fps_with_bbox(t, case.k, *case.blocks)
    torch.cuda.synchronize()
    got = idx.cpu().numpy().astype(np.uint64)
    exp = GOLD_NPZ[name + "/indices"].astype(np.uint64)
    np.testing.assert_array_equal(got, exp)
    # the harness reports file record numbers (Point3D(x, y, z, i)): kept
    # records, in file order
    rn = recno[got.astype(np.int64)]
    assert rn.max() < rec.shape[0] and np.all(rec[rn, 2] >= -5.0)


def _wide_cloud(rs, n, kind):
    if kind == 0:
        return (rs.rand(n, 3) * 1000.0).astype(np.float32)
    c = rs.rand(30, 3) * 1000.0
    return (c[rs.randint(0, 30, n)] + rs.randn(n, 3) * 15.0).astype(np.float32)


@pytest.mark.parametrize("blocks", [(128, 4, 2), (8, 256, 4), (2, 2, 1024)])
@pytest.mark.parametrize("n,batch", [(20_000, 1), (20_000, 2), (110_000, 1)])
def test_wide_axis_seeded_grids_match_oracle(blocks, n, batch):
    """One cloud: the grid-wide loop; two ~20k-point clouds: a cluster each."""
    rs = np.random.RandomState(sum(blocks) + n)
    clouds = [_wide_cloud(rs, n, (blocks.index(max(blocks)) + n // 10000 + i) % 2)
              for i in range(batch)]
    allp = np.concatenate(clouds)
    lo, hi = allp.min(0) - 1e-3, allp.max(0) + 1e-3
    bounds = (lo[0], hi[0], lo[1], hi[1], lo[2], hi[2])
    k = 2500
    got, prof = _profiled(lambda: capi.fps_batched(clouds, k, bounds, blocks))
    mode = MODE_GRID if batch == 1 else MODE_ROUNDS
    assert prof.mode == mode, f"expected loop mode {mode}, ran {prof.mode}"
    for g, c in zip(got, clouds):
        np.testing.assert_array_equal(g, oracle.fps(c, k, bounds, blocks))
