"""The .bin point-cloud reader follows the reference benchmark's reader and
z filter (eval/src_cpu/compare_cpu_test_kitti.cpp:70-133, :202-216).

Where the reference checkout is present (this build machine, not the GPU
box), its own SemanticKITTI frames also pin the CPU oracle to the compiled
reference in the benchmark's setting: the bounding box +- 1e-6 with
128 x 128 x 2 blocks (:230-245).  The frames are read in place and never
copied into this repository; the GPU tests use synthetic frames of the same
shape (ns_fps_b200.synthetic.kitti_records) with goldens from the compiled
reference.
"""
import glob
import os

import numpy as np
import pytest

import oracle
from ns_fps_b200 import kitti, synthetic
from tests.conftest import reference_dir


def test_load_bin_stride4_filter_and_order(tmp_path):
    rec = np.array([[1, 2, 3, 0.5], [4, 5, -6, 0.1], [7, 8, -5, 0.2], [9, 10, np.nan, 0.3],
                    [11, 12, 0, 0.4]], dtype="<f4")
    f = tmp_path / "a.bin"
    rec.tofile(f)
    pts, idx = kitti.load_bin(f, return_index=True)
    assert pts.dtype == np.float32 and pts.shape == (3, 3)
    np.testing.assert_array_equal(pts, rec[[0, 2, 4], :3])  # z >= -5 kept (-5 included), NaN dropped
    np.testing.assert_array_equal(idx, [0, 2, 4])


def test_load_bin_truncates_partial_record_and_stride3(tmp_path):
    vals = np.arange(14, dtype="<f4")  # 3 full records of 4, 2 values left over
    f = tmp_path / "b.bin"
    vals.tofile(f)
    pts = kitti.load_bin(f)
    np.testing.assert_array_equal(pts, vals[:12].reshape(3, 4)[:, :3])
    pts3 = kitti.load_bin(f, stride=3, z_min=-1e30)
    np.testing.assert_array_equal(pts3, vals[:12].reshape(4, 3))


def test_load_bin_empty_file_raises(tmp_path):
    f = tmp_path / "c.bin"
    f.write_bytes(b"")
    with pytest.raises(ValueError):
        kitti.load_bin(f)


def test_synthetic_frame_shape_and_filter():
    rec = synthetic.kitti_records(0)
    assert rec.dtype == np.float32 and rec.shape == (124_672, 4)
    pts, idx = kitti.filter_records(rec, return_index=True)
    assert pts.shape[0] == rec.shape[0] - 24  # 24 records below z = -5, one at exactly -5
    assert np.all(pts[:, 2] >= -5.0) and np.any(pts[:, 2] == -5.0)
    np.testing.assert_array_equal(pts, rec[idx, :3])


def _reference_frames():
    ref = reference_dir()
    if not ref:
        return []
    return sorted(glob.glob(os.path.join(ref, "eval", "kitti_data", "*.bin")))


@pytest.mark.skipif(not _reference_frames() or not oracle.have_ref(),
                    reason="the reference checkout and its compiled build are not on this machine")
@pytest.mark.parametrize("frame", range(6))
def test_reference_frames_oracle_equals_compiled_reference(frame):
    files = _reference_frames()
    if frame >= len(files):
        pytest.skip("frame not present")
    pts, recno = kitti.load_bin(files[frame], return_index=True)
    k = 16384
    blocks = (128, 128, 2)
    exp = oracle.ref_fps(pts, k, None, blocks)        # the harness's range: compute_bbox
    got = oracle.fps(pts, k, oracle.ref_bbox(pts, blocks), blocks)
    assert len(exp) == k
    np.testing.assert_array_equal(got, exp)
    assert np.all(np.diff(recno) > 0)
