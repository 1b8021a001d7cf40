"""The .bin point-cloud reader follows the reference benchmark's reader and
z filter (eval/src_cpu/compare_cpu_test_kitti.cpp:70-133, :202-216)."""
import numpy as np
import pytest

from ns_fps_b200 import kitti


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
