"""Point clouds stored as raw little-endian float32 records (the KITTI
velodyne ``.bin`` layout: x, y, z, intensity per point).

Follows the reference benchmark's reader and filter
(eval/src_cpu/compare_cpu_test_kitti.cpp:70-133 and :202-216): the file is
read as float32 values, ``floor(values / stride)`` points are taken (a
trailing partial record is ignored), the first three values of each record
are x, y, z, and only the points with ``z >= -5`` are kept, in file order.
"""
from __future__ import annotations

import numpy as np

__all__ = ["load_bin", "filter_records"]


def filter_records(rec: np.ndarray, z_min: float = -5.0, return_index: bool = False):
    """The benchmark's filter on (N, stride) records: the x, y, z of the
    records with ``z >= z_min``, in file order (a NaN z is dropped, as
    ``z >= -5`` is false), and optionally their record numbers."""
    keep = rec[:, 2] >= np.float32(z_min)
    pts = np.ascontiguousarray(rec[keep, :3], dtype=np.float32)
    if return_index:
        return pts, np.nonzero(keep)[0]
    return pts


def load_bin(path, stride: int = 4, z_min: float = -5.0, return_index: bool = False,
             device=None):
    """Read a ``.bin`` point cloud.

    Returns an (N, 3) float32 array (or a CUDA tensor when ``device`` is
    given) of the kept points; with ``return_index`` also the record number
    of each kept point in the file.  An empty file raises ``ValueError``.
    """
    if stride < 3:
        raise ValueError("stride must be at least 3 (x, y, z)")
    raw = np.fromfile(path, dtype="<f4")
    if raw.size == 0:
        raise ValueError(f"empty point cloud file: {path}")
    n = raw.size // stride
    rec = raw[: n * stride].reshape(n, stride)
    pts, idx = filter_records(rec, z_min, return_index=True)
    if device is not None:
        import torch
        pts = torch.from_numpy(pts).to(device)
    if return_index:
        return pts, idx
    return pts
