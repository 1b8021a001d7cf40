"""Clouds already in GPU memory: the device entry point with no range (the
bounding box computed on the device, like fps(range=None)) and the PyTorch
tensor entry return exactly the reference's samples."""
import numpy as np
import pytest

import oracle
from ns_fps_b200 import synthetic
from tests import capi

pytestmark = pytest.mark.gpu


def _clouds():
    g = synthetic.gaussian_cloud(12_000, seed=31)
    lidar = synthetic.lidar_scan(seed=32)[::3][:30_000]
    sc = synthetic.sphere_cube_cloud(9_000, seed=33) * np.float32(7.0) - np.float32(2.5)
    return [np.ascontiguousarray(c, dtype=np.float32) for c in (g, lidar, sc)]


def test_device_bbox_matches_reference_bbox_path():
    import torch
    clouds = _clouds()
    k = 1500
    packed = torch.from_numpy(np.concatenate(clouds)).cuda()
    offs = np.concatenate([[0], np.cumsum([c.shape[0] for c in clouds])])
    out = torch.full((len(clouds) * k,), -1, dtype=torch.int64, device="cuda")
    lens = capi.fps_device(packed.data_ptr(), offs, k, None, False, out.data_ptr(),
                           torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    res = out.cpu().numpy().astype(np.uint64)
    for i, c in enumerate(clouds):
        got = res[i * k: i * k + lens[i]]
        want = oracle.fps(c, k, oracle.bbox(c), (16, 16, 16))
        np.testing.assert_array_equal(got, want)
        np.testing.assert_array_equal(got, capi.fps(c, k))  # host bbox path


def test_torch_entry_single_and_batched():
    import torch
    from ns_fps_b200 import torch_fps
    clouds = [c[:9000] for c in _clouds()]
    k = 800
    one = torch_fps.fps(torch.from_numpy(clouds[0]).cuda(), k)
    assert one.is_cuda and one.dtype == torch.int64
    np.testing.assert_array_equal(one.cpu().numpy().astype(np.uint64),
                                  oracle.fps(clouds[0], k, oracle.bbox(clouds[0]), (16, 16, 16)))
    batch = torch.from_numpy(np.stack(clouds)).cuda()
    rng = ((-12.0, 12.0, -12.0, 12.0, -12.0, 12.0), (16, 16, 16))
    outs = torch_fps.fps(batch, k, range=rng)
    for c, o in zip(clouds, outs):
        np.testing.assert_array_equal(o.cpu().numpy().astype(np.uint64), oracle.fps(c, k, *rng))


def test_device_bbox_slices_extremes_and_signed_zeros():
    """The on-device box (sliced over many blocks, merged with integer
    atomics) equals compute_bbox's on clouds whose extremes sit at the first
    and last points, at slice edges, on signed zeros, and on large clouds."""
    import torch
    rs = np.random.default_rng(21)
    a = rs.normal(size=(7000, 3)).astype(np.float32)
    a[0] = [9.0, -9.0, 0.5]
    a[-1] = [-9.5, 9.5, -0.5]
    b = rs.normal(size=(5000, 3)).astype(np.float32)
    b[:, 2] = np.where(rs.random(5000) < 0.5, np.float32(0.0), np.float32(-0.0))
    b[2047, 0], b[2048, 0], b[4095, 1] = 30.0, -30.0, 12.0  # slice boundaries
    c = np.repeat(rs.normal(size=(3, 3)).astype(np.float32), 700, axis=0)
    big = synthetic.lidar_scan(seed=5)
    tiny = np.array([[1.0, 2.0, 3.0], [-1.0, 0.0, 5.0]], dtype=np.float32)
    clouds = [a, b, c, big, tiny]
    k = 600
    packed = torch.from_numpy(np.concatenate(clouds)).cuda()
    offs = np.concatenate([[0], np.cumsum([x.shape[0] for x in clouds])])
    out = torch.full((len(clouds) * k,), -1, dtype=torch.int64, device="cuda")
    # tiny has fewer points than k: sample the others, then tiny on its own
    lens = capi.fps_device(packed.data_ptr(), offs[:5], k, None, False, out.data_ptr(),
                           torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    res = out.cpu().numpy().astype(np.uint64)
    for i, cl in enumerate(clouds[:4]):
        got = res[i * k: i * k + lens[i]]
        np.testing.assert_array_equal(got, oracle.fps(cl, k, oracle.bbox(cl), (16, 16, 16)))
        np.testing.assert_array_equal(got, capi.fps(cl, k))
    t = torch.from_numpy(tiny).cuda()
    o1 = torch.full((1,), -1, dtype=torch.int64, device="cuda")
    ln = capi.fps_device(t.data_ptr(), [0, 2], 1, None, False, o1.data_ptr(),
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert ln == [1] and int(o1[0]) == 0
