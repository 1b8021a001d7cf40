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
