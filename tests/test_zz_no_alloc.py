"""nsfps_fps_device_static: sampling with no device allocation.

Some callers cannot allocate device memory in the middle of a run: a host
that has handed all device memory to its own pool allocator, or a loop that
must not stall, since cudaMalloc / cudaFree synchronise the device.  This
entry point runs out of one fixed scratch array compiled into the library.

Collected last (file name) so that it also runs after every other test has
grown the per-device workspace of the allocating entry points.  It calls the
C ABI directly and compares each result with the CPU oracle and with the
allocating entry points (nsfps_fps_device and nsfps_fps) on the same
device-resident input.  Sample indices are integers, so the tolerance is exact
equality.  The cases cover power-of-two grids (the round loop: a small cloud
set up by one CTA and launched without a plan round trip, a mid-size one and
one at the size limit) and a non-power-of-two grid at the size limit (the
per-step loop with its bucket preimage table: the largest layout the fixed
array must hold), on the legacy default stream and on a separate stream.
"""
import numpy as np
import pytest

import oracle
from ns_fps_b200 import synthetic

pytestmark = pytest.mark.gpu

STATIC_MAX_POINTS = 65536


def _bounds(p):
    lo, hi = p.min(0) - 1e-6, p.max(0) + 1e-6
    return (lo[0], hi[0], lo[1], hi[1], lo[2], hi[2])


def _on_device(p):
    import torch
    return torch.from_numpy(np.ascontiguousarray(p, dtype=np.float32)).cuda(0)


def _via_device(capi, d, n, k, bounds, blocks):
    import torch
    out = torch.zeros(k, dtype=torch.int64, device="cuda:0")
    (ln,) = capi.fps_device(d.data_ptr(), [0, n], k, (bounds, blocks), False, out.data_ptr())
    torch.cuda.synchronize()
    return out[:ln].cpu().numpy().astype(np.uint64)


def _via_static(capi, d, n, k, bounds, blocks, out, stream=None):
    import torch
    sp = stream.cuda_stream if stream is not None else 0
    ln = capi.fps_device_static(d.data_ptr(), n, k, bounds, blocks, out.data_ptr(), sp)
    torch.cuda.synchronize()
    return out[:ln].cpu().numpy().astype(np.uint64)


def _cases():
    s = synthetic.gaussian_cloud(10_000, seed=10)
    a = synthetic.gaussian_cloud(20_000, seed=11)
    b = synthetic.sphere_cube_cloud(STATIC_MAX_POINTS, seed=12)
    c = synthetic.gaussian_cloud(STATIC_MAX_POINTS, seed=14)
    return [(s, 1_000, (16, 16, 16)), (a, 2_000, (16, 16, 16)), (b, 4_096, (32, 32, 32)),
            (c, 3_000, (20, 20, 20))]


def test_static_matches_oracle_and_allocating_entry_points_two_calls(capi):
    import torch
    cases = _cases()
    dev = [_on_device(p) for p, _, _ in cases]
    outs = [torch.zeros(k, dtype=torch.int64, device="cuda:0") for _, k, _ in cases]
    want = []
    for (p, k, bl), d in zip(cases, dev):
        w = oracle.fps(p, k, _bounds(p), bl)
        np.testing.assert_array_equal(_via_device(capi, d, p.shape[0], k, _bounds(p), bl), w)
        np.testing.assert_array_equal(capi.fps(p, k, _bounds(p), bl), w)
        want.append(w)
    # the first call on the device sets up the scratch array's address
    for (p, k, bl), d, o, w in zip(cases, dev, outs, want):
        o.fill_(-1)
        np.testing.assert_array_equal(_via_static(capi, d, p.shape[0], k, _bounds(p), bl, o), w)
    # two more calls in a row per cloud, each reusing the scratch the one
    # before left behind, the second on a separate stream; the device's free
    # memory must not change
    side = torch.cuda.Stream(device="cuda:0")
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(0)
    for stream in (None, side):
        for (p, k, bl), d, o, w in zip(cases, dev, outs, want):
            o.fill_(-1)
            torch.cuda.synchronize()
            got = _via_static(capi, d, p.shape[0], k, _bounds(p), bl, o, stream)
            np.testing.assert_array_equal(got, w)
    free1, _ = torch.cuda.mem_get_info(0)
    assert free0 == free1


def test_static_rejects_clouds_above_its_capacity(capi):
    import torch
    p = synthetic.gaussian_cloud(STATIC_MAX_POINTS + 1, seed=13)
    d = _on_device(p)
    out = torch.zeros(100, dtype=torch.int64, device="cuda:0")
    with pytest.raises(RuntimeError, match="NSFPS_STATIC_MAX_POINTS"):
        _via_static(capi, d, p.shape[0], 100, _bounds(p), (16, 16, 16), out)
