"""Sampling of clouds that already live in GPU memory as PyTorch tensors.

A thin layer over ``nsfps_fps_device``: the points stay on the device, the
work runs on PyTorch's current stream, and the indices come back as a CUDA
tensor, so a training loop pays no host round trip for the cloud.
"""
from __future__ import annotations

import builtins

from . import capi

__all__ = ["fps", "fps_with_bbox"]


def _range_arg(rng):
    if rng is None:
        return None
    if hasattr(rng, "min_x"):  # a SpaceRange (or anything with its fields)
        return ((rng.min_x, rng.max_x, rng.min_y, rng.max_y, rng.min_z, rng.max_z),
                (rng.x_blocks, rng.y_blocks, rng.z_blocks))
    bounds, blocks = rng
    return tuple(bounds), tuple(blocks)


def _as_batch(points):
    import torch
    if not isinstance(points, torch.Tensor) or not points.is_cuda:
        raise TypeError("points must be a CUDA tensor")
    if points.dtype != torch.float32:
        raise TypeError("points must be float32")
    single = points.dim() == 2
    if single:
        points = points.unsqueeze(0)
    if points.dim() != 3 or points.shape[2] != 3:
        raise ValueError("Expected tensor with shape (N, 3) or (B, N, 3)")
    return points.contiguous(), single


def fps_with_bbox(points, sample_count: int, x_blocks: int = 16, y_blocks: int = 16,
                  z_blocks: int = 16):
    """``fps_with_bbox`` of CUDA tensors: each cloud's bounding box (reduced
    on the device, widened by 1e-6 like compute_bbox) with the given block
    counts.  Shapes and results as in ``fps``."""
    import torch
    pts, single = _as_batch(points)
    B, N = int(pts.shape[0]), int(pts.shape[1])
    k = int(sample_count)
    out = torch.empty(B * k, dtype=torch.int64, device=pts.device)
    with torch.cuda.device(pts.device):
        stream = torch.cuda.current_stream(pts.device)
        lens = capi.fps_device_with_bbox(pts.data_ptr(), [i * N for i in builtins.range(B + 1)],
                                         k, (x_blocks, y_blocks, z_blocks), out.data_ptr(),
                                         stream.cuda_stream)
    res = [out[i * k: i * k + lens[i]] for i in builtins.range(B)]
    return res[0] if single else res


def fps(points, sample_count: int, range=None):
    """Farthest point sampling of CUDA tensors.

    points        float32 CUDA tensor of shape (N, 3), or (B, N, 3) for B clouds
    sample_count  samples per cloud; 0 < sample_count < N
    range         None (each cloud's bounding box with 16 x 16 x 16 blocks,
                  computed on the device, like ``fps(range=None)``), a
                  SpaceRange, or ``((min_x, max_x, min_y, max_y, min_z, max_z),
                  (x_blocks, y_blocks, z_blocks))`` shared by every cloud

    Returns an int64 CUDA tensor of indices for (N, 3) input, or a list of B
    of them; a result is shorter than ``sample_count`` when the reference
    stops early (every remaining point at distance 0).
    """
    import torch
    pts, single = _as_batch(points)
    B, N = int(pts.shape[0]), int(pts.shape[1])
    k = int(sample_count)
    out = torch.empty(B * k, dtype=torch.int64, device=pts.device)
    with torch.cuda.device(pts.device):
        stream = torch.cuda.current_stream(pts.device)
        lens = capi.fps_device(pts.data_ptr(), [i * N for i in builtins.range(B + 1)], k,
                               _range_arg(range), False, out.data_ptr(), stream.cuda_stream)
    res = [out[i * k: i * k + lens[i]] for i in builtins.range(B)]
    return res[0] if single else res
