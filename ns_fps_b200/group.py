"""Grouping after sampling on CUDA tensors: the PointNet++ operators that
follow farthest point sampling.

* ``ball_query(points, centers, radius, nsample)``: for each centre, the
  first ``nsample`` point indices (ascending) within ``radius``; the unfilled
  slots repeat the first hit (index 0 when there is none), and ``hits`` holds
  how many were found (at most ``nsample``).
* ``gather_points(points, idx)``: the coordinates of the indexed points.
* ``group_points(points, centers, idx)``: those of ``idx`` (M, nsample)
  minus their centre, shape (M, nsample, 3).

Each takes one cloud (N, 3) or a batch (B, N, 3) with matching (B, M, ...)
centres / indices, runs on PyTorch's current stream through the C ABI
(``nsfps_ball_query_device`` and friends) and returns CUDA tensors.  The
distance test is the sampler's: d2 = (dx*dx + dy*dy) + dz*dz, fp32 rounded
per operation without multiply-add contraction, hit iff d2 < radius * radius.
"""
from __future__ import annotations

from . import capi

__all__ = ["ball_query", "gather_points", "group_points"]


def _cloud_batch(t, name):
    import torch
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    if t.dtype != torch.float32:
        raise TypeError(f"{name} must be float32")
    single = t.dim() == 2
    if single:
        t = t.unsqueeze(0)
    if t.dim() != 3 or t.shape[2] != 3:
        raise ValueError(f"{name}: expected shape (N, 3) or (B, N, 3)")
    return t.contiguous(), single


def _offsets(B, n):
    return [i * n for i in range(B + 1)]


def ball_query(points, centers, radius: float, nsample: int):
    """Returns (idx int64 (M, nsample) or (B, M, nsample), hits int32 (M,) or
    (B, M))."""
    import torch
    pts, single = _cloud_batch(points, "points")
    ctr, single_c = _cloud_batch(centers, "centers")
    if single != single_c or pts.shape[0] != ctr.shape[0]:
        raise ValueError("points and centers must have the same batch layout")
    if pts.device != ctr.device:
        raise ValueError("points and centers must be on the same device")
    B, N, M = int(pts.shape[0]), int(pts.shape[1]), int(ctr.shape[1])
    S = int(nsample)
    idx = torch.empty((B, M, S), dtype=torch.int64, device=pts.device)
    hits = torch.empty((B, M), dtype=torch.int32, device=pts.device)
    with torch.cuda.device(pts.device):
        stream = torch.cuda.current_stream(pts.device)
        capi.ball_query_device(pts.data_ptr(), _offsets(B, N), ctr.data_ptr(), _offsets(B, M),
                               float(radius), S, idx.data_ptr(), hits.data_ptr(),
                               stream.cuda_stream)
    return (idx[0], hits[0]) if single else (idx, hits)


def gather_points(points, idx):
    """Coordinates of the points ``idx`` ((M,) or (B, M) int64) selects:
    (M, 3) or (B, M, 3)."""
    import torch
    pts, single = _cloud_batch(points, "points")
    if idx.dtype != torch.int64 or not idx.is_cuda:
        raise TypeError("idx must be an int64 CUDA tensor")
    ix = idx.unsqueeze(0) if single else idx
    if ix.dim() != 2 or ix.shape[0] != pts.shape[0]:
        raise ValueError("idx must have shape (M,) for (N, 3) points or (B, M) for (B, N, 3)")
    ix = ix.contiguous()
    B, N, M = int(pts.shape[0]), int(pts.shape[1]), int(ix.shape[1])
    out = torch.empty((B, M, 3), dtype=torch.float32, device=pts.device)
    with torch.cuda.device(pts.device):
        stream = torch.cuda.current_stream(pts.device)
        capi.gather_points_device(pts.data_ptr(), _offsets(B, N), ix.data_ptr(), _offsets(B, M),
                                  out.data_ptr(), stream.cuda_stream)
    return out[0] if single else out


def group_points(points, centers, idx):
    """``points[idx] - centers`` per group: (M, nsample, 3) or
    (B, M, nsample, 3), idx as returned by ``ball_query``."""
    import torch
    pts, single = _cloud_batch(points, "points")
    ctr, single_c = _cloud_batch(centers, "centers")
    if single != single_c or pts.shape[0] != ctr.shape[0]:
        raise ValueError("points and centers must have the same batch layout")
    if idx.dtype != torch.int64 or not idx.is_cuda:
        raise TypeError("idx must be an int64 CUDA tensor")
    ix = idx.unsqueeze(0) if single else idx
    if ix.dim() != 3 or ix.shape[0] != pts.shape[0] or ix.shape[1] != ctr.shape[1]:
        raise ValueError("idx must have shape (M, nsample) or (B, M, nsample)")
    ix = ix.contiguous()
    B, N, M, S = int(pts.shape[0]), int(pts.shape[1]), int(ctr.shape[1]), int(ix.shape[2])
    out = torch.empty((B, M, S, 3), dtype=torch.float32, device=pts.device)
    with torch.cuda.device(pts.device):
        stream = torch.cuda.current_stream(pts.device)
        capi.group_points_device(pts.data_ptr(), _offsets(B, N), ctr.data_ptr(), _offsets(B, M),
                                 S, ix.data_ptr(), out.data_ptr(), stream.cuda_stream)
    return out[0] if single else out
