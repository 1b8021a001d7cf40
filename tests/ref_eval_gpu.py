"""The reference's evaluation GPU sampler (satreeby/ns_fps
eval/src_gpu/yuezu_fps_gpu_optimized.cu), timed beside this engine on the same
synthetic inputs: a reported GPU baseline.  It is not bit-exact with the
reference's CPU sampler (its distances start from 1e30, its cube is one cell
wider, and nvcc may contract its distance sums), so only timing and the length
of the prefix it shares with the bit-exact engine are reported.

Test infrastructure: it loads oracle/_ref/libref_eval_gpu.so (built by
oracle/Makefile from the reference's sources) and is never imported by the
product.  Run on a GPU host as

    python -m tests.ref_eval_gpu [c1 c2 c3 c4] [--reps 3]

which prints one JSON line per config: the reference sampler's initialize /
sample / total host wall times (median over reps, after one warm-up), this
engine's host-to-host time for the same cloud through nsfps_fps, and the
shared prefix.  c3 runs its 32 clouds one after another (the reference
sampler takes one cloud per call).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import time

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "oracle", "_ref", "libref_eval_gpu.so")
_lib = None


def available() -> bool:
    return os.path.exists(LIB_PATH)


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(LIB_PATH)
        f = _lib.ref_eval_gpu_fps
        f.restype = ctypes.c_int
        f.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_void_p,
                      ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64),
                      ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]
    return _lib


def fps(points: np.ndarray, k: int, bounds, blocks):
    """Indices from the reference's FpsGPU, plus (init_ms, sample_ms)."""
    pts = np.ascontiguousarray(points, dtype=np.float32)
    r6 = np.asarray(bounds, dtype=np.float32)
    b3 = np.asarray(blocks, dtype=np.uint32)
    out = np.zeros(max(int(k), 1), dtype=np.uint64)
    n_out = ctypes.c_uint64(0)
    ti, ts = ctypes.c_double(0.0), ctypes.c_double(0.0)
    rc = lib().ref_eval_gpu_fps(pts.ctypes.data, pts.shape[0], int(k), r6.ctypes.data,
                                b3.ctypes.data, out.ctypes.data, ctypes.byref(n_out),
                                ctypes.byref(ti), ctypes.byref(ts))
    if rc != 0:
        raise RuntimeError(f"ref_eval_gpu_fps rc={rc}")
    return out[: n_out.value].copy(), ti.value, ts.value


def shared_prefix(a: np.ndarray, b: np.ndarray) -> int:
    m = min(len(a), len(b))
    diff = np.nonzero(a[:m] != b[:m])[0]
    return int(diff[0]) if len(diff) else m


def run(config: str, reps: int = 3, seed: int = 0) -> dict:
    from ns_fps_b200 import capi, synthetic

    c = synthetic.CONFIGS[config]
    clouds = synthetic.make(config, seed)
    ref_i, ref_s, ref_t, ours = [], [], [], []
    prefix = []
    for rep in range(reps + 1):
        ti_sum = ts_sum = 0.0
        t_ours = 0.0
        for cl in clouds:
            idx_ref, ti, ts = fps(cl, c.k, c.rng, c.blocks)
            ti_sum += ti
            ts_sum += ts
            t0 = time.perf_counter()
            idx_ours = capi.fps(cl, c.k, c.rng, c.blocks)
            t_ours += (time.perf_counter() - t0) * 1e3
            if rep == 0:
                prefix.append(shared_prefix(idx_ref, np.asarray(idx_ours, dtype=np.uint64)))
        if rep == 0:
            continue  # warm-up
        ref_i.append(ti_sum)
        ref_s.append(ts_sum)
        ref_t.append(ti_sum + ts_sum)
        ours.append(t_ours)
    return {
        "config": config, "clouds": len(clouds), "n": c.n, "k": c.k, "reps": reps,
        "ref_eval_gpu_init_ms": statistics.median(ref_i),
        "ref_eval_gpu_sample_ms": statistics.median(ref_s),
        "ref_eval_gpu_total_ms": statistics.median(ref_t),
        "nsfps_host_to_host_ms": statistics.median(ours),
        "shared_prefix_min": min(prefix), "shared_prefix_of": c.k,
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("configs", nargs="*", default=["c1", "c2", "c3", "c4"])
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    for cfg in args.configs:
        print(json.dumps(run(cfg, args.reps)), flush=True)


if __name__ == "__main__":
    main()
