"""Failure paths of the engine, driven without faulting the GPU.

The reference's GPU prototype ignores every CUDA error
(eval/src_gpu/yuezu_fps_gpu_optimized.cu:904-910) and its CPU path has no
failure mode, so these pin this engine's own contract:

* every in-kernel wait is bounded: one CTA of a cloud withholds its candidate
  list (round loops) or its proposals (per-step loop) at one round / step --
  a flag nothing else sets -- so every wait for it runs out; the call must
  return NSFPS_ERR_TIMEOUT, and the next call on the same device must return
  the oracle's samples (the context is still usable).  This runs each loop
  variant: the grid-wide round loop (lists in global memory; a single
  cloud), the round loop in thread-block clusters (a batch of two clouds,
  one cluster each) and the per-step loop (both writing into other CTAs'
  shared memory, so their exit must wait for every CTA);
* a workspace request that fails returns NSFPS_ERR_OOM with a message, also
  from one worker thread of the multi-device sharder, and the next call
  succeeds;
* the sharder itself, run with two device entries (the same GPU twice when
  the box has one), returns every cloud's oracle samples.
"""
import numpy as np
import pytest

import oracle
from ns_fps_b200 import synthetic as S
from tests import capi

pytestmark = pytest.mark.gpu

MODE_LOOP, MODE_ROUNDS, MODE_GRID = 0, 2, 3
WAIT_NS = 200_000_000  # 0.2 s per bounded wait in these tests


@pytest.fixture(autouse=True)
def _reset_hooks():
    capi.set_test_hooks(reset=True)
    yield
    capi.set_test_hooks(reset=True)


def _profiled(fn):
    capi.set_profiling(True)
    try:
        out = fn()
        return out, capi.last_profile()
    finally:
        capi.set_profiling(False)


def _cases():
    c2 = S.CONFIGS["c2"]
    scan = S.lidar_scan(seed=21)                       # 122,880 points: grid-wide loop
    c1 = S.CONFIGS["c1"]
    gauss = [S.gaussian_cloud(c1.n, 5), S.gaussian_cloud(c1.n, 6)]  # a cluster each
    rs = np.random.RandomState(9)
    hashed = (rs.rand(6000, 3) * [3, 5, 7]).astype(np.float32)
    return {
        "grid": (scan, 3000, c2.rng, c2.blocks, MODE_GRID, 7, 3),
        "cluster": (gauss, 800, c1.rng, c1.blocks, MODE_ROUNDS, 1, 2),
        "step": (hashed, 700, (0, 3, 0, 5, 0, 7), (6, 10, 12), MODE_LOOP, 0, 5),
    }


@pytest.mark.parametrize("variant", ["grid", "cluster", "step"])
def test_withheld_exchange_times_out_and_device_recovers(variant):
    clouds, k, bounds, blocks, mode, cta, step = _cases()[variant]
    if not isinstance(clouds, list):
        clouds = [clouds]
    exp = [oracle.fps(c, k, bounds, blocks) for c in clouds]
    run = lambda: capi.fps_batched(clouds, k, bounds, blocks)

    def check(got):
        for g, e in zip(got, exp):
            np.testing.assert_array_equal(g, e)
    # the layout under test is the one that runs
    got, prof = _profiled(run)
    assert prof.mode == mode, f"expected loop mode {mode}, ran {prof.mode}"
    assert prof.ctas_per_cloud > cta
    check(got)

    capi.set_test_hooks(wait_limit_ns=WAIT_NS, withhold_cta=cta, withhold_step=step)
    with pytest.raises(RuntimeError, match=f"rc={capi.ERR_TIMEOUT}.*timed out"):
        run()
    capi.set_test_hooks(reset=True)
    # the same device, the next call: exact samples again (twice)
    for _ in range(2):
        check(run())


def test_withhold_after_the_last_round_changes_nothing():
    """A hook aimed at a round the call never reaches leaves the call alone."""
    clouds, k, bounds, blocks, _, cta, _ = _cases()["cluster"]
    capi.set_test_hooks(wait_limit_ns=WAIT_NS, withhold_cta=cta, withhold_step=1_000_000)
    got = capi.fps_batched(clouds, k, bounds, blocks)
    for g, c in zip(got, clouds):
        np.testing.assert_array_equal(g, oracle.fps(c, k, bounds, blocks))


def test_failed_workspace_request_returns_oom_then_recovers():
    pts, k, bounds, blocks, _, _, _ = _cases()["cluster"]
    pts = pts[0]
    exp = oracle.fps(pts, k, bounds, blocks)
    capi.set_test_hooks(fail_alloc_device=0)
    with pytest.raises(RuntimeError, match=f"rc={capi.ERR_OOM}.*injected"):
        capi.fps(pts, k, bounds, blocks)
    # one-shot: the next call runs normally
    np.testing.assert_array_equal(capi.fps(pts, k, bounds, blocks), exp)


def _sharder_devices():
    import torch
    return (0, 1) if torch.cuda.device_count() >= 2 else (0, 0)


def test_sharder_two_device_entries_match_oracle():
    """nsfps_fps_batched deals whole clouds round-robin over its device list,
    one host thread per entry; two entries naming the same GPU share its
    context and run one after the other."""
    cfg = S.CONFIGS["c3"]
    clouds = S.make("c3", seed=41, count=5)
    devs = _sharder_devices()
    got = capi.fps_batched(clouds, cfg.k, cfg.rng, cfg.blocks, devices=devs)
    for i, cl in enumerate(clouds):
        np.testing.assert_array_equal(got[i], oracle.fps(cl, cfg.k, cfg.rng, cfg.blocks),
                                      err_msg=f"cloud {i} on device {devs[i % 2]}")


def test_sharder_worker_failure_is_reported_then_recovers():
    cfg = S.CONFIGS["c3"]
    clouds = S.make("c3", seed=42, count=4)
    devs = _sharder_devices()
    capi.set_test_hooks(fail_alloc_device=devs[0])
    with pytest.raises(RuntimeError, match=f"rc={capi.ERR_OOM}.*device {devs[0]}.*injected"):
        capi.fps_batched(clouds, cfg.k, cfg.rng, cfg.blocks, devices=devs)
    got = capi.fps_batched(clouds, cfg.k, cfg.rng, cfg.blocks, devices=devs)
    for i, cl in enumerate(clouds):
        np.testing.assert_array_equal(got[i], oracle.fps(cl, cfg.k, cfg.rng, cfg.blocks))


def test_withheld_list_in_cta_groups_times_out_and_recovers():
    """Groups of 4 CTAs over more clouds than groups: group 0 withholds a list
    on its first cloud; its waits run out while the other groups finish; the
    call reports the timeout and the next call is exact."""
    import os
    cfg = S.CONFIGS["c3"]
    clouds = [S.sphere_cube_cloud(4096, seed=70 + i) for i in range(40)]
    k = 500
    os.environ["NSFPS_BATCH_GROUP_CTAS"] = "4"
    try:
        capi.set_test_hooks(wait_limit_ns=WAIT_NS, withhold_cta=2, withhold_step=1)
        with pytest.raises(RuntimeError, match=f"rc={capi.ERR_TIMEOUT}.*timed out"):
            capi.fps_batched(clouds, k, cfg.rng, cfg.blocks)
        capi.set_test_hooks(reset=True)
        got = capi.fps_batched(clouds, k, cfg.rng, cfg.blocks)
    finally:
        os.environ.pop("NSFPS_BATCH_GROUP_CTAS", None)
    for i in (0, 1, 37, 39):
        np.testing.assert_array_equal(got[i], oracle.fps(clouds[i], k, cfg.rng, cfg.blocks))
