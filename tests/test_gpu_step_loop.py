"""The per-step loop (fps_loop_cluster, selected for every grid by
NSFPS_STEP_LOOP=1) and the round-based loop (fps_rounds_cluster, the default
for grids whose buckets are their cells) return identical samples.

The variable is read once per process, so each engine runs in its own
subprocess; both are compared with each other and with the oracle."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from ns_fps_b200 import synthetic

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

RUNNER = r"""
import json, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
from ns_fps_b200 import capi
d = np.load(sys.argv[2])
spec = json.loads(sys.argv[3])
out = {}
capi.set_profiling(True)
for name, (k, bounds, blocks) in spec.items():
    r = capi.fps(d[name], k, bounds, blocks)
    out[name] = r
    out[name + "_mode"] = np.array([capi.last_profile().mode])
np.savez(sys.argv[4], **out)
"""


def _run(tmp_path, clouds, spec, env_extra, tag):
    inp = tmp_path / "in.npz"
    np.savez(inp, **clouds)
    outp = tmp_path / f"out_{tag}.npz"
    env = dict(os.environ)
    env.pop("NSFPS_STEP_LOOP", None)
    env.update(env_extra)
    subprocess.run([sys.executable, "-c", RUNNER, ROOT, str(inp), json.dumps(spec), str(outp)],
                   check=True, env=env, timeout=600)
    return np.load(outp)


def test_step_loop_matches_round_loop(tmp_path):
    import oracle
    c1 = synthetic.make("c1", seed=3, count=1)[0]
    lidar = synthetic.lidar_scan(seed=5)[:40_000]
    sphere = synthetic.sphere_cube_cloud(16_384, seed=6)
    clouds = {"c1": c1, "lidar": lidar, "sphere": sphere}
    b = lambda p: [float(v) for v in (p[:, 0].min() - 1e-3, p[:, 0].max() + 1e-3,
                                      p[:, 1].min() - 1e-3, p[:, 1].max() + 1e-3,
                                      p[:, 2].min() - 1e-3, p[:, 2].max() + 1e-3)]
    spec = {"c1": [1000, [-4, 4, -4, 4, -4, 4], [16, 16, 16]],
            "lidar": [4096, b(lidar), [32, 32, 8]],
            "sphere": [2048, b(sphere), [16, 16, 16]]}
    rounds = _run(tmp_path, clouds, spec, {}, "rounds")
    steps = _run(tmp_path, clouds, spec, {"NSFPS_STEP_LOOP": "1"}, "steps")
    for name, (k, bounds, blocks) in spec.items():
        assert int(rounds[name + "_mode"][0]) in (2, 3), name  # a round-based loop ran
        assert int(steps[name + "_mode"][0]) == 0, name   # the per-step loop ran
        np.testing.assert_array_equal(rounds[name], steps[name], err_msg=name)
        if name == "c1":
            np.testing.assert_array_equal(rounds[name], oracle.fps(clouds[name], k, bounds, blocks))


def test_grid_wide_round_loop_matches_oracle():
    """A single cloud too large for one cluster's shared memory runs the
    round loop over co-resident CTAs (lists through global memory)."""
    import oracle
    from tests import capi
    pts = synthetic.cluster_cloud(n=400_000, seed=21, n_clusters=20)
    bounds = (-100, 100, -100, 100, -100, 100)
    blocks = (32, 32, 32)
    capi.set_profiling(True)
    got = capi.fps(pts, 3000, bounds, blocks)
    assert capi.last_profile().mode == 3  # the grid-wide round loop ran
    assert capi.last_profile().ctas_per_cloud > 16
    np.testing.assert_array_equal(got, oracle.fps(pts, 3000, bounds, blocks))
