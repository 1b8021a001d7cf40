"""The reference's evaluation GPU sampler, built from its own sources
(oracle/Makefile), runs here as a reported baseline: it returns K distinct
indices starting at point 0 (eval/src_gpu/yuezu_fps_gpu_optimized.cu:989-1061),
and on the c1 cloud it agrees with the bit-exact engine for a prefix of the
samples (its distances may be contracted, so not necessarily all)."""
import numpy as np
import pytest

from ns_fps_b200 import synthetic
from tests import capi, ref_eval_gpu

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not ref_eval_gpu.available(),
                       reason="oracle/_ref/libref_eval_gpu.so not built (the reference sources were absent)"),
]


def test_reference_eval_sampler_runs_beside_the_engine():
    c = synthetic.CONFIGS["c1"]
    cl = synthetic.make("c1", seed=0)[0]
    idx, init_ms, sample_ms = ref_eval_gpu.fps(cl, c.k, c.rng, c.blocks)
    assert len(idx) == c.k
    assert idx[0] == 0
    assert len(np.unique(idx)) == c.k
    assert init_ms > 0.0 and sample_ms > 0.0
    ours = capi.fps(cl, c.k, c.rng, c.blocks)
    assert ref_eval_gpu.shared_prefix(idx, ours) >= 2
