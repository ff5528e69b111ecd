"""Recogniser logits at network level (benchmark config 3): 16 lines of
48 x 320, and lanes of mixed widths, through the whole recogniser (stem,
depthwise-separable blocks, SE, pooling, two SVTR blocks with LayerNorm and
8-head attention, final LayerNorm) ending in the CTC head's logits (a 1x1
conv 120 -> 18 710), on the tensor-core path (3xTF32) against the CPU
oracle: |logit difference| <= 1e-4 absolute, the bound the north-star
specification states for recogniser logits. Weights N(0, 0.02) as config 3
states, and fan-in scaled weights (activations of order one through the
depth)."""

from __future__ import annotations

import numpy as np
import pytest

from ppocr_native_b200 import synth

pytestmark = pytest.mark.gpu

TOL = 1e-4


@pytest.mark.parametrize("std", [0.02, None])
@pytest.mark.parametrize("widths", [[320] * 16, [320, 96, 1280, 640, 320, 48 * 7]])
def test_recogniser_logits_within_1e4(cuda_mod, oracle_mod, std, widths):
    plan = synth.rec_plan(seed=3, std=std, logits=True)
    rng = np.random.default_rng(len(widths))
    xs = [rng.standard_normal(48 * w * 3).astype(np.float32) for w in widths]
    with cuda_mod.Model(plan) as m:
        m.set_sizes([(48, w) for w in widths])
        for i, x in enumerate(xs):
            m.lane_input_mut(i)[:] = x
        m.run(120_000)
        got = [m.lane_output(i).copy() for i in range(len(widths))]
    o = oracle_mod.Oracle(plan)
    worst = 0.0
    for w, x, g in zip(widths, xs, got):
        o.set_size(48, w)
        want = o.run(x)[0]
        assert g.shape == want.shape and np.isfinite(g).all()
        worst = max(worst, float(np.max(np.abs(g.astype(np.float64) - want))))
    assert worst <= TOL, worst
