"""The committed golden vectors (tests/golden/*.npz, written by
tests/golden/make_golden.py from the CPU oracle on the reference's test
miniatures and small cases of the benchmark configurations): the oracle
still reproduces them bit for bit (CPU), and the CUDA path matches them
without the oracle in the loop (GPU): bit for bit with every contraction on
the FP32 cores, within the tolerance on the tensor cores."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from common import max_gap
from ppocr_native_b200 import synth

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.stem for p in GOLDEN.glob("*.npz"))
TOL = 1e-4


def load(name: str):
    d = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(bytes(d["meta"]).decode())
    if meta["synth"] is None:
        plan = bytes(d["plan"])
    else:
        args = {k: tuple(v) if isinstance(v, list) else v for k, v in meta["args"].items()}
        plan = getattr(synth, meta["synth"])(**args)
    sizes = [tuple(int(v) for v in hw) for hw in d["sizes"]]
    xs = [d[f"x{n}"] for n in range(len(sizes))]
    ys = [d[f"y{n}"] for n in range(len(sizes))]
    return plan, sizes, xs, ys


def argmax_head(name: str) -> bool:
    return name.startswith(("rec", "line"))


def test_golden_cases_exist():
    assert {"page_model_16x16", "line_model_3_lanes", "fused_layer_8x12", "det_96x64", "rec_3_lanes"} <= set(CASES)


@pytest.mark.parametrize("name", CASES)
def test_oracle_reproduces_golden(oracle_mod, name):
    plan, sizes, xs, ys = load(name)
    o = oracle_mod.Oracle(plan)
    for (h, w), x, y in zip(sizes, xs, ys):
        o.set_size(h, w)
        assert np.array_equal(o.run(x)[0], y)


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_cuda_matches_golden(cuda_mod, name):
    plan, sizes, xs, ys = load(name)
    for options in (0, cuda_mod.OPT_NO_TENSOR_CORES):
        with cuda_mod.Model(plan) as m:
            if options:
                m.set_options(options)
            m.set_sizes(sizes)
            for n, x in enumerate(xs):
                m.lane_input_mut(n)[:] = x
            m.run(60_000)
            for n, y in enumerate(ys):
                got = m.lane_output(n).copy()
                assert got.shape == y.shape
                if argmax_head(name):
                    # (class, 1 / sum exp) per time step: classes identical
                    g, w = got.reshape(-1, 2), y.reshape(-1, 2)
                    assert np.array_equal(g[:, 0], w[:, 0])
                    assert max_gap(g[:, 1], w[:, 1]) <= 1e-5
                elif options:
                    assert np.array_equal(got, y), max_gap(got, y)
                else:
                    assert max_gap(got, y) <= TOL * max(1.0, float(np.abs(y).max()))
