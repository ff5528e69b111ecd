"""Writes the golden vectors under tests/golden/: inputs and outputs of the
CPU oracle (oracle/ppocr_oracle.c, the C restatement of the reference engine,
itself pinned to the reference's known-answer tests in tests/test_oracle.py)
on the reference's own test miniatures and on small cases of the benchmark
configurations. The GPU tests compare the CUDA path with these files without
running the oracle; the CPU tests check that the oracle still reproduces them
bit for bit.

    python tests/golden/make_golden.py

Each case is one .npz: `plan` (the PPOCRPL1 bytes, or empty when the plan is
rebuilt from `synth` with the stored `synth` and `args`), `sizes` (per lane
h, w), `x<n>` (lane n's input) and `y<n>` (lane n's output).
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(ROOT))

import conftest  # noqa: E402  (loads the package by path)
from ppocr_native_b200 import synth  # noqa: E402


def plan_of(case: dict) -> bytes:
    if case["synth"] is None:
        return case["plan"]
    return getattr(synth, case["synth"])(**case["args"])


def cases() -> list[dict]:
    rng = np.random.default_rng(20250101)
    out = []
    # the reference's engine test miniatures (src/engine/mod.rs:1374-1468)
    # with its input fill cos(0.013 i)
    for h, w in ((16, 16), (40, 8)):
        out.append(dict(name=f"page_model_{h}x{w}", synth=None, args={}, plan=synth.page_model_plan(16, 16),
                        sizes=[(h, w)], xs=[synth.ramp_input(h * w * 3)]))
    widths = [40, 17, 96]
    out.append(dict(name="line_model_3_lanes", synth=None, args={}, plan=synth.line_model_plan(40),
                    sizes=[(2, w) for w in widths], xs=[synth.stripes(2, w, phase=5 * i) for i, w in enumerate(widths)]))
    # benchmark config 1 (the fused depthwise 5x5 -> pointwise 96 -> 192
    # layer) at 8 x 12, input ~U(-1, 1)
    out.append(dict(name="fused_layer_8x12", synth="fused_layer_plan", args=dict(seed=0, h=8, w=12), plan=None,
                    sizes=[(8, 12)], xs=[rng.uniform(-1, 1, 8 * 12 * 96).astype(np.float32)]))
    # the detector and recogniser architectures at small sizes (weights
    # N(0, 0.02) from the seed), inputs ~N(0, 1)
    out.append(dict(name="det_96x64", synth="det_plan", args=dict(seed=3, size=(96, 64)), plan=None,
                    sizes=[(96, 64)], xs=[rng.standard_normal(96 * 64 * 3).astype(np.float32)]))
    rw = [64, 200, 33]
    out.append(dict(name="rec_3_lanes", synth="rec_plan", args=dict(seed=4, width=64), plan=None,
                    sizes=[(48, w) for w in rw], xs=[rng.standard_normal(48 * w * 3).astype(np.float32) for w in rw]))
    return out


def main() -> None:
    import oracle.oracle as oracle_mod

    oracle_mod.build()
    for case in cases():
        plan = plan_of(case)
        o = oracle_mod.Oracle(plan)
        arrays = {"plan": np.frombuffer(case["plan"] or b"", np.uint8),
                  "sizes": np.array(case["sizes"], np.int64),
                  "meta": np.frombuffer(json.dumps({"synth": case["synth"], "args": case["args"]}).encode(), np.uint8)}
        for n, ((h, w), x) in enumerate(zip(case["sizes"], case["xs"])):
            o.set_size(h, w)
            arrays[f"x{n}"] = x
            arrays[f"y{n}"] = o.run(x)[0]
        np.savez_compressed(HERE / f"{case['name']}.npz", **arrays)
        print(case["name"], {k: v.shape for k, v in arrays.items()})


if __name__ == "__main__":
    main()
