"""The CTC argmax entry point that allocates nothing.

Some callers cannot allocate device memory: a host that owns a fixed
device-memory budget and hands every buffer out itself, or a loop that must
not stall on cudaMalloc / cudaFree (both can synchronize the whole device).
Those callers cannot use the model API, which allocates its tensors and
scratch. `ppocr_ctc_argmax_noalloc` runs the recogniser's CTC argmax head
over buffers the caller owns, with its scratch in a fixed array inside the
library.

The entry point is called in a fresh process that never builds a model (as
such a caller would: nothing else of the library has set the device up), on
buffers that process allocated itself, twice in a row (the second call finds
the first call's scratch contents). Both results are checked against the CPU
oracle and against the model API's output for the same head: classes
identical, 1 / sum within the 1e-5 the reference's own CTC test allows
(`src/engine/layers.rs:1313`). The same calls are then made in this process
after a model has run. The file runs last in the suite and also alone.
"""

from __future__ import annotations

import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest

from ppocr_native_b200.plan import Op, encode

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent

# The caller's side: its own buffers (cudaMalloc through the runtime it links),
# two calls of the entry point, nothing of the model API.
CALLER = textwrap.dedent("""
    import ctypes, glob, os, sys
    import numpy as np
    sys.path.insert(0, sys.argv[1])
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "ppocr_native_b200", os.path.join(sys.argv[1], "ppocr-native_b200", "__init__.py"),
        submodule_search_locations=[os.path.join(sys.argv[1], "ppocr-native_b200")])
    pkg = importlib.util.module_from_spec(spec); sys.modules["ppocr_native_b200"] = pkg; spec.loader.exec_module(pkg)
    from ppocr_native_b200 import cuda

    def cudart():
        here = os.path.dirname(np.__file__)
        for p in glob.glob(os.path.join(here, "..", "nvidia", "cuda_runtime", "lib", "libcudart.so*")) + [
                "libcudart.so.12", "/usr/local/cuda/lib64/libcudart.so"]:
            try:
                rt = ctypes.CDLL(p)
            except OSError:
                continue
            rt.cudaMalloc.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_size_t]
            rt.cudaFree.argtypes = [ctypes.c_void_p]
            rt.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
            return rt
        raise SystemExit("no libcudart for the caller's own buffers")

    data = np.load(sys.argv[2])
    t, ci, vocab = (int(v) for v in data["dims"])
    host = {"x": data["x"], "w": data["w"], "b": data["b"], "y": np.zeros((t, 2), np.float32)}
    rt = cudart()
    dev = {}
    outs = []
    try:
        for k, a in host.items():
            p = ctypes.c_void_p()
            assert rt.cudaMalloc(ctypes.byref(p), a.nbytes) == 0
            dev[k] = p.value
            assert rt.cudaMemcpy(dev[k], a.ctypes.data, a.nbytes, 1) == 0
        for call in range(2):
            cuda.ctc_argmax_noalloc(dev["x"], dev["w"], dev["b"], dev["y"], t, ci, vocab)
            got = np.zeros((t, 2), np.float32)
            # cudaMemcpy on the default stream waits for the call's kernels
            assert rt.cudaMemcpy(got.ctypes.data, dev["y"], got.nbytes, 2) == 0
            outs.append(got)
    finally:
        for p in dev.values():
            rt.cudaFree(p)
    np.save(sys.argv[3], np.stack(outs))
""")


def head(t: int, ci: int, vocab: int, seed: int = 5):
    rng = np.random.default_rng(seed)
    cols = -(-vocab // 16) * 16
    logical = rng.normal(0, ci ** -0.5, (ci, vocab)).astype(np.float32)
    full = np.zeros((ci, cols), np.float32)
    full[:, :vocab] = logical
    panels = np.ascontiguousarray(full.reshape(ci, cols // 16, 16).transpose(1, 0, 2))
    bias = np.full(cols, -1e30, np.float32)
    bias[:vocab] = rng.normal(0, 0.1, vocab).astype(np.float32)
    x = rng.normal(0, 1, (t, ci)).astype(np.float32)
    op = Op("ctcargmax", x=0, y=1, ic=ci, oc=2, n2=vocab, w=(0, panels.size), b=(panels.size, cols))
    plan = encode((0, 1, t, ci), 2, [1], [op], np.concatenate([panels.reshape(-1), bias]))
    return plan, x, panels, bias


def check(got: np.ndarray, want: np.ndarray, what: str) -> None:
    assert np.array_equal(got[:, 0], want[:, 0]), f"{what}: classes differ"
    gap = float(np.max(np.abs(got[:, 1].astype(np.float64) - want[:, 1])))
    assert gap <= 1e-5, f"{what}: 1/sum differs by {gap}"


def test_noalloc_ctc_argmax_in_a_fresh_process(cuda_mod, oracle_mod, tmp_path):
    t, ci, vocab = 300, 120, 18710
    plan, x, panels, bias = head(t, ci, vocab)
    inputs = tmp_path / "head.npz"
    np.savez(inputs, x=x, w=panels, b=bias, dims=np.array([t, ci, vocab]))
    result = tmp_path / "noalloc.npy"
    r = subprocess.run([sys.executable, "-c", CALLER, str(ROOT), str(inputs), str(result)],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    fresh = np.load(result)

    want_oracle = oracle_mod.Oracle(plan).run(x.reshape(-1))[0].reshape(t, 2)
    with cuda_mod.Model(plan) as m:
        m.input_mut()[:] = x.reshape(-1)
        m.run(60_000)
        want_model = m.output().copy().reshape(t, 2)
    for call in range(2):
        check(fresh[call], want_oracle, f"fresh process, call {call} vs the oracle")
        check(fresh[call], want_model, f"fresh process, call {call} vs the model API")


def test_noalloc_ctc_argmax_after_the_model_api(cuda_mod, oracle_mod):
    import ctypes
    import glob
    import os

    t, ci, vocab = 300, 120, 18710
    plan, x, panels, bias = head(t, ci, vocab, seed=6)
    want = oracle_mod.Oracle(plan).run(x.reshape(-1))[0].reshape(t, 2)
    with cuda_mod.Model(plan) as m:
        m.input_mut()[:] = x.reshape(-1)
        m.run(60_000)
        check(m.output().copy().reshape(t, 2), want, "model API vs the oracle")

    rt = None
    here = os.path.dirname(np.__file__)
    for p in glob.glob(os.path.join(here, "..", "nvidia", "cuda_runtime", "lib", "libcudart.so*")) + [
            "libcudart.so.12", "/usr/local/cuda/lib64/libcudart.so"]:
        try:
            rt = ctypes.CDLL(p)
            break
        except OSError:
            continue
    assert rt is not None, "no libcudart for the caller's own buffers"
    rt.cudaMalloc.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_size_t]
    rt.cudaFree.argtypes = [ctypes.c_void_p]
    rt.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    host = {"x": x, "w": panels, "b": bias, "y": np.zeros((t, 2), np.float32)}
    dev = {}
    try:
        for k, a in host.items():
            p = ctypes.c_void_p()
            assert rt.cudaMalloc(ctypes.byref(p), a.nbytes) == 0
            dev[k] = p.value
            assert rt.cudaMemcpy(dev[k], a.ctypes.data, a.nbytes, 1) == 0
        for call in range(2):
            cuda_mod.ctc_argmax_noalloc(dev["x"], dev["w"], dev["b"], dev["y"], t, ci, vocab)
            got = np.zeros((t, 2), np.float32)
            assert rt.cudaMemcpy(got.ctypes.data, dev["y"], got.nbytes, 2) == 0
            check(got, want, f"call {call} vs the oracle")
        # a call larger than the fixed scratch is refused before any work
        with pytest.raises(cuda_mod.PpocrError) as e:
            cuda_mod.ctc_argmax_noalloc(dev["x"], dev["w"], dev["b"], dev["y"], 10_000, ci, vocab)
        assert e.value.code == cuda_mod.E_SIZE
    finally:
        for p in dev.values():
            rt.cudaFree(p)
