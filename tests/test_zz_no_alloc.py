"""The CTC argmax entry point that allocates nothing.

Callers that manage a fixed device-memory budget themselves, or that must
not stall on cudaMalloc / cudaFree, cannot use the model API (it allocates
its tensors and scratch). `ppocr_ctc_argmax_noalloc` runs the recogniser's
CTC argmax head over buffers the caller owns, with its scratch in a fixed
array inside the library. This test allocates the caller's buffers itself,
runs the entry point twice in a row (the second call finds the first one's
scratch contents) and checks both results against the model API's output for
the same head: classes identical, 1 / sum within the 1e-5 the reference's
own CTC test allows. It runs last in the suite (file name) and also alone.
"""

from __future__ import annotations

import ctypes
import glob
import os

import numpy as np
import pytest

from ppocr_native_b200.plan import Op, encode

pytestmark = pytest.mark.gpu


def _cudart():
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
    pytest.fail("no libcudart for the caller's own buffers")


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


def test_noalloc_ctc_argmax_matches_model_api(cuda_mod):
    t, ci, vocab = 300, 120, 18710
    plan, x, panels, bias = head(t, ci, vocab)
    with cuda_mod.Model(plan) as m:
        m.input_mut()[:] = x.reshape(-1)
        m.run(60_000)
        want = m.output().copy().reshape(t, 2)

    rt = _cudart()
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
            # cudaMemcpy on the default stream waits for the call's kernels
            assert rt.cudaMemcpy(got.ctypes.data, dev["y"], got.nbytes, 2) == 0
            assert np.array_equal(got[:, 0], want[:, 0]), f"call {call}: classes differ"
            assert float(np.max(np.abs(got[:, 1] - want[:, 1]))) <= 1e-5, f"call {call}"
        # a call larger than the fixed scratch is refused before any work
        with pytest.raises(cuda_mod.PpocrError) as e:
            cuda_mod.ctc_argmax_noalloc(dev["x"], dev["w"], dev["b"], dev["y"], 10_000, ci, vocab)
        assert e.value.code == cuda_mod.E_SIZE
    finally:
        for p in dev.values():
            rt.cudaFree(p)
