"""Shared test helpers: the reference tests' deterministic inputs and small
single-operation plans."""

from __future__ import annotations

import numpy as np

from ppocr_native_b200.plan import Op, encode, window


def noise(n: int, seed: int, scale: float) -> np.ndarray:
    """Deterministic values in [-scale, scale): the xorshift generator of the
    reference tests (`src/engine/layers.rs:1082-1092`)."""
    state = (seed | 1) & 0xFFFFFFFF
    out = np.empty(n, np.float32)
    for i in range(n):
        state ^= (state << 13) & 0xFFFFFFFF
        state ^= state >> 17
        state ^= (state << 5) & 0xFFFFFFFF
        out[i] = (np.float32(state >> 8) / np.float32(8388608.0) - np.float32(1.0)) * np.float32(scale)
    return out


def rng_values(n: int, seed: int, scale: float = 1.0) -> np.ndarray:
    return (np.random.default_rng(seed).uniform(-1, 1, n) * scale).astype(np.float32)


def single(op: Op, input_shape, weights: np.ndarray, buffers: int | None = None, second=None) -> bytes:
    """A plan of one op from buffer 0 (the image) to buffer 1, or of a
    producer for the second input followed by the op."""
    h, w, c = input_shape
    if second is None:
        return encode((0, h, w, c), buffers or 2, [op.y], [op], weights)
    return encode((0, h, w, c), buffers or 3, [op.y], [second, op], weights)


def max_gap(a: np.ndarray, b: np.ndarray) -> float:
    assert a.shape == b.shape
    assert np.isfinite(a).all() and np.isfinite(b).all()
    return float(np.max(np.abs(a.astype(np.float64) - b.astype(np.float64)))) if a.size else 0.0


__all__ = ["noise", "rng_values", "single", "max_gap", "Op", "window", "encode"]


# ------------------------------------------------ device buffers for tests

def cudart():
    """The CUDA runtime through ctypes, for tests that hold device buffers of
    their own (the C ABI's entry points take device pointers)."""
    import ctypes
    import glob
    import os

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
        rt.cudaMemset.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t]
        rt.cudaDeviceSynchronize.argtypes = []
        return rt
    raise RuntimeError("no libcudart for the test's device buffers")


class Device:
    """Device buffers a test owns: `put(array)` copies a host array in and
    returns its pointer, `alloc(nbytes)` reserves one, `get(ptr, like)` copies
    one back; everything is freed on exit."""

    def __init__(self):
        self.rt = cudart()
        self.ptrs = []

    def __enter__(self):
        return self

    def alloc(self, nbytes: int) -> int:
        import ctypes

        p = ctypes.c_void_p()
        assert self.rt.cudaMalloc(ctypes.byref(p), max(int(nbytes), 1)) == 0
        self.ptrs.append(p.value)
        return p.value

    def put(self, a: np.ndarray) -> int:
        a = np.ascontiguousarray(a)
        p = self.alloc(a.nbytes)
        assert self.rt.cudaMemcpy(p, a.ctypes.data, a.nbytes, 1) == 0
        return p

    def get(self, p: int, shape, dtype) -> np.ndarray:
        out = np.empty(shape, dtype)
        assert self.rt.cudaMemcpy(out.ctypes.data, p, out.nbytes, 2) == 0
        return out

    def __exit__(self, *exc):
        for p in self.ptrs:
            self.rt.cudaFree(p)
        self.ptrs = []
