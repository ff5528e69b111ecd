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
