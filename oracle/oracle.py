"""TEST INFRASTRUCTURE ONLY: ctypes access to the CPU oracle
(`oracle/libppocr_oracle.so`, a C restatement of ppocr-native's CPU engine).

Only tests/, `__graft_entry__.smoke()` and bench.py's CPU baseline use this;
the product library never does. `build()` compiles the library with the
recipe in `oracle/Makefile`.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "libppocr_oracle.so"


def build(force: bool = False) -> Path:
    """Compile the oracle (gcc, -O3 -mavx2 -mfma -fopenmp -ffp-contract=off)."""
    src = [HERE / "ppocr_oracle.c", HERE / "ppocr_oracle.h", HERE / "Makefile"]
    if force or not LIB.exists() or any(s.stat().st_mtime > LIB.stat().st_mtime for s in src):
        subprocess.run(["make", "-s", "-C", str(HERE), "libppocr_oracle.so"], check=True)
    return LIB


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = ctypes.CDLL(str(LIB))
        L.orc_load.restype = ctypes.c_void_p
        L.orc_load.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t]
        L.orc_free.argtypes = [ctypes.c_void_p]
        L.orc_set_size.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t,
                                   ctypes.c_char_p, ctypes.c_size_t]
        L.orc_input_len.restype = ctypes.c_size_t
        L.orc_input_len.argtypes = [ctypes.c_void_p]
        L.orc_output_count.restype = ctypes.c_size_t
        L.orc_output_count.argtypes = [ctypes.c_void_p]
        L.orc_output_len.restype = ctypes.c_size_t
        L.orc_output_len.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
        L.orc_run.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        L.orc_exp_neg.restype = ctypes.c_float
        L.orc_exp_neg.argtypes = [ctypes.c_float]
        L.orc_activation.restype = ctypes.c_float
        L.orc_activation.argtypes = [ctypes.c_int, ctypes.c_float]
        L.orc_rec_input_hwc.restype = ctypes.c_size_t
        L.orc_rec_input_hwc.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p]
        L.orc_det_input_hwc.restype = ctypes.c_int
        L.orc_det_input_hwc.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                                        ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        _lib = L
    return _lib


class OracleError(RuntimeError):
    pass


class Oracle:
    """A plan on the CPU oracle: `run(image)` gives the outputs."""

    def __init__(self, plan: bytes):
        err = ctypes.create_string_buffer(512)
        self._p = lib().orc_load(plan, len(plan), err, 512)
        if not self._p:
            raise OracleError(err.value.decode())

    def __del__(self):
        if getattr(self, "_p", None):
            lib().orc_free(self._p)
            self._p = None

    def set_size(self, h: int, w: int) -> None:
        err = ctypes.create_string_buffer(512)
        if lib().orc_set_size(self._p, h, w, err, 512) != 0:
            raise OracleError(err.value.decode())

    @property
    def input_len(self) -> int:
        return lib().orc_input_len(self._p)

    def output_len(self, k: int = 0) -> int:
        return lib().orc_output_len(self._p, k)

    def run(self, image: np.ndarray, threads: int = 0) -> list[np.ndarray]:
        x = np.ascontiguousarray(image, dtype=np.float32).reshape(-1)
        if x.size != self.input_len:
            raise OracleError(f"input holds {x.size} floats, the plan wants {self.input_len}")
        n = lib().orc_output_count(self._p)
        outs = [np.empty(self.output_len(k), np.float32) for k in range(n)]
        ptrs = (ctypes.c_void_p * max(n, 1))(*[o.ctypes.data for o in outs])
        if lib().orc_run(self._p, x.ctypes.data, ptrs, int(threads)) != 0:
            raise OracleError("oracle run failed")
        return outs


def exp_neg(z: float) -> float:
    return lib().orc_exp_neg(z)


def activation(code: int, x: float) -> float:
    return lib().orc_activation(code, x)


def det_input_hwc(image: np.ndarray, ow: int, oh: int, mean, std) -> np.ndarray:
    """The detector input of an (ih, iw, 3) uint8 image at ow x oh,
    (oh, ow, 3) float32 (orc_det_input_hwc)."""
    image = np.ascontiguousarray(image, dtype=np.uint8)
    ih, iw, _ = image.shape
    out = np.empty((oh, ow, 3), np.float32)
    m = np.asarray(mean, np.float64)
    s = np.asarray(std, np.float64)
    if lib().orc_det_input_hwc(image.ctypes.data, iw, ih, ow, oh, m.ctypes.data, s.ctypes.data, out.ctypes.data):
        raise OracleError("empty size")
    return out


def rec_input_hwc(crop: np.ndarray) -> np.ndarray:
    """The recogniser's input of an (h, w, 3) uint8 crop, (48, width, 3)
    float32 (orc_rec_input_hwc)."""
    crop = np.ascontiguousarray(crop, dtype=np.uint8)
    ch, cw, _ = crop.shape
    width = lib().orc_rec_input_hwc(crop.ctypes.data, cw, ch, None)
    if not width:
        raise OracleError("empty crop")
    out = np.empty((48, width, 3), np.float32)
    lib().orc_rec_input_hwc(crop.ctypes.data, cw, ch, out.ctypes.data)
    return out


def threads_available() -> int:
    return len(os.sched_getaffinity(0))
