"""ctypes binding of libppocr_cuda.so (`include/ppocr_cuda.h`), shaped like
the reference's `GpuModel` (ppocr-native `src/engine/gpu/mod.rs:81-291`):
load, set_input_size / set_sizes, input_mut / lane_input_mut, run, output /
lane_output.

There is no fallback: without the built library (ppocr-native_b200/build.py)
or without a CUDA device every call raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "libppocr_cuda.so"

OK, E_PLAN, E_SIZE, E_NOMEM, E_DEVICE, E_TIMEOUT, E_UNSUPPORTED, E_ARG = range(8)
OPT_NO_FUSION, OPT_NO_GRAPH, OPT_NO_TENSOR_CORES = 1, 2, 4

# The exported C entry points and their signatures; tests check the library
# exports every one the header declares.
_SIG = {
    "ppocr_device_count": (ctypes.c_int, []),
    "ppocr_last_error": (ctypes.c_char_p, []),
    "ppocr_model_load": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]),
    "ppocr_model_load_bytes": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_int,
                                              ctypes.POINTER(ctypes.c_void_p)]),
    "ppocr_model_share_weights": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "ppocr_model_free": (None, [ctypes.c_void_p]),
    "ppocr_model_device_name": (ctypes.c_char_p, [ctypes.c_void_p]),
    "ppocr_model_integrated": (ctypes.c_int, [ctypes.c_void_p]),
    "ppocr_model_max_lanes": (ctypes.c_size_t, [ctypes.c_void_p]),
    "ppocr_model_output_count": (ctypes.c_size_t, [ctypes.c_void_p]),
    "ppocr_model_set_input_size": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32]),
    "ppocr_model_set_sizes": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32), ctypes.c_size_t]),
    "ppocr_model_lane_input": (ctypes.POINTER(ctypes.c_float),
                               [ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    "ppocr_model_lane_output": (ctypes.POINTER(ctypes.c_float),
                                [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    "ppocr_model_run": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32]),
    "ppocr_model_enqueue": (ctypes.c_int, [ctypes.c_void_p]),
    "ppocr_model_wait": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32]),
    "ppocr_model_lane_device_input": (ctypes.c_void_p,
                                      [ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    "ppocr_model_lane_device_output": (ctypes.c_void_p, [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t,
                                                         ctypes.POINTER(ctypes.c_size_t)]),
    "ppocr_model_enqueue_device": (ctypes.c_int, [ctypes.c_void_p]),
    "ppocr_model_stream": (ctypes.c_void_p, [ctypes.c_void_p]),
    "ppocr_model_set_stream": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "ppocr_model_set_options": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32]),
    "ppocr_model_launches": (ctypes.c_size_t, [ctypes.c_void_p]),
    "ppocr_model_step_name": (ctypes.c_char_p, [ctypes.c_void_p, ctypes.c_size_t]),
    "ppocr_ctc_argmax_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t,
                                                ctypes.c_size_t, ctypes.c_void_p]),
    "ppocr_rec_input_hwc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p,
                                           ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t), ctypes.c_void_p]),
    "ppocr_db_mask": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_float, ctypes.c_void_p,
                                     ctypes.c_void_p]),
    "ppocr_det_input_hwc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                                           ctypes.c_size_t, ctypes.POINTER(ctypes.c_double),
                                           ctypes.POINTER(ctypes.c_double), ctypes.c_void_p, ctypes.c_size_t,
                                           ctypes.c_void_p]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library; raises when it was not built."""
    global _lib
    if _lib is None:
        path = Path(os.environ.get("PPOCR_CUDA_LIB", LIB))
        if not path.exists():
            raise RuntimeError(f"{path} is missing: build it with ppocr-native_b200/build.py")
        L = ctypes.CDLL(str(path))
        for name, (res, args) in _SIG.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


class PpocrError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


def _check(code: int) -> None:
    if code != OK:
        raise PpocrError(code, lib().ppocr_last_error().decode())


def device_count() -> int:
    return lib().ppocr_device_count()


class Model:
    """A plan on one GPU (`GpuModel`). `plan` is the file's bytes or a path."""

    def __init__(self, plan: bytes | str | os.PathLike, device: int = 0, _handle=None):
        self._h = ctypes.c_void_p()
        if _handle is not None:
            self._h = _handle
        elif isinstance(plan, (bytes, bytearray)):
            _check(lib().ppocr_model_load_bytes(bytes(plan), len(plan), device, ctypes.byref(self._h)))
        else:
            _check(lib().ppocr_model_load(os.fsencode(plan), device, ctypes.byref(self._h)))

    def close(self) -> None:
        if self._h:
            lib().ppocr_model_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def share_weights(self) -> "Model":
        h = ctypes.c_void_p()
        _check(lib().ppocr_model_share_weights(self._h, ctypes.byref(h)))
        return Model(b"", _handle=h)

    # -- GpuModel surface ---------------------------------------------------
    @property
    def device(self) -> str:
        return lib().ppocr_model_device_name(self._h).decode()

    @property
    def integrated(self) -> bool:
        return bool(lib().ppocr_model_integrated(self._h))

    def max_lanes(self) -> int:
        return lib().ppocr_model_max_lanes(self._h)

    def output_count(self) -> int:
        return lib().ppocr_model_output_count(self._h)

    def set_input_size(self, h: int, w: int) -> None:
        _check(lib().ppocr_model_set_input_size(self._h, h, w))

    def set_sizes(self, sizes) -> None:
        flat = [v for hw in sizes for v in hw]
        arr = (ctypes.c_uint32 * max(len(flat), 1))(*flat)
        _check(lib().ppocr_model_set_sizes(self._h, arr, len(sizes)))

    def lane_input_mut(self, lane: int = 0) -> np.ndarray:
        n = ctypes.c_size_t()
        p = lib().ppocr_model_lane_input(self._h, lane, ctypes.byref(n))
        if not p:
            _check(E_ARG)
        return np.ctypeslib.as_array(p, shape=(n.value,))

    def input_mut(self) -> np.ndarray:
        return self.lane_input_mut(0)

    def lane_output(self, lane: int = 0, index: int = 0) -> np.ndarray:
        n = ctypes.c_size_t()
        p = lib().ppocr_model_lane_output(self._h, lane, index, ctypes.byref(n))
        if not p:
            _check(E_ARG)
        return np.ctypeslib.as_array(p, shape=(n.value,))

    def output(self, index: int = 0) -> np.ndarray:
        return self.lane_output(0, index)

    def run(self, timeout_ms: int = 0) -> None:
        _check(lib().ppocr_model_run(self._h, timeout_ms))

    def enqueue(self) -> None:
        _check(lib().ppocr_model_enqueue(self._h))

    def wait(self, timeout_ms: int = 0) -> None:
        _check(lib().ppocr_model_wait(self._h, timeout_ms))

    # -- device-resident use ------------------------------------------------
    def lane_device_input(self, lane: int = 0) -> tuple[int, int]:
        n = ctypes.c_size_t()
        p = lib().ppocr_model_lane_device_input(self._h, lane, ctypes.byref(n))
        if not p:
            _check(E_ARG)
        return p, n.value

    def lane_device_output(self, lane: int = 0, index: int = 0) -> tuple[int, int]:
        n = ctypes.c_size_t()
        p = lib().ppocr_model_lane_device_output(self._h, lane, index, ctypes.byref(n))
        if not p:
            _check(E_ARG)
        return p, n.value

    def enqueue_device(self) -> None:
        _check(lib().ppocr_model_enqueue_device(self._h))

    @property
    def stream(self) -> int:
        return lib().ppocr_model_stream(self._h) or 0

    def set_stream(self, stream: int | None) -> None:
        _check(lib().ppocr_model_set_stream(self._h, stream or None))

    def set_options(self, options: int) -> None:
        _check(lib().ppocr_model_set_options(self._h, options))

    @property
    def launches(self) -> int:
        return lib().ppocr_model_launches(self._h)

    def steps(self) -> list[str]:
        out = []
        while True:
            s = lib().ppocr_model_step_name(self._h, len(out))
            if s is None:
                return out
            out.append(s.decode())


def ctc_argmax_noalloc(x: int, w: int, b: int, y: int, pixels: int, ci: int, vocab: int,
                       stream: int | None = None) -> None:
    """The CTC argmax head over caller-owned device buffers (device
    pointers as ints), for callers that may not allocate device memory; see
    `ppocr_ctc_argmax_noalloc` in include/ppocr_cuda.h for the scratch limit
    and the sharing rules."""
    _check(lib().ppocr_ctc_argmax_noalloc(x, w, b, y, pixels, ci, vocab, stream or None))


def det_input_hwc(image: int, width: int, height: int, out_width: int, out_height: int, mean, std, out: int,
                  capacity: int | None = None, stream: int | None = None) -> None:
    """The detector's input from an RGB byte image, on the GPU (device
    pointers as ints): resized to out_width x out_height and normalized,
    channels together, into out (capacity floats; default exactly
    out_width x out_height x 3); see `ppocr_det_input_hwc` in
    include/ppocr_cuda.h."""
    m = (ctypes.c_double * 3)(*[float(v) for v in mean])
    s = (ctypes.c_double * 3)(*[float(v) for v in std])
    cap = out_width * out_height * 3 if capacity is None else capacity
    _check(lib().ppocr_det_input_hwc(image, width, height, out_width, out_height, m, s, out, cap, stream or None))


def rec_input_width(width: int, height: int) -> int:
    """The recogniser tensor width of a width x height crop."""
    w = ctypes.c_size_t()
    _check(lib().ppocr_rec_input_hwc(None, width, height, None, 0, ctypes.byref(w), None))
    return w.value


def rec_input_hwc(crop: int, width: int, height: int, out: int, capacity: int, stream: int | None = None) -> int:
    """The recogniser's input of one RGB byte crop, on the GPU (device
    pointers as ints): 48 x tensor width x 3 floats into out (capacity
    floats); returns the tensor width. See `ppocr_rec_input_hwc` in
    include/ppocr_cuda.h."""
    w = ctypes.c_size_t()
    _check(lib().ppocr_rec_input_hwc(crop, width, height, out, capacity, ctypes.byref(w), stream or None))
    return w.value


def db_mask(prob: int, pixels: int, thresh: float, mask: int, stream: int | None = None) -> None:
    """The DB text mask prob > thresh (device pointers as ints); see
    `ppocr_db_mask` in include/ppocr_cuda.h."""
    _check(lib().ppocr_db_mask(prob, pixels, thresh, mask, stream or None))
