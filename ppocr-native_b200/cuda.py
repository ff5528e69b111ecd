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
OPT_NO_FUSION, OPT_NO_GRAPH, OPT_NO_TENSOR_CORES, OPT_THROUGHPUT = 1, 2, 4, 8

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
    # page steps and the reader
    "ppocr_reader_options_default": (None, [ctypes.c_void_p]),
    "ppocr_reader_create": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t,
                                           ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "ppocr_reader_free": (None, [ctypes.c_void_p]),
    "ppocr_reader_stream": (ctypes.c_void_p, [ctypes.c_void_p]),
    "ppocr_reader_page": (ctypes.POINTER(ctypes.c_uint8), [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t]),
    "ppocr_reader_detect": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t,
                                           ctypes.c_uint32]),
    "ppocr_reader_detect_device": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                                  ctypes.c_size_t, ctypes.c_uint32]),
    "ppocr_reader_launches": (ctypes.c_size_t, [ctypes.c_void_p]),
    "ppocr_reader_box_count": (ctypes.c_size_t, [ctypes.c_void_p]),
    "ppocr_reader_boxes": (ctypes.POINTER(ctypes.c_float), [ctypes.c_void_p]),
    "ppocr_reader_prepared": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_size_t),
                                             ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_double),
                                             ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_size_t)]),
    "ppocr_reader_recognise": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32]),
    "ppocr_reader_text_count": (ctypes.c_size_t, [ctypes.c_void_p]),
    "ppocr_reader_text": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_char_p),
                                         ctypes.POINTER(ctypes.c_double)]),
    "ppocr_reader_read": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t,
                                         ctypes.c_uint32]),
    "ppocr_reader_line_count": (ctypes.c_size_t, [ctypes.c_void_p]),
    "ppocr_reader_line": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                         ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_double)]),
    "ppocr_reader_set_options": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32]),
    "ppocr_reader_prob_map": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                             ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_size_t)]),
    "ppocr_reader_host_times": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "ppocr_reader_stats": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_size_t),
                                          ctypes.POINTER(ctypes.c_size_t)]),
    "ppocr_find_contours": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p,
                                           ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t,
                                           ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_size_t)]),
    "ppocr_contour_mean": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p,
                                          ctypes.c_size_t, ctypes.POINTER(ctypes.c_double)]),
    "ppocr_min_area_rect": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "ppocr_box_points": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "ppocr_mini_box": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                      ctypes.POINTER(ctypes.c_float)]),
    "ppocr_unclip": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_double, ctypes.c_void_p, ctypes.c_size_t,
                                    ctypes.POINTER(ctypes.c_size_t)]),
    "ppocr_boxes_from_prob": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                                             ctypes.c_size_t, ctypes.c_float, ctypes.c_double, ctypes.c_double,
                                             ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t,
                                             ctypes.POINTER(ctypes.c_size_t)]),
    "ppocr_det_size": (ctypes.c_int, [ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                                      ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_size_t)]),
    "ppocr_prepare_page": (ctypes.c_int, [ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p,
                                          ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_size_t),
                                          ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double),
                                          ctypes.POINTER(ctypes.c_size_t)]),
    "ppocr_crop_size": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_size_t),
                                       ctypes.POINTER(ctypes.c_size_t)]),
    "ppocr_crop_text": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "ppocr_dictionary_load": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]),
    "ppocr_dictionary_size": (ctypes.c_size_t, [ctypes.c_void_p]),
    "ppocr_dictionary_class": (ctypes.c_void_p, [ctypes.c_void_p, ctypes.c_size_t,
                                                 ctypes.POINTER(ctypes.c_size_t)]),
    "ppocr_dictionary_free": (None, [ctypes.c_void_p]),
    "ppocr_ctc_decode": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_char_p,
                                        ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t),
                                        ctypes.POINTER(ctypes.c_double)]),
    "ppocr_text_is_blank": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_size_t]),
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


# ---------------------------------------------------------------- page steps

class ReaderOptions(ctypes.Structure):
    """`ppocr_reader_options` (the worker's page, DB and normalization options)."""

    _fields_ = [("thresh", ctypes.c_float), ("box_thresh", ctypes.c_double), ("unclip_ratio", ctypes.c_double),
                ("max_candidates", ctypes.c_uint32), ("text_score", ctypes.c_double),
                ("min_side", ctypes.c_uint32), ("max_side", ctypes.c_uint32),
                ("width_height_ratio", ctypes.c_double), ("min_height", ctypes.c_uint32),
                ("limit_min", ctypes.c_uint32), ("mean", ctypes.c_double * 3), ("std", ctypes.c_double * 3)]

    @classmethod
    def default(cls) -> "ReaderOptions":
        o = cls()
        lib().ppocr_reader_options_default(ctypes.byref(o))
        return o


def _i32(points) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(points, np.int32).reshape(-1, 2))


def _quad(q) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(q, np.float32).reshape(8))


def find_contours(mask: np.ndarray) -> list[list[list[int]]]:
    """`ppocr_find_contours` of an (h, w) mask: lists of [x, y] points."""
    mask = np.ascontiguousarray(mask, np.uint8)
    h, w = mask.shape
    nc, npnt = ctypes.c_size_t(), ctypes.c_size_t()
    code = lib().ppocr_find_contours(mask.ctypes.data, w, h, None, 0, None, 0, ctypes.byref(nc), ctypes.byref(npnt))
    if code not in (OK, E_SIZE):
        _check(code)
    pts = np.empty((max(npnt.value, 1), 2), np.int32)
    starts = np.empty(nc.value + 1, np.uintp)
    _check(lib().ppocr_find_contours(mask.ctypes.data, w, h, pts.ctypes.data, npnt.value, starts.ctypes.data,
                                     nc.value + 1, ctypes.byref(nc), ctypes.byref(npnt)))
    return [pts[starts[i]:starts[i + 1]].tolist() for i in range(nc.value)]


def contour_mean(prob: np.ndarray, points) -> float:
    prob = np.ascontiguousarray(prob, np.float32)
    p = _i32(points)
    out = ctypes.c_double()
    _check(lib().ppocr_contour_mean(prob.ctypes.data, prob.shape[1], prob.shape[0], p.ctypes.data, len(p),
                                    ctypes.byref(out)))
    return out.value


def min_area_rect_points(points) -> np.ndarray:
    """cv2.boxPoints(cv2.minAreaRect(points)) through the C ABI, (4, 2) f32."""
    p = _i32(points)
    rect = np.empty(5, np.float32)
    quad = np.empty((4, 2), np.float32)
    _check(lib().ppocr_min_area_rect(p.ctypes.data, len(p), rect.ctypes.data))
    _check(lib().ppocr_box_points(rect.ctypes.data, quad.ctypes.data))
    return quad


def mini_box(points):
    p = _i32(points)
    quad = np.empty((4, 2), np.float32)
    side = ctypes.c_float()
    _check(lib().ppocr_mini_box(p.ctypes.data, len(p), quad.ctypes.data, ctypes.byref(side)))
    return quad, side.value


def unclip(quad, ratio: float = 1.5) -> list[list[int]]:
    q = _quad(quad)
    n = ctypes.c_size_t()
    out = np.empty((4096, 2), np.int32)
    _check(lib().ppocr_unclip(q.ctypes.data, ratio, out.ctypes.data, 4096, ctypes.byref(n)))
    return out[:n.value].tolist()


def boxes_from_prob(prob: np.ndarray, dest_w: int, dest_h: int, thresh: float = 0.3, box_thresh: float = 0.5,
                    unclip_ratio: float = 1.5, max_candidates: int = 1000) -> np.ndarray:
    prob = np.ascontiguousarray(prob, np.float32)
    mh, mw = prob.shape
    n = ctypes.c_size_t()
    cap = 4096
    out = np.empty((cap, 4, 2), np.float32)
    _check(lib().ppocr_boxes_from_prob(prob.ctypes.data, mw, mh, dest_w, dest_h, thresh, box_thresh, unclip_ratio,
                                       max_candidates, out.ctypes.data, cap, ctypes.byref(n)))
    return out[:n.value].copy()


def det_size(w: int, h: int, limit_min: int = 0):
    ow, oh = ctypes.c_size_t(), ctypes.c_size_t()
    if lib().ppocr_det_size(w, h, limit_min, ctypes.byref(ow), ctypes.byref(oh)) != OK:
        return None
    return ow.value, oh.value


def prepare_page(w: int, h: int, options: ReaderOptions | None = None):
    """(width, height, ratio_h, ratio_w, pad_top) of the prepared page, or None."""
    fw, fh, pad = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
    rw, rh = ctypes.c_double(), ctypes.c_double()
    if lib().ppocr_prepare_page(w, h, ctypes.byref(options) if options else None, ctypes.byref(fw),
                                ctypes.byref(fh), ctypes.byref(rw), ctypes.byref(rh), ctypes.byref(pad)) != OK:
        return None
    return fw.value, fh.value, rh.value, rw.value, pad.value


def crop_size(quad) -> tuple[int, int]:
    """(width, height) of crop_text's result, turned when tall."""
    q = _quad(quad)
    w, h = ctypes.c_size_t(), ctypes.c_size_t()
    _check(lib().ppocr_crop_size(q.ctypes.data, ctypes.byref(w), ctypes.byref(h)))
    return w.value, h.value


def crop_text(image: int, width: int, height: int, quad, out: int, capacity: int, stream: int | None = None):
    """crop_text on the GPU (device pointers as ints)."""
    q = _quad(quad)
    _check(lib().ppocr_crop_text(image, width, height, q.ctypes.data, out, capacity, stream or None))


class Dictionary:
    """The recogniser's classes (`ppocr_dictionary`)."""

    def __init__(self, text: str | bytes):
        data = text.encode("utf-8") if isinstance(text, str) else bytes(text)
        self._h = ctypes.c_void_p()
        _check(lib().ppocr_dictionary_load(data, len(data), ctypes.byref(self._h)))

    def __del__(self):
        if getattr(self, "_h", None):
            lib().ppocr_dictionary_free(self._h)
            self._h = None

    def __len__(self) -> int:
        return lib().ppocr_dictionary_size(self._h)

    def __getitem__(self, i: int) -> str:
        n = ctypes.c_size_t()
        p = lib().ppocr_dictionary_class(self._h, i, ctypes.byref(n))
        if p is None:
            raise IndexError(i)
        return ctypes.string_at(p, n.value).decode("utf-8")

    def decode(self, output) -> tuple[str, float]:
        """`ppocr_ctc_decode` of an argmax recogniser's [steps][2] output."""
        out = np.ascontiguousarray(np.asarray(output, np.float32).reshape(-1, 2))
        cap = 8 * len(out) * 16 + 16
        buf = ctypes.create_string_buffer(cap)
        n, score = ctypes.c_size_t(), ctypes.c_double()
        _check(lib().ppocr_ctc_decode(out.ctypes.data, len(out), self._h, buf, cap, ctypes.byref(n),
                                      ctypes.byref(score)))
        return buf.raw[:n.value].decode("utf-8"), score.value


def is_blank(text: str) -> bool:
    data = text.encode("utf-8")
    return bool(lib().ppocr_text_is_blank(data, len(data)))


class Reader:
    """A page reader (`ppocr_reader`) over a detector and a recogniser."""

    def __init__(self, det: Model, rec: Model, characters: str | bytes, options: ReaderOptions | None = None):
        data = characters.encode("utf-8") if isinstance(characters, str) else bytes(characters)
        self._h = ctypes.c_void_p()
        _check(lib().ppocr_reader_create(det._h, rec._h, data, len(data),
                                         ctypes.byref(options) if options else None, ctypes.byref(self._h)))

    def close(self) -> None:
        if self._h:
            lib().ppocr_reader_free(self._h)
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

    @property
    def stream(self) -> int:
        return lib().ppocr_reader_stream(self._h) or 0

    def page_buffer(self, width: int, height: int) -> np.ndarray:
        """The reader's page-locked page buffer, (height, width, 3) uint8."""
        p = lib().ppocr_reader_page(self._h, width, height)
        if not p:
            _check(E_ARG)
        return np.ctypeslib.as_array(p, shape=(height, width, 3))

    def detect(self, page: np.ndarray, timeout_ms: int = 60_000) -> np.ndarray:
        """Boxes (n, 4, 2) on the prepared page."""
        h, w = page.shape[:2]
        _check(lib().ppocr_reader_detect(self._h, page.ctypes.data, w, h, timeout_ms))
        return self.boxes()

    def detect_ptr(self, page: int, width: int, height: int, on_device: bool = False,
                   timeout_ms: int = 60_000) -> int:
        """Detection of a page given by pointer (host memory, or device
        memory with on_device); returns the number of boxes."""
        f = lib().ppocr_reader_detect_device if on_device else lib().ppocr_reader_detect
        _check(f(self._h, page, width, height, timeout_ms))
        return lib().ppocr_reader_box_count(self._h)

    def recognise_ptr(self, quads: int, n: int, timeout_ms: int = 60_000) -> None:
        _check(lib().ppocr_reader_recognise(self._h, quads, n, timeout_ms))

    @property
    def launches(self) -> int:
        return lib().ppocr_reader_launches(self._h)

    def boxes(self) -> np.ndarray:
        n = lib().ppocr_reader_box_count(self._h)
        if not n:
            return np.zeros((0, 4, 2), np.float32)
        return np.ctypeslib.as_array(lib().ppocr_reader_boxes(self._h), shape=(n, 4, 2)).copy()

    def prepared(self):
        """(width, height, ratio_w, ratio_h, pad_top) of the last detected page."""
        w, h, pad = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
        rw, rh = ctypes.c_double(), ctypes.c_double()
        _check(lib().ppocr_reader_prepared(self._h, ctypes.byref(w), ctypes.byref(h), ctypes.byref(rw),
                                           ctypes.byref(rh), ctypes.byref(pad)))
        return w.value, h.value, rw.value, rh.value, pad.value

    def recognise(self, quads, timeout_ms: int = 60_000) -> list[tuple[str, float]]:
        q = np.ascontiguousarray(np.asarray(quads, np.float32).reshape(-1, 8))
        _check(lib().ppocr_reader_recognise(self._h, q.ctypes.data, len(q), timeout_ms))
        return self.texts()

    def texts(self) -> list[tuple[str, float]]:
        out = []
        t, s = ctypes.c_char_p(), ctypes.c_double()
        for i in range(lib().ppocr_reader_text_count(self._h)):
            _check(lib().ppocr_reader_text(self._h, i, ctypes.byref(t), ctypes.byref(s)))
            out.append((t.value.decode("utf-8"), s.value))
        return out

    def read(self, page: np.ndarray, timeout_ms: int = 60_000):
        """Lines (quad (4, 2) on the page as given, text, score)."""
        h, w = page.shape[:2]
        _check(lib().ppocr_reader_read(self._h, page.ctypes.data, w, h, timeout_ms))
        return self.lines()

    def lines(self):
        out = []
        q = np.empty(8, np.float32)
        t, s = ctypes.c_char_p(), ctypes.c_double()
        for i in range(lib().ppocr_reader_line_count(self._h)):
            _check(lib().ppocr_reader_line(self._h, i, q.ctypes.data, ctypes.byref(t), ctypes.byref(s)))
            out.append((q.reshape(4, 2).copy(), t.value.decode("utf-8"), s.value))
        return out

    def set_options(self, options: int) -> None:
        _check(lib().ppocr_reader_set_options(self._h, options))

    def prob_map(self) -> np.ndarray:
        """The detector's map of the last detection, (h, w) float32."""
        w, h = ctypes.c_size_t(), ctypes.c_size_t()
        code = lib().ppocr_reader_prob_map(self._h, None, 0, ctypes.byref(w), ctypes.byref(h))
        if code not in (OK, E_SIZE):
            _check(code)
        out = np.empty((h.value, w.value), np.float32)
        _check(lib().ppocr_reader_prob_map(self._h, out.ctypes.data, out.size, ctypes.byref(w), ctypes.byref(h)))
        return out

    def host_times(self) -> dict:
        """Host seconds by step, summed over this reader's calls."""
        out = np.zeros(5, np.float64)
        _check(lib().ppocr_reader_host_times(self._h, out.ctypes.data))
        return dict(zip(("wait", "contours", "boxes", "recogniser_setup", "decode"), out.tolist()))

    def stats(self) -> tuple[int, int]:
        a, b = ctypes.c_size_t(), ctypes.c_size_t()
        _check(lib().ppocr_reader_stats(self._h, ctypes.byref(a), ctypes.byref(b)))
        return a.value, b.value
