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
    src = [HERE / "ppocr_oracle.c", HERE / "page_oracle.c", HERE / "ppocr_oracle.h", HERE / "Makefile"]
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
        L.orc_set_fast.argtypes = [ctypes.c_int]
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


def set_fast(on: bool) -> None:
    """The register-tiled timed path (same bits as the plain loops)."""
    lib().orc_set_fast(1 if on else 0)


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


# ------------------------------------------------------------ page steps

def _page_lib() -> ctypes.CDLL:
    L = lib()
    if getattr(L, "_page_ready", False):
        return L
    c_sz, c_vp = ctypes.c_size_t, ctypes.c_void_p
    L.orc_resize_linear.restype = ctypes.c_int
    L.orc_resize_linear.argtypes = [c_vp, c_sz, c_sz, c_sz, c_sz, c_vp]
    L.orc_rotate_ccw.argtypes = [c_vp, c_sz, c_sz, c_vp]
    L.orc_det_size.restype = ctypes.c_int
    L.orc_det_size.argtypes = [c_sz, c_sz, c_sz, ctypes.POINTER(c_sz), ctypes.POINTER(c_sz)]
    L.orc_prepare_page.restype = ctypes.c_int
    L.orc_prepare_page.argtypes = [c_sz, c_sz, c_sz, c_sz, ctypes.c_double, c_sz, ctypes.POINTER(c_sz),
                                   ctypes.POINTER(c_sz), ctypes.POINTER(ctypes.c_double),
                                   ctypes.POINTER(ctypes.c_double), ctypes.POINTER(c_sz)]
    L.orc_find_contours.restype = c_vp
    L.orc_find_contours.argtypes = [c_vp, c_sz, c_sz]
    L.orc_contours_count.restype = c_sz
    L.orc_contours_count.argtypes = [c_vp]
    L.orc_contour.restype = ctypes.POINTER(ctypes.c_int32)
    L.orc_contour.argtypes = [c_vp, c_sz, ctypes.POINTER(c_sz)]
    L.orc_contours_free.argtypes = [c_vp]
    L.orc_contour_mean.restype = ctypes.c_double
    L.orc_contour_mean.argtypes = [c_vp, c_sz, c_sz, c_vp, c_sz]
    L.orc_min_area_rect.argtypes = [c_vp, c_sz, c_vp]
    L.orc_box_points.argtypes = [c_vp, c_vp]
    L.orc_mini_box.restype = ctypes.c_float
    L.orc_mini_box.argtypes = [c_vp, c_sz, c_vp]
    L.orc_unclip.restype = ctypes.c_long
    L.orc_unclip.argtypes = [c_vp, ctypes.c_double, c_vp, c_sz]
    L.orc_boxes_from_prob.restype = c_sz
    L.orc_boxes_from_prob.argtypes = [c_vp, c_sz, c_sz, c_sz, c_sz, ctypes.c_float, ctypes.c_double,
                                      ctypes.c_double, c_sz, c_vp, c_sz]
    L.orc_crop_size.argtypes = [c_vp, ctypes.POINTER(c_sz), ctypes.POINTER(c_sz), ctypes.POINTER(ctypes.c_int)]
    L.orc_crop_text.restype = ctypes.c_int
    L.orc_crop_text.argtypes = [c_vp, c_sz, c_sz, c_vp, c_vp]
    L.orc_ctc_decode.restype = ctypes.c_double
    L.orc_ctc_decode.argtypes = [c_vp, c_vp, c_sz, c_vp, ctypes.POINTER(c_sz)]
    L.orc_to_page.argtypes = [c_vp, ctypes.c_double, ctypes.c_double, c_sz, c_sz, c_sz, c_vp]
    L._page_ready = True
    return L


def _u8(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint8)


def resize_linear(image: np.ndarray, ow: int, oh: int) -> np.ndarray:
    """cv2.resize INTER_LINEAR of an (h, w, 3) uint8 image (image.rs:91-142)."""
    image = _u8(image)
    out = np.empty((oh, ow, 3), np.uint8)
    if _page_lib().orc_resize_linear(image.ctypes.data, image.shape[1], image.shape[0], ow, oh, out.ctypes.data):
        raise OracleError("empty size")
    return out


def det_size(w: int, h: int, limit_min: int = 0):
    """det_size (det.rs:166-193): (width, height) or None."""
    ow, oh = ctypes.c_size_t(), ctypes.c_size_t()
    if not _page_lib().orc_det_size(w, h, limit_min, ctypes.byref(ow), ctypes.byref(oh)):
        return None
    return ow.value, oh.value


def prepare_page(w: int, h: int, min_side: int = 30, max_side: int = 4096, whr: float = 8.0,
                 min_height: int = 30):
    """prepare_page's sizes (det.rs:44-131): (fw, fh, ratio_h, ratio_w, pad_top) or None."""
    fw, fh, pad = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
    rh, rw = ctypes.c_double(), ctypes.c_double()
    if not _page_lib().orc_prepare_page(w, h, min_side, max_side, whr, min_height, ctypes.byref(fw),
                                        ctypes.byref(fh), ctypes.byref(rh), ctypes.byref(rw), ctypes.byref(pad)):
        return None
    return fw.value, fh.value, rh.value, rw.value, pad.value


def find_contours(mask: np.ndarray) -> list[list[list[int]]]:
    """cv2.findContours LIST/SIMPLE of an (h, w) mask (contour.rs:44-130)."""
    mask = _u8(mask)
    L = _page_lib()
    c = L.orc_find_contours(mask.ctypes.data, mask.shape[1], mask.shape[0])
    if not c:
        raise OracleError("out of memory")
    try:
        out = []
        for i in range(L.orc_contours_count(c)):
            n = ctypes.c_size_t()
            p = L.orc_contour(c, i, ctypes.byref(n))
            pts = np.ctypeslib.as_array(p, shape=(n.value, 2)).tolist() if n.value else []
            out.append(pts)
        return out
    finally:
        L.orc_contours_free(c)


def _pts(points) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(points, np.int32).reshape(-1, 2))


def contour_mean(prob: np.ndarray, points) -> float:
    prob = np.ascontiguousarray(prob, np.float32)
    p = _pts(points)
    return _page_lib().orc_contour_mean(prob.ctypes.data, prob.shape[1], prob.shape[0], p.ctypes.data, len(p))


def min_area_rect_points(points) -> np.ndarray:
    """cv2.boxPoints(cv2.minAreaRect(points)) (geometry.rs:228-240, 406-457), (4, 2) f32."""
    p = _pts(points)
    rect = np.empty(5, np.float32)
    quad = np.empty((4, 2), np.float32)
    L = _page_lib()
    L.orc_min_area_rect(p.ctypes.data, len(p), rect.ctypes.data)
    L.orc_box_points(rect.ctypes.data, quad.ctypes.data)
    return quad


def mini_box(points):
    p = _pts(points)
    quad = np.empty((4, 2), np.float32)
    side = _page_lib().orc_mini_box(p.ctypes.data, len(p), quad.ctypes.data)
    return quad, side


def unclip(quad, ratio: float = 1.5) -> list[list[int]]:
    q = np.ascontiguousarray(np.asarray(quad, np.float32).reshape(8))
    out = np.empty((4096, 2), np.int32)
    n = _page_lib().orc_unclip(q.ctypes.data, ratio, out.ctypes.data, 4096)
    if n < 0:
        raise OracleError("ring too long")
    return out[:n].tolist()


def boxes_from_prob(prob: np.ndarray, dest_w: int, dest_h: int, thresh: float = 0.3, box_thresh: float = 0.5,
                    unclip_ratio: float = 1.5, max_candidates: int = 1000) -> np.ndarray:
    """The DB postprocess (det.rs:430-452): (n, 4, 2) f32 quads in reading order."""
    prob = np.ascontiguousarray(prob, np.float32)
    mh, mw = prob.shape
    cap = 4096
    out = np.empty((cap, 4, 2), np.float32)
    n = _page_lib().orc_boxes_from_prob(prob.ctypes.data, mw, mh, dest_w, dest_h, thresh, box_thresh,
                                        unclip_ratio, max_candidates, out.ctypes.data, cap)
    if n > cap:
        raise OracleError(f"{n} boxes exceed {cap}")
    return out[:n].copy()


def crop_text(image: np.ndarray, quad) -> np.ndarray:
    """crop_text (crop.rs:84-127): the (h, w, 3) uint8 crop, turned when tall."""
    image = _u8(image)
    q = np.ascontiguousarray(np.asarray(quad, np.float32).reshape(8))
    w, h, turns = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_int()
    L = _page_lib()
    L.orc_crop_size(q.ctypes.data, ctypes.byref(w), ctypes.byref(h), ctypes.byref(turns))
    shape = (w.value, h.value, 3) if turns.value else (h.value, w.value, 3)
    out = np.zeros(shape, np.uint8)
    if L.orc_crop_text(image.ctypes.data, image.shape[1], image.shape[0], q.ctypes.data, out.ctypes.data):
        raise OracleError("empty page")
    return out


def dictionary(text: str) -> list[str]:
    """Dictionary::from_metadata (rec.rs:54-79): blank, the lines as Python's
    str.splitlines splits them (the reference restates exactly that), space."""
    return ["blank", *text.splitlines(), " "]


def ctc_decode(best, prob, classes: list[str]) -> tuple[str, float]:
    """ctc_decode (rec.rs:144-161): the text and the score."""
    b = np.ascontiguousarray(np.asarray(best, np.uint32))
    p = np.ascontiguousarray(np.asarray(prob, np.float32))
    kept = np.empty(max(len(b), 1), np.uint32)
    n = ctypes.c_size_t()
    score = _page_lib().orc_ctc_decode(b.ctypes.data, p.ctypes.data, len(b), kept.ctypes.data, ctypes.byref(n))
    return "".join(classes[int(c)] for c in kept[:n.value]), score


def to_page(quad, ratio_w: float, ratio_h: float, pad_top: int, width: int, height: int) -> np.ndarray:
    q = np.ascontiguousarray(np.asarray(quad, np.float32).reshape(8))
    out = np.empty((4, 2), np.float32)
    _page_lib().orc_to_page(q.ctypes.data, ratio_w, ratio_h, pad_top, width, height, out.ctypes.data)
    return out


def is_blank(text: str) -> bool:
    """rec.rs:168-172: nothing but whitespace and the separators 0x1c-0x1f."""
    return all(c.isspace() or "\x1c" <= c <= "\x1f" for c in text)


def page_lines(boxes, reads, ratio_w: float, ratio_h: float, pad_top: int, width: int, height: int,
               text_score: float = 0.3):
    """page_lines (lib.rs:96-117): (quad, text, score) of the kept lines; a
    NaN score is never under text_score."""
    out = []
    for quad, (text, score) in zip(boxes, reads):
        if is_blank(text) or score < text_score:
            continue
        out.append((to_page(quad, ratio_w, ratio_h, pad_top, width, height), text, score))
    return out


# ------------------------------------------------------ a whole page

MEAN = (0.485, 0.456, 0.406)  # the worker's detector normalization (ocr.rs:20-25)
STD = (0.229, 0.224, 0.225)


def prepared_image(page: np.ndarray, min_side: int = 30, max_side: int = 4096, whr: float = 8.0,
                   min_height: int = 30):
    """prepare_page (det.rs:110-131): the fitted, padded page and its
    (ratio_w, ratio_h, pad_top), or None."""
    h, w = page.shape[:2]
    got = prepare_page(w, h, min_side, max_side, whr, min_height)
    if got is None:
        return None
    fw, fh, rh, rw, pad = got
    fit_h = fh - 2 * pad
    img = page if (fw, fit_h) == (w, h) else resize_linear(page, fw, fit_h)
    if pad:
        band = np.zeros((pad, fw, 3), np.uint8)
        img = np.concatenate([band, img, band], axis=0)
    return np.ascontiguousarray(img), (rw, rh, pad)


def read_page(page: np.ndarray, det: "Oracle", rec: "Oracle", classes: list[str], quads=None, threads: int = 0,
              text_score: float = 0.3, limit_min: int = 0, max_side: int = 4096):
    """The worker's page read on the CPU oracle (ocr.rs:205-263 without the
    vertical re-read): prepare, detect at det_size, DB boxes, crops,
    recogniser inputs, recogniser, CTC decode, page_lines. With `quads`,
    those are recognised instead of the detected boxes (and no page lines
    are formed). Returns dict(boxes, reads, lines, prob)."""
    prep = prepared_image(page, max_side=max_side)
    if prep is None:
        return {"boxes": np.zeros((0, 4, 2), np.float32), "reads": [], "lines": [], "prob": None}
    img, (rw, rh, pad) = prep
    ph, pw = img.shape[:2]
    size = det_size(pw, ph, limit_min)
    if size is None or size[0] * size[1] > max_side * max_side:
        size = det_size(pw, ph, 0)
    dw, dh = size
    x = det_input_hwc(img, dw, dh, MEAN, STD)
    det.set_size(dh, dw)
    prob = det.run(x.reshape(-1), threads=threads)[0].reshape(dh, dw)
    boxes = boxes_from_prob(prob, pw, ph)
    todo = boxes if quads is None else np.asarray(quads, np.float32).reshape(-1, 4, 2)
    reads = []
    crops = []
    for q in todo:
        crop = crop_text(img, q)
        crops.append(crop)
        if crop.shape[0] == 0 or crop.shape[1] == 0:
            reads.append(("", 0.0))
            continue
        xin = rec_input_hwc(crop)
        rec.set_size(48, xin.shape[1])
        out = rec.run(xin.reshape(-1), threads=threads)[0].reshape(-1, 2)
        reads.append(ctc_decode(out[:, 0].astype(np.uint32), out[:, 1], classes))
    lines = []
    if quads is None:
        lines = page_lines(boxes, reads, rw, rh, pad, page.shape[1], page.shape[0], text_score)
    return {"boxes": boxes, "reads": reads, "lines": lines, "prob": prob, "crops": crops}
