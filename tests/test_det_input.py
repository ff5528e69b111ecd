"""The detector's and the recogniser's input preparation (reference
src/det.rs:230-292 det_input_hwc and src/rec.rs:19-43 rec_input, both over
the INTER_LINEAR resize of src/image.rs:46-142): the oracle against an
independent numpy restatement and identity / constant images, on the CPU;
the GPU entry points `ppocr_det_input_hwc` and `ppocr_rec_input_hwc` against
the oracle, bit for bit."""

from __future__ import annotations

import ctypes
import glob
import os

import numpy as np
import pytest

MEAN, STD = [0.485, 0.456, 0.406], [0.229, 0.224, 0.225]  # the reference worker's (ocr.rs)


def taps(src: int, dst: int):
    d = np.arange(dst, dtype=np.float64)
    f = ((d + 0.5) * (1.0 / (dst / src)) - 0.5).astype(np.float32)
    fl = np.floor(f)
    a = (f - fl).astype(np.float32)
    s = fl.astype(np.int64)
    near, far = np.clip(s, 0, src - 1), np.clip(s + 1, 0, src - 1)
    nw = np.rint((np.float32(1.0) - a) * np.float32(2048.0)).astype(np.int32)
    fw = np.rint(a * np.float32(2048.0)).astype(np.int32)
    return near, far, nw, fw


def det_input_numpy(image: np.ndarray, ow: int, oh: int, mean, std) -> np.ndarray:
    ih, iw, _ = image.shape
    xn, xf, xnw, xfw = taps(iw, ow)
    yn, yf, ynw, yfw = taps(ih, oh)
    img = image.astype(np.int32)
    horiz = img[:, xn, :] * xnw[None, :, None] + img[:, xf, :] * xfw[None, :, None]  # (ih, ow, 3)
    a, b = horiz[yn], horiz[yf]
    v = (((a >> 4) * ynw[:, None, None]) >> 16) + (((b >> 4) * yfw[:, None, None]) >> 16)
    byte = np.clip((v + 2) >> 2, 0, 255)
    x = byte.astype(np.float32) * np.float32(1.0 / 255.0)
    return ((x.astype(np.float64) - np.asarray(mean)) / np.asarray(std)).astype(np.float32)


SIZES = [((17, 23), (13, 32)), ((3300, 2550)[::1], (1984, 1536)), ((5, 7), (48, 64)), ((1, 1), (5, 3)),
         ((40, 9), (40, 9)), ((33, 65), (11, 22))]


@pytest.mark.parametrize("src,dst", [s for s in SIZES if s[0][0] * s[0][1] < 10 ** 5])
def test_oracle_matches_numpy_restatement(oracle_mod, src, dst):
    rng = np.random.default_rng(src[0] * 7 + dst[1])
    image = rng.integers(0, 256, (*src, 3), dtype=np.uint8)
    got = oracle_mod.det_input_hwc(image, dst[1], dst[0], MEAN, STD)
    want = det_input_numpy(image, dst[1], dst[0], MEAN, STD)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_oracle_identity_and_constant_images(oracle_mod):
    rng = np.random.default_rng(3)
    image = rng.integers(0, 256, (21, 19, 3), dtype=np.uint8)
    # same size: the resize returns the bytes themselves
    got = oracle_mod.det_input_hwc(image, 19, 21, [0, 0, 0], [1, 1, 1])
    assert np.array_equal(got, image.astype(np.float32) * np.float32(1.0 / 255.0))
    # any size: a constant image stays constant
    flat = np.full((31, 17, 3), 200, np.uint8)
    got = oracle_mod.det_input_hwc(flat, 40, 9, [0, 0, 0], [1, 1, 1])
    assert np.all(got == np.float32(200) * np.float32(1.0 / 255.0))


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
    pytest.fail("no libcudart for the test's device buffers")


@pytest.mark.gpu
@pytest.mark.parametrize("src,dst", SIZES)
def test_gpu_det_input_matches_oracle(cuda_mod, oracle_mod, src, dst):
    rng = np.random.default_rng(src[1] * 3 + dst[0])
    image = rng.integers(0, 256, (*src, 3), dtype=np.uint8)
    want = oracle_mod.det_input_hwc(image, dst[1], dst[0], MEAN, STD)
    rt = _cudart()
    din, dout = ctypes.c_void_p(), ctypes.c_void_p()
    assert rt.cudaMalloc(ctypes.byref(din), image.nbytes) == 0
    assert rt.cudaMalloc(ctypes.byref(dout), want.nbytes) == 0
    try:
        assert rt.cudaMemcpy(din, image.ctypes.data, image.nbytes, 1) == 0
        cuda_mod.det_input_hwc(din.value, src[1], src[0], dst[1], dst[0], MEAN, STD, dout.value)
        got = np.empty_like(want)
        assert rt.cudaMemcpy(got.ctypes.data, dout, got.nbytes, 2) == 0
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), float(np.abs(got - want).max())
    finally:
        rt.cudaFree(din)
        rt.cudaFree(dout)


# ------------------------------------------------------- recogniser input

def rec_input_numpy(crop: np.ndarray) -> np.ndarray:
    """reference rec.rs:19-43 (HWC as ocr.rs:534-549 turns it)."""
    ch, cw, _ = crop.shape
    h, w, rows = float(ch), float(cw), 48.0
    width = int(rows * max(320.0 / rows, w / h))
    fitted = np.ceil(rows * (w / h))
    rw = width if fitted > width else int(fitted)
    xn, xf, xnw, xfw = taps(cw, rw)
    yn, yf, ynw, yfw = taps(ch, 48)
    img = crop.astype(np.int32)
    horiz = img[:, xn, :] * xnw[None, :, None] + img[:, xf, :] * xfw[None, :, None]
    a, b = horiz[yn], horiz[yf]
    v = (((a >> 4) * ynw[:, None, None]) >> 16) + (((b >> 4) * yfw[:, None, None]) >> 16)
    byte = np.clip((v + 2) >> 2, 0, 255).astype(np.float32)
    out = np.zeros((48, width, 3), np.float32)
    out[:, :rw] = (byte / np.float32(255.0) - np.float32(0.5)) / np.float32(0.5)
    return out


CROPS = [(30, 200), (48, 48), (17, 1500), (60, 33), (1, 1), (9, 61), (100, 2000)]


@pytest.mark.parametrize("crop", CROPS)
def test_oracle_rec_input_matches_numpy_restatement(oracle_mod, crop):
    rng = np.random.default_rng(crop[0] * 13 + crop[1])
    image = rng.integers(0, 256, (*crop, 3), dtype=np.uint8)
    got = oracle_mod.rec_input_hwc(image)
    want = rec_input_numpy(image)
    assert got.shape == want.shape
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("crop", CROPS)
def test_gpu_rec_input_matches_oracle(cuda_mod, oracle_mod, crop):
    rng = np.random.default_rng(crop[1] * 5 + crop[0])
    image = rng.integers(0, 256, (*crop, 3), dtype=np.uint8)
    want = oracle_mod.rec_input_hwc(image)
    width = cuda_mod.rec_input_width(crop[1], crop[0])
    assert width == want.shape[1]
    rt = _cudart()
    din, dout = ctypes.c_void_p(), ctypes.c_void_p()
    assert rt.cudaMalloc(ctypes.byref(din), image.nbytes) == 0
    assert rt.cudaMalloc(ctypes.byref(dout), want.nbytes) == 0
    try:
        assert rt.cudaMemcpy(din, image.ctypes.data, image.nbytes, 1) == 0
        got_w = cuda_mod.rec_input_hwc(din.value, crop[1], crop[0], dout.value, want.size)
        assert got_w == width
        got = np.empty_like(want)
        assert rt.cudaMemcpy(got.ctypes.data, dout, got.nbytes, 2) == 0
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), float(np.abs(got - want).max())
    finally:
        rt.cudaFree(din)
        rt.cudaFree(dout)


# ------------------------------------------------------------- DB mask

@pytest.mark.gpu
def test_gpu_db_mask_matches_f32_comparison(cuda_mod):
    """mask = prob > thresh in f32 (det.rs:438), values at and around the
    threshold included."""
    rng = np.random.default_rng(11)
    thresh = np.float32(0.3)
    prob = rng.random(1984 * 1536 + 7).astype(np.float32)
    prob[:5] = [thresh, np.nextafter(thresh, np.float32(1)), np.nextafter(thresh, np.float32(0)), 0.0, 1.0]
    want = (prob > thresh).astype(np.uint8)
    rt = _cudart()
    dp, dm = ctypes.c_void_p(), ctypes.c_void_p()
    assert rt.cudaMalloc(ctypes.byref(dp), prob.nbytes) == 0
    assert rt.cudaMalloc(ctypes.byref(dm), want.nbytes) == 0
    try:
        assert rt.cudaMemcpy(dp, prob.ctypes.data, prob.nbytes, 1) == 0
        cuda_mod.db_mask(dp.value, prob.size, float(thresh), dm.value)
        got = np.empty_like(want)
        assert rt.cudaMemcpy(got.ctypes.data, dm, got.nbytes, 2) == 0
        assert np.array_equal(got, want)
    finally:
        rt.cudaFree(dp)
        rt.cudaFree(dm)
