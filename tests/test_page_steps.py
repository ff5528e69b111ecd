"""The product's host page steps (ppocr-native_b200/csrc/page.cpp, through
the C ABI) on the CPU: the reference's own fixtures, asserted as its
tests/parity.rs asserts them, and seeded random inputs against the oracle's
independent restatement (oracle/page_oracle.c): masks with blobs and holes,
probability maps, point sets, quads, recogniser outputs."""

from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np
import pytest

from ppocr_native_b200 import cuda

REF = Path(__file__).resolve().parent / "golden" / "ref"
FIX = json.loads((REF / "fixtures.json").read_text())


def npy(name: str) -> np.ndarray:
    return np.load(REF / name)


# ------------------------------------------------------------- fixtures

def test_contours_match_opencv():
    for i, case in enumerate(FIX["contours"]):
        assert cuda.find_contours(npy(case["file"])) == case["contours"], f"mask {i}"


def test_db_boxes_match_rapidocr():
    case = FIX["boxes"]
    got = cuda.boxes_from_prob(npy(case["file"]), *case["dest"])
    assert np.array_equal(got, np.asarray(case["boxes"], np.float32))


def test_min_area_rect_matches_opencv():
    for case in FIX["min_area_rect"]:
        assert np.array_equal(cuda.min_area_rect_points(case["points"]), np.asarray(case["box"], np.float32))


def test_unclip_matches_pyclipper():
    for case in FIX["unclip"]:
        assert cuda.unclip(case["quad"], 1.5) == case["ring"], case["quad"]


def test_ctc_matches_rapidocr():
    d = cuda.Dictionary((REF / "characters.txt").read_bytes())
    assert len(d) == 18710
    for case in FIX["ctc"]:
        best = npy(f"{case['stem']}_argmax.npy").astype(np.float32)
        prob = npy(f"{case['stem']}_maxprob.npy")
        text, score = d.decode(np.stack([best, prob], axis=1))
        assert (text, score) == (case["text"], case["score"]), case["stem"]


def test_dictionary_and_blank_like_python():
    d = cuda.Dictionary("a\r\nb\x1cc \nd\n")
    assert [d[i] for i in range(len(d))] == ["blank", "a", "b", "c", "", "d", " "]
    assert cuda.is_blank(" \t\x1c　 ") and not cuda.is_blank(" a ") and cuda.is_blank("")
    # an out-of-dictionary class: NaN score, nothing added (the model and the dictionary disagree)
    text, score = cuda.Dictionary("a\nb\n").decode([[1, 0.5], [7, 0.9]])
    assert text == "a" and math.isnan(score)


def test_page_sizes_follow_the_reference():
    assert cuda.det_size(40, 28) == (32, 32)
    assert cuda.det_size(2550, 3300) == (1536, 1984)  # 2000 snaps to 1984 (ties to even)
    for w, h in [(100, 0), (0, 100), (0, 0)]:
        assert cuda.prepare_page(w, h) is None and cuda.det_size(w, h) is None
    assert cuda.prepare_page(4096, 1) is None
    fw, fh, _, _, pad = cuda.prepare_page(4096, 20)
    assert (fw, fh, pad) == (6144, 1536, 752)
    assert cuda.prepare_page(2550, 3300) == (2550, 3300, 1.0, 1.0, 0)


# ------------------------------------------------ against the oracle

def blob_mask(rng, h, w, blobs):
    m = np.zeros((h, w), np.uint8)
    for _ in range(blobs):
        y, x = rng.integers(0, h), rng.integers(0, w)
        ry, rx = rng.integers(1, max(2, h // 4)), rng.integers(1, max(2, w // 4))
        yy, xx = np.ogrid[:h, :w]
        inside = ((yy - y) / ry) ** 2 + ((xx - x) / rx) ** 2 <= 1
        m[inside] = 1 - m[inside] if rng.random() < 0.3 else 1  # holes now and then
    m[rng.random((h, w)) < 0.02] ^= 1  # speckle
    return m


@pytest.mark.parametrize("seed", range(12))
def test_contours_and_boxes_match_the_oracle(oracle_mod, seed):
    rng = np.random.default_rng(seed)
    h, w = int(rng.integers(1, 90)), int(rng.integers(1, 120))
    m = blob_mask(rng, h, w, int(rng.integers(0, 8)))
    assert cuda.find_contours(m) == oracle_mod.find_contours(m)
    # a probability map whose text pixels follow the mask, scores around box_thresh
    prob = np.where(m, rng.uniform(0.25, 0.9, m.shape), rng.uniform(0, 0.35, m.shape)).astype(np.float32)
    dw, dh = int(w * rng.uniform(0.5, 3)) + 1, int(h * rng.uniform(0.5, 3)) + 1
    assert np.array_equal(cuda.boxes_from_prob(prob, dw, dh), oracle_mod.boxes_from_prob(prob, dw, dh))
    for c in oracle_mod.find_contours(m)[:20]:
        assert cuda.contour_mean(prob, c) == oracle_mod.contour_mean(prob, c)


@pytest.mark.parametrize("seed", range(6))
def test_wide_mask_contours_match_the_oracle(oracle_mod, seed):
    """Rows long enough for the sixteen-byte start scan, with borders at
    every offset within a block and at the row ends: blobs, a checkerboard,
    all foreground, single rows and columns."""
    rng = np.random.default_rng(200 + seed)
    h, w = int(rng.integers(1, 40)), int(rng.integers(16, 700))
    masks = [blob_mask(rng, h, w, int(rng.integers(1, 12))), np.ones((h, w), np.uint8),
             (np.indices((h, w)).sum(axis=0) % 2).astype(np.uint8), np.ones((1, w), np.uint8),
             np.ones((h, 1), np.uint8), (rng.random((h, w)) < 0.5).astype(np.uint8)]
    for m in masks:
        assert cuda.find_contours(m) == oracle_mod.find_contours(m)


@pytest.mark.parametrize("seed", range(8))
def test_geometry_matches_the_oracle(oracle_mod, seed):
    rng = np.random.default_rng(100 + seed)
    for _ in range(50):
        n = int(rng.integers(1, 40))
        span = int(rng.choice([3, 20, 2000]))
        pts = rng.integers(-5, span, (n, 2))
        assert np.array_equal(cuda.min_area_rect_points(pts), oracle_mod.min_area_rect_points(pts)), pts.tolist()
        q1, s1 = cuda.mini_box(pts)
        q2, s2 = oracle_mod.mini_box(pts)
        assert np.array_equal(q1, q2) and s1 == s2
        quad = q1 + rng.uniform(-3, 3, q1.shape).astype(np.float32)
        ratio = float(rng.uniform(0.5, 3))
        assert cuda.unclip(quad, ratio) == oracle_mod.unclip(quad, ratio)


def test_ctc_decode_matches_the_oracle(oracle_mod):
    rng = np.random.default_rng(7)
    text = "".join(chr(0x4E00 + i) + "\n" for i in range(200))
    d = cuda.Dictionary(text)
    classes = oracle_mod.dictionary(text)
    assert [d[i] for i in range(len(d))] == classes
    for steps in (0, 1, 7, 8, 40, 129, 497):
        best = rng.integers(0, 6, steps) * rng.integers(0, 40, steps)  # blanks and repeats
        prob = rng.uniform(0, 1, steps).astype(np.float32)
        got = d.decode(np.stack([best.astype(np.float32), prob], axis=1))
        assert got == oracle_mod.ctc_decode(best.astype(np.uint32), prob, classes), steps
