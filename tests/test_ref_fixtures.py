"""The reference's own parity fixtures (its tests/fixtures, written from
OpenCV 5.0, pyclipper 1.4, RapidOCR 3.9 and numpy by its
tools/make_fixtures.py; copied unchanged into tests/golden/ref by
tests/golden/make_ref_fixtures.py), asserted the way the reference's
tests/parity.rs asserts them:

- on the CPU, the oracle's restatement of every host page step: resize
  (parity.rs:48), the detector tensor (:67), contours (:83), DB boxes (:107),
  minimum-area rectangles (:127), unclip (:141), crops (:155; the reference
  allows 1% of values one level off, the oracle matches all of these), the
  recogniser tensor (:192), CTC decode with the 18 710-class dictionary
  (:214), page lines (:256), and the small cases of :233-337;
- on the GPU, the product's input preparation (`ppocr_det_input_hwc`,
  `ppocr_rec_input_hwc`) and text mask (`ppocr_db_mask`) on the same
  fixtures, bit for bit.
"""

from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np
import pytest

from common import Device

REF = Path(__file__).resolve().parent / "golden" / "ref"
FIX = json.loads((REF / "fixtures.json").read_text())


def npy(name: str) -> np.ndarray:
    return np.load(REF / name)


# ------------------------------------------------------------------ oracle

def test_resize_matches_opencv(oracle_mod):
    noise = npy("noise.npy")
    for case in FIX["resize"]:
        got = oracle_mod.resize_linear(noise, case["width"], case["height"])
        assert np.array_equal(got, npy(case["file"])), case


def test_det_input_matches_rapidocr(oracle_mod):
    noise = npy("noise.npy")
    w, h = oracle_mod.det_size(noise.shape[1], noise.shape[0])
    assert (w, h) == (32, 32), "40x28 snaps to 32x32"
    want = npy(FIX["det_input"]["file"])[0].transpose(1, 2, 0)
    got = oracle_mod.det_input_hwc(noise, w, h, FIX["det_input"]["mean"], FIX["det_input"]["std"])
    assert np.array_equal(got.view(np.uint32), np.ascontiguousarray(want).view(np.uint32))


def test_contours_match_opencv(oracle_mod):
    for i, case in enumerate(FIX["contours"]):
        assert oracle_mod.find_contours(npy(case["file"])) == case["contours"], f"mask {i}"


def test_db_boxes_match_rapidocr(oracle_mod):
    case = FIX["boxes"]
    got = oracle_mod.boxes_from_prob(npy(case["file"]), *case["dest"])
    assert np.array_equal(got, np.asarray(case["boxes"], np.float32))


def test_min_area_rect_matches_opencv(oracle_mod):
    for case in FIX["min_area_rect"]:
        got = oracle_mod.min_area_rect_points(case["points"])
        assert np.array_equal(got, np.asarray(case["box"], np.float32)), case["points"]


def test_unclip_matches_pyclipper(oracle_mod):
    for case in FIX["unclip"]:
        assert oracle_mod.unclip(case["quad"], 1.5) == case["ring"], case["quad"]


def test_crops_match_opencv(oracle_mod):
    page = npy("page.npy")
    for case in FIX["crops"]:
        want = npy(case["file"])
        got = oracle_mod.crop_text(page, case["quad"])
        assert got.shape == want.shape, case["quad"]
        off = got.astype(np.int16) - want.astype(np.int16)
        assert np.abs(off).max() <= 1 and np.count_nonzero(off) * 100 <= off.size, case["quad"]


def test_rec_input_matches_rapidocr(oracle_mod):
    for case in FIX["rec_input"]:
        want = npy(case["input"])
        got = oracle_mod.rec_input_hwc(npy(case["crop"]))
        assert got.shape[1] == want.shape[3]
        assert np.array_equal(got, want[0].transpose(1, 2, 0))


def test_ctc_matches_rapidocr(oracle_mod):
    classes = oracle_mod.dictionary((REF / "characters.txt").read_text(encoding="utf-8"))
    assert len(classes) == 18710, "classes of PP-OCRv6 small"
    for case in FIX["ctc"]:
        best = npy(f"{case['stem']}_argmax.npy").astype(np.uint32)
        prob = npy(f"{case['stem']}_maxprob.npy")
        text, score = oracle_mod.ctc_decode(best, prob, classes)
        assert text == case["text"], case["stem"]
        assert score == case["score"], case["stem"]


def test_dictionary_splits_like_python(oracle_mod):
    assert oracle_mod.dictionary("a\r\nb\x1cc \nd\n") == ["blank", "a", "b", "c", "", "d", " "]


def test_page_lines_match_worker(oracle_mod):
    case = FIX["page_lines"]
    h, w = case["image_hw"]
    lines = oracle_mod.page_lines(np.asarray(case["boxes"], np.float32), [tuple(r) for r in case["reads"]],
                                  case["ratio_w"], case["ratio_h"], 0, w, h)
    exp = case["expected"]
    assert np.array_equal(np.array([q for q, _, _ in lines]), np.asarray(exp["boxes"], np.float32))
    assert [t for _, t, _ in lines] == exp["txts"]
    assert [s for _, _, s in lines] == exp["scores"]


def test_padding_score_filter_and_empty_pages(oracle_mod):
    # apply_vertical_padding with width_height_ratio -1, min_height 30 (parity.rs:296-299)
    for h, w, pad in [(100, 100, 0), (20, 100, 20), (10, 200, 25)]:
        got = oracle_mod.prepare_page(w, h, min_side=1, whr=-1.0, min_height=30)  # no upscale: the band alone
        assert got is not None and got[4] == pad, (w, h, got)
    quad = [[0, 0], [9, 0], [9, 9], [0, 9]]
    lines = oracle_mod.page_lines([quad, quad], [("ab", math.nan), ("cd", 0.1)], 1.0, 1.0, 0, 10, 10)
    assert [t for _, t, _ in lines] == ["ab"]
    for w, h in [(100, 0), (0, 100), (0, 0)]:
        assert oracle_mod.prepare_page(w, h) is None
        assert oracle_mod.det_size(w, h, 32) is None and oracle_mod.det_size(w, h) is None
    assert oracle_mod.prepare_page(4096, 1) is None  # padded past 4096 squared
    fw, fh, _, _, pad = oracle_mod.prepare_page(4096, 20)  # a line: 6144 x 32, padded to 1536 rows
    assert (fw, fh, pad) == (6144, 1536, 752)
    # the benchmark page: 2550 x 3300 keeps its size and goes to the detector at 1536 x 1984
    assert oracle_mod.prepare_page(2550, 3300) == (2550, 3300, 1.0, 1.0, 0)
    assert oracle_mod.det_size(2550, 3300) == (1536, 1984)


# --------------------------------------------------------------------- GPU

@pytest.mark.gpu
def test_gpu_det_input_on_the_reference_fixture(cuda_mod):
    noise = npy("noise.npy")
    want = np.ascontiguousarray(npy(FIX["det_input"]["file"])[0].transpose(1, 2, 0))
    with Device() as dev:
        din, dout = dev.put(noise), dev.alloc(want.nbytes)
        cuda_mod.det_input_hwc(din, 40, 28, 32, 32, FIX["det_input"]["mean"], FIX["det_input"]["std"], dout)
        got = dev.get(dout, want.shape, np.float32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.gpu
def test_gpu_resize_stage_on_the_reference_fixtures(cuda_mod):
    """The detector-input kernel with mean 0 and std 1/255 in f64 returns
    byte * (f32)(1/255) * 255 rounded: the resized byte itself, so the
    kernel's resize is checked against OpenCV's outputs at all five sizes."""
    noise = npy("noise.npy")
    for case in FIX["resize"]:
        w, h = case["width"], case["height"]
        want = npy(case["file"])
        with Device() as dev:
            din, dout = dev.put(noise), dev.alloc(w * h * 3 * 4)
            cuda_mod.det_input_hwc(din, 40, 28, w, h, [0, 0, 0], [1 / 255] * 3, dout)
            got = dev.get(dout, (h, w, 3), np.float32)
        assert np.array_equal(np.rint(got).astype(np.uint8), want), case


@pytest.mark.gpu
def test_gpu_rec_input_on_the_reference_fixtures(cuda_mod):
    for case in FIX["rec_input"]:
        crop = npy(case["crop"])
        want = np.ascontiguousarray(npy(case["input"])[0].transpose(1, 2, 0))
        with Device() as dev:
            din, dout = dev.put(crop), dev.alloc(want.nbytes)
            width = cuda_mod.rec_input_hwc(din, crop.shape[1], crop.shape[0], dout, want.size)
            got = dev.get(dout, want.shape, np.float32)
        assert width == want.shape[1]
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.gpu
def test_gpu_db_mask_on_the_reference_prob_map(cuda_mod, oracle_mod):
    """The mask of prob.npy gives the contours the oracle finds, and through
    them the fixture's 11 boxes."""
    prob = npy(FIX["boxes"]["file"])
    with Device() as dev:
        dp, dm = dev.put(prob), dev.alloc(prob.size)
        cuda_mod.db_mask(dp, prob.size, 0.3, dm)
        mask = dev.get(dm, prob.shape, np.uint8)
    assert np.array_equal(mask, (prob > np.float32(0.3)).astype(np.uint8))
    assert oracle_mod.find_contours(mask) == oracle_mod.find_contours((prob > np.float32(0.3)).astype(np.uint8))
