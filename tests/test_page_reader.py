"""The page path on the GPU: crop_text (`ppocr_crop_text`) and the page
reader (`ppocr_reader_*`: page fit, detector input, detector, mask, box
scores, DB boxes, crops, recogniser inputs, recogniser, CTC decode, page
lines) against the CPU oracle's whole-page read (oracle/oracle.py
read_page: the oracle's engine and page steps, pinned to the reference's
fixtures).

In the exact mode (PPOCR_OPT_NO_TENSOR_CORES) the detector gives the
oracle's bits, so maps and boxes must be identical, and the recogniser's
classes too; its 1/sum of exponentials is summed per column block and
merged (within 1e-5 of the reference's online sum), so a score, the mean
of probabilities rounded to five decimals, is checked within 2e-5. With the
tensor cores (3xTF32) the maps and probabilities differ from the oracle's by
the 3xTF32 rounding: the boxes are checked against the oracle's DB
postprocess on the reader's own map (identical), the texts against the
oracle's recogniser on the same crops (classes are exact by construction,
so identical texts), the scores within 2e-5 (two roundings to five
decimals of probabilities within 1e-5).

Pages: a small seeded synthetic page with a set-weight "darkness" detector
(real text boxes), and the benchmark's full-size 2550 x 3300 page with the
random-init detector and an 18 710-class recogniser (its map is a near-
constant 0.5: one page-sized box; its 44 generator quads are recognised).
"""

from __future__ import annotations

import threading

import numpy as np
import pytest

from common import Device
from ppocr_native_b200 import synth, workload

pytestmark = pytest.mark.gpu

SMALL_VOCAB = 500


@pytest.fixture(scope="module")
def small(cuda_mod, oracle_mod):
    det_plan, rec_plan = synth.darkness_det_plan(), synth.rec_plan(seed=12, std=None, vocab=SMALL_VOCAB)
    text = synth.characters(SMALL_VOCAB)
    det, rec = cuda_mod.Model(det_plan), cuda_mod.Model(rec_plan)
    yield dict(det=det, rec=rec, text=text, det_plan=det_plan, rec_plan=rec_plan,
               classes=oracle_mod.dictionary(text))
    det.close()
    rec.close()


def oracle_read(oracle_mod, env, page, quads=None):
    return oracle_mod.read_page(page, oracle_mod.Oracle(env["det_plan"]), oracle_mod.Oracle(env["rec_plan"]),
                                env["classes"], quads=quads)


def same_reads(got, want):
    assert [t for t, _ in got] == [t for t, _ in want]
    assert all(abs(a - b) <= 2e-5 for (_, a), (_, b) in zip(got, want))


def same_lines(got, want):
    assert len(got) == len(want)
    for (q1, t1, s1), (q2, t2, s2) in zip(got, want):
        assert np.array_equal(q1, q2) and t1 == t2 and abs(s1 - s2) <= 2e-5


# ------------------------------------------------------------------- crops

QUADS = [[[6, 9], [200, 9], [200, 31], [6, 31]], [[10.5, 40.25], [190.75, 44.5], [189.5, 70.0], [9.25, 66.75]],
         [[30, 20], [52, 20], [52, 110], [30, 110]], [[-3, 100], [230, 98], [231, 125], [-2, 127]],
         [[200, 5], [215, 5], [215, 119], [200, 119]], [[0, 0], [1, 0], [1, 1], [0, 1]],
         [[100, 50], [100.4, 50], [100.4, 50.2], [100, 50.2]], [[219, 119], [300, 130], [310, 160], [215, 140]]]


def test_gpu_crops_are_the_oracles(cuda_mod, oracle_mod):
    """Bit for bit against the oracle (itself identical to OpenCV's crops on
    the reference fixtures), on the fixture page: turned, out-of-page,
    sub-pixel and empty crops."""
    page = np.load(__import__("pathlib").Path(__file__).resolve().parent / "golden" / "ref" / "page.npy")
    rng = np.random.default_rng(4)
    quads = QUADS + [(np.array(QUADS[1]) + rng.uniform(-8, 8, (4, 2))).tolist() for _ in range(20)]
    with Device() as dev:
        dimg = dev.put(page)
        for q in quads:
            want = oracle_mod.crop_text(page, q)
            w, h = cuda_mod.crop_size(q)
            assert (h, w) == want.shape[:2], q
            dout = dev.alloc(max(want.nbytes, 1))
            cuda_mod.crop_text(dimg, page.shape[1], page.shape[0], q, dout, want.nbytes)
            got = dev.get(dout, want.shape, np.uint8)
            assert np.array_equal(got, want), q


def test_gpu_crops_of_the_benchmark_page(cuda_mod, oracle_mod):
    page, quads = workload.synthetic_page(5)
    with Device() as dev:
        dimg = dev.put(page)
        for q in quads[::4]:
            want = oracle_mod.crop_text(page, q)
            dout = dev.alloc(want.nbytes)
            cuda_mod.crop_text(dimg, page.shape[1], page.shape[0], q, dout, want.nbytes)
            assert np.array_equal(dev.get(dout, want.shape, np.uint8), want)


# ------------------------------------------------------------------ reader

def test_reader_exact_mode_is_the_oracle(cuda_mod, oracle_mod, small):
    page, _ = workload.synthetic_page(3, lines=8, width=640, height=800)
    want = oracle_read(oracle_mod, small, page)
    assert len(want["boxes"]) > 8
    with cuda_mod.Reader(small["det"], small["rec"], small["text"]) as r:
        r.set_options(cuda_mod.OPT_NO_TENSOR_CORES)
        for _ in range(2):  # the second page reuses every buffer
            lines = r.read(page)
            assert np.array_equal(r.prob_map(), want["prob"])
            assert np.array_equal(r.boxes(), want["boxes"])
            same_reads(r.texts(), want["reads"])
            same_lines(lines, want["lines"])


def test_reader_tensor_cores(cuda_mod, oracle_mod, small):
    page, quads = workload.synthetic_page(8, lines=10, width=700, height=900)
    with cuda_mod.Reader(small["det"], small["rec"], small["text"]) as r:
        boxes = r.detect(page)
        prob = r.prob_map()
        want = oracle_read(oracle_mod, small, page)
        assert float(np.abs(prob - want["prob"]).max()) <= 1e-4
        assert np.array_equal(boxes, oracle_mod.boxes_from_prob(prob, 700, 900))
        scored, rescored = r.stats()
        assert scored >= len(boxes) and rescored <= scored
        reads = r.recognise(quads)
        same_reads(reads, oracle_read(oracle_mod, small, page, quads=quads)["reads"])


@pytest.mark.parametrize("size", [(5000, 300), (2000, 100), (25, 200), (20, 10)])
def test_reader_fits_and_pads_pages(cuda_mod, oracle_mod, small, size):
    """Pages the reference resizes (long side over 4096, short side under
    30) or pads (wider than 8 x their height), exact mode."""
    w, h = size
    rng = np.random.default_rng(w + h)
    page = np.full((h, w, 3), 255, np.uint8)
    for _ in range(6):
        y, x = int(rng.integers(0, max(1, h - 8))), int(rng.integers(0, max(1, w - 30)))
        page[y:y + int(rng.integers(3, 30)), x:x + int(rng.integers(5, 200))] = int(rng.integers(0, 80))
    want = oracle_read(oracle_mod, small, page)
    with cuda_mod.Reader(small["det"], small["rec"], small["text"]) as r:
        r.set_options(cuda_mod.OPT_NO_TENSOR_CORES)
        lines = r.read(page)
        prep = oracle_mod.prepared_image(page)
        assert r.prepared()[:2] == prep[0].shape[1::-1]
        assert np.array_equal(r.boxes(), want["boxes"])
        same_reads(r.texts(), want["reads"])
        same_lines(lines, want["lines"])


def test_readers_on_threads_agree(cuda_mod, small):
    """Readers on several host threads (shared weights, own streams) give
    each page the same lines as one reader alone."""
    pages = [workload.synthetic_page(20 + i, lines=6, width=600, height=700)[0] for i in range(4)]
    with cuda_mod.Reader(small["det"], small["rec"], small["text"]) as r:
        alone = [r.read(p) for p in pages]
    readers = [cuda_mod.Reader(small["det"], small["rec"], small["text"]) for _ in range(4)]
    got = [None] * 4
    errors = []

    def work(i):
        try:
            got[i] = [readers[i].read(pages[(i + k) % 4]) for k in range(4)]
        except Exception as e:  # surfaced below
            errors.append(e)

    threads = [threading.Thread(target=work, args=(i,)) for i in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    for rd in readers:
        rd.close()
    assert not errors, errors
    for i in range(4):
        for k in range(4):
            same_lines(got[i][k], alone[(i + k) % 4])


def test_reader_on_the_benchmark_page(cuda_mod, oracle_mod):
    """Benchmark config 4: a 2550 x 3300 page, the random-init detector at
    1984 x 1536 and the 18 710-class recogniser. The DB boxes are the
    oracle's on the reader's own map; the 44 generator quads read the
    oracle's texts."""
    page, quads = workload.synthetic_page(1)
    det_plan, rec_plan = synth.det_plan(seed=0), synth.rec_plan(seed=1)
    text = synth.characters(synth.VOCAB)
    classes = oracle_mod.dictionary(text)
    with cuda_mod.Model(det_plan) as det, cuda_mod.Model(rec_plan) as rec, \
            cuda_mod.Reader(det, rec, text) as r:
        boxes = r.detect(page)
        assert r.prepared() == (2550, 3300, 1.0, 1.0, 0)
        prob = r.prob_map()
        assert prob.shape == (1984, 1536)
        assert np.array_equal(boxes, oracle_mod.boxes_from_prob(prob, 2550, 3300))
        reads = r.recognise(quads)
    rec_o = oracle_mod.Oracle(rec_plan)
    for q, (t, s) in list(zip(quads, reads))[::6]:
        crop = oracle_mod.crop_text(page, q)
        x = oracle_mod.rec_input_hwc(crop)
        rec_o.set_size(48, x.shape[1])
        out = rec_o.run(x.reshape(-1))[0].reshape(-1, 2)
        wt, ws = oracle_mod.ctc_decode(out[:, 0].astype(np.uint32), out[:, 1], classes)
        assert t == wt and abs(s - ws) <= 2e-5


def test_reader_without_a_page(cuda_mod, small):
    with cuda_mod.Reader(small["det"], small["rec"], small["text"]) as r:
        with pytest.raises(cuda_mod.PpocrError) as e:
            r.recognise([[0, 0], [9, 0], [9, 9], [0, 9]])
        assert e.value.code == cuda_mod.E_ARG
        empty = np.zeros((0, 0, 3), np.uint8)
        assert r.read(empty) == [] and len(r.boxes()) == 0


def test_reader_pages_of_changing_line_counts(cuda_mod, small):
    """Pages whose line counts and widths change from page to page (config 5's
    stream: the recogniser's lanes are laid out anew for every page while
    its buffers are kept) read each as a fresh reader reads it alone."""
    pages = [workload.synthetic_page(40 + i, lines=n, width=500, height=900) for i, n in enumerate((9, 2, 12, 1, 6))]
    alone = []
    for page, quads in pages:
        with cuda_mod.Reader(small["det"], small["rec"], small["text"]) as r:
            r.detect(page)
            alone.append(r.recognise(quads))
    with cuda_mod.Reader(small["det"], small["rec"], small["text"]) as r:
        for _ in range(3):
            for (page, quads), want in zip(pages, alone):
                r.detect(page)
                assert r.recognise(quads) == want
