"""Synthetic benchmark inputs with the shapes of the reference's page stream.

A 300-dpi page of 2550 x 3300 pixels goes to the detector at 1984 x 1536
(`det_size`, ppocr-native `src/det.rs:166-189`: the long side to 2000, both
snapped to multiples of 32), and each of its text lines to the recogniser at
height 48 and width max(320, 48 * w / h) (`src/rec.rs:19-43`), up to 16
lines per run (`src/bin/ppocr-native/ocr.rs:424`). The benchmark pages carry
44 lines whose crops are 80-1600 px wide at height 48 (benchmark config 4);
tensor values are ~N(0, 1) (configs 2-3). No dataset is involved: the
reference's own measurement set (10 printed pages) is not in its repository.
"""

from __future__ import annotations

import numpy as np

from .synth import PAGE_DET_SIZE, REC_HEIGHT

REC_MIN_WIDTH = 320
LINES_PER_PAGE = 44
LINES_PER_RUN = 16


def line_widths(seed: int, lines: int = LINES_PER_PAGE) -> list[int]:
    """Recogniser input widths of one page's lines: crops 80-1600 px wide at
    height 48, narrower ones padded to 320."""
    rng = np.random.default_rng(seed)
    crops = rng.integers(80, 1601, size=lines)
    return [max(REC_MIN_WIDTH, int(w)) for w in crops]


def runs(widths: list[int], per_run: int = LINES_PER_RUN) -> list[list[int]]:
    """The lines in reading order, cut into runs of at most 16."""
    return [widths[i:i + per_run] for i in range(0, len(widths), per_run)]


class Page:
    """One page's detector input and recogniser inputs (HWC f32)."""

    def __init__(self, seed: int, det_size: tuple[int, int] = PAGE_DET_SIZE, lines: int = LINES_PER_PAGE):
        rng = np.random.default_rng(seed)
        h, w = det_size
        self.det = rng.standard_normal((h, w, 3), dtype=np.float32)
        self.widths = line_widths(seed + 1, lines)
        self.lines = [rng.standard_normal((REC_HEIGHT, wd, 3), dtype=np.float32) for wd in self.widths]

    @property
    def runs(self) -> list[list[int]]:
        """Line indices per recogniser run."""
        idx = list(range(len(self.widths)))
        return [idx[i:i + LINES_PER_RUN] for i in range(0, len(idx), LINES_PER_RUN)]

    def input_bytes(self) -> int:
        return self.det.nbytes + sum(x.nbytes for x in self.lines)


# ------------------------------------------------------- synthetic pages

PAGE_WIDTH, PAGE_HEIGHT = 2550, 3300  # a 300-dpi letter page


def synthetic_page(seed: int, lines: int = LINES_PER_PAGE, width: int = PAGE_WIDTH, height: int = PAGE_HEIGHT):
    """A seeded 300-dpi page as benchmark config 4 describes it: white, `lines`
    horizontal rows of dark glyph-like rectangles of random widths, 20-40 px
    tall with 1-3 px gaps, gray noise of sigma 4; 8-bit, channels together.

    Each row's length is chosen so that its crop at height 48 is 80-1600 px
    wide. Returns the page (height, width, 3) uint8 and the rows' quads
    (lines, 4, 2) float32 (top-left, top-right, bottom-right, bottom-left:
    each row's outer edges) on the page.
    """
    rng = np.random.default_rng(seed)
    page = np.full((height, width), 255.0, np.float32)
    pitch = (height - 200) / max(lines, 1)
    quads = np.zeros((lines, 4, 2), np.float32)
    for i in range(lines):
        h = int(rng.integers(20, 41))
        y0 = int(100 + i * pitch + rng.integers(0, max(1, int(pitch) - h)))
        target = int(rng.integers(80, 1601))  # crop width at height 48
        length = min(max(int(round(target * h / 48)), 8), width - 200)
        x0 = int(rng.integers(100, width - 100 - length + 1))
        x, end = x0, x0 + length
        while x < end:
            gw = min(int(rng.integers(4, 25)), end - x)
            page[y0:y0 + h, x:x + gw] = float(rng.integers(0, 90))
            x += gw + int(rng.integers(1, 4))
        quads[i] = [[x0, y0], [end, y0], [end, y0 + h], [x0, y0 + h]]
    page += rng.standard_normal(page.shape, dtype=np.float32) * np.float32(4.0)
    gray = np.clip(np.rint(page), 0, 255).astype(np.uint8)
    return np.repeat(gray[:, :, None], 3, axis=2), quads


def page_stream(seed: int, pages: int, distinct: int | None = None):
    """Benchmark config 5's stream: `pages` pages with 20-60 lines each, drawn
    from `distinct` seeded pages (all distinct when None)."""
    rng = np.random.default_rng(seed)
    counts = rng.integers(20, 61, size=pages if distinct is None else distinct)
    return [(seed * 100003 + k, int(counts[k])) for k in range(len(counts))]
