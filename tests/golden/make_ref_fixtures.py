"""Copy the reference's own parity fixtures into tests/golden/ref/.

    python tests/golden/make_ref_fixtures.py REFERENCE_ROOT

ppocr-native's `tests/fixtures/` holds the outputs of the libraries its host
page steps reproduce (OpenCV 5.0, pyclipper 1.4, RapidOCR 3.9, numpy 2.5),
written by its `tools/make_fixtures.py` and asserted by its
`tests/parity.rs:47-337`: resize (`resize_*.npy` from `noise.npy`), the
detector tensor (`det_input.npy`), contours (`mask_*.npy`), DB boxes
(`prob.npy`), minimum-area rectangles, unclip rings, crops (`page.npy` ->
`crop_*.npy`), recogniser tensors (`rec_crop_*` -> `rec_input_*`), CTC decode
(`ctc_*_{argmax,maxprob}.npy` + `characters.txt`) and page lines, with the
expected values in `fixtures.json`. They are data, copied unchanged, so the
tests here run on the GPU box where the reference tree does not exist.
"""

from __future__ import annotations

import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "ref"


def main(root: str) -> None:
    src = Path(root) / "tests" / "fixtures"
    if not src.is_dir():
        raise SystemExit(f"{src} is missing")
    OUT.mkdir(exist_ok=True)
    names = sorted(p.name for p in src.iterdir() if p.suffix in (".npy", ".json", ".txt"))
    for name in names:
        shutil.copyfile(src / name, OUT / name)
    print(f"copied {len(names)} files into {OUT}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_ref_fixtures.py REFERENCE_ROOT")
    main(sys.argv[1])
