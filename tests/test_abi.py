"""The C ABI without a GPU: the library builds, loads, exports every entry
point `include/ppocr_cuda.h` declares, and checks plans on the host exactly
as the reference does before touching a device."""

from __future__ import annotations

import re
from pathlib import Path

import numpy as np
import pytest

from ppocr_native_b200 import cuda, synth
from test_oracle import good_file, malformed_files

ROOT = Path(__file__).resolve().parent.parent


def declared() -> set[str]:
    text = (ROOT / "include" / "ppocr_cuda.h").read_text()
    return set(re.findall(r"\b(ppocr_[a-z_0-9]+)\s*\(", text))


def test_library_exports_every_declared_entry_point():
    lib = cuda.lib()
    names = declared()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), name
    assert names <= set(cuda._SIG), names - set(cuda._SIG)


@pytest.mark.parametrize("what,data", malformed_files(), ids=[c[0] for c in malformed_files()])
def test_malformed_plans_refused_before_any_device(what, data):
    with pytest.raises(cuda.PpocrError) as e:
        cuda.Model(data)
    assert e.value.code == cuda.E_PLAN, (what, str(e.value))


def test_plans_that_parse_reach_the_device_check():
    for plan in (good_file(), synth.page_model_plan(16, 16), synth.line_model_plan(40),
                 synth.fused_layer_plan(h=8, w=8)):
        if cuda.device_count() == 0:
            with pytest.raises(cuda.PpocrError) as e:
                cuda.Model(plan, device=0)
            assert e.value.code == cuda.E_DEVICE
        with pytest.raises(cuda.PpocrError) as e:
            cuda.Model(plan, device=99)
        assert e.value.code == cuda.E_DEVICE


def test_plan_file_path_errors():
    with pytest.raises(cuda.PpocrError) as e:
        cuda.Model("/nonexistent/plan")
    assert e.value.code == cuda.E_PLAN


def test_det_and_rec_plans_parse(tmp_path):
    # the synthetic networks are valid PPOCRPL1 files with codes 0-6 only
    from ppocr_native_b200.plan import describe

    for plan in (synth.det_plan(), synth.rec_plan()):
        d = describe(plan)
        assert all(op.fused != "hardswish" for op in d["ops"])
        p = tmp_path / "x.plan"
        p.write_bytes(plan)
        with pytest.raises(cuda.PpocrError) as e:
            cuda.Model(p, device=99)
        assert e.value.code == cuda.E_DEVICE
    assert np.isfinite(describe(synth.det_plan())["weights"]).all()


def test_input_preparation_arguments_checked_before_any_device():
    """The GPU input-preparation entry points refuse null pointers and empty
    or oversized images with their codes before touching a device, and the
    recogniser's tensor width follows rec.rs:20-31 (no device needed)."""
    with pytest.raises(cuda.PpocrError) as e:
        cuda.det_input_hwc(0, 10, 10, 8, 8, [0, 0, 0], [1, 1, 1], 0)
    assert e.value.code == cuda.E_ARG
    with pytest.raises(cuda.PpocrError) as e:
        cuda.det_input_hwc(16, 0, 10, 8, 8, [0, 0, 0], [1, 1, 1], 16)
    assert e.value.code == cuda.E_SIZE
    with pytest.raises(cuda.PpocrError) as e:
        cuda.db_mask(0, 10, 0.3, 16)
    assert e.value.code == cuda.E_ARG
    with pytest.raises(cuda.PpocrError) as e:
        cuda.rec_input_width(0, 48)
    assert e.value.code == cuda.E_SIZE
    # the tensor width: at least 320, else trunc(48 * w / h)
    assert cuda.rec_input_width(100, 48) == 320
    assert cuda.rec_input_width(1500, 17) == int(48 * (1500 / 17))
    assert cuda.rec_input_width(2000, 100) == 960
    with pytest.raises(cuda.PpocrError) as e:  # out too small for 48 x 320 x 3
        cuda.rec_input_hwc(16, 100, 48, 16, 10)
    assert e.value.code == cuda.E_SIZE
    with pytest.raises(cuda.PpocrError) as e:  # out too small for 8 x 8 x 3
        cuda.det_input_hwc(16, 10, 10, 8, 8, [0, 0, 0], [1, 1, 1], 16, capacity=8 * 8 * 3 - 1)
    assert e.value.code == cuda.E_SIZE


def test_noalloc_refuses_misaligned_buffers_before_any_launch():
    """The no-allocation CTC head reads its weight panels as 16-byte vectors:
    a w that is not 16-byte aligned (or a float buffer that is not 4-byte
    aligned) is an argument error, returned before any device work."""
    for x, w, b, y in ((256, 260, 512, 768), (257, 256, 512, 768), (256, 256, 514, 768), (256, 256, 512, 770)):
        with pytest.raises(cuda.PpocrError) as e:
            cuda.ctc_argmax_noalloc(x, w, b, y, 40, 120, 18710)
        assert e.value.code == cuda.E_ARG, (x, w, b, y)
        assert "aligned" in str(e.value)
