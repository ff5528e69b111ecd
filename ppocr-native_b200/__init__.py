"""ppocr-native B200: the neural inference hot path of ppocr-native (the
PP-OCRv6 detector and recogniser executed from PPOCRPL1 plans) as
hand-written sm_100a CUDA kernels behind a C ABI (`include/ppocr_cuda.h`).

Python here is the binding and the test/bench harness: `cuda` wraps the C ABI
with ctypes (the library is opened on first use), `plan` writes plan files,
`synth` builds the synthetic networks.
"""

from . import cuda, plan, synth, workload  # noqa: F401

__all__ = ["cuda", "plan", "synth", "workload"]
