"""Benchmark: synthetic 300-dpi pages read end to end on B200, one process per
GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload page|stream|neural|det|rec|layer|conv3x3|dw3x3]

The headline workload (`page`, benchmark config 4): a seeded 2550 x 3300
8-bit page (44 rows of glyph-like rectangles) goes through the public page
reader (include/ppocr_cuda.h `ppocr_reader_*`): the page bytes to the GPU,
the detector's input (OpenCV resize + normalization) at 1984 x 1536, the
detector, the text mask, border following and box scores, the DB boxes, the
crops of the page's 44 line quads, their recogniser inputs, the recogniser
over all lines of the page as lanes of one run, the CTC decode. The
detector's weights are random-init (N(0, 0.02)) as the configuration asks,
so its map is a near-constant 0.5 and the DB postprocess finds one
page-sized box; the lines recognised are therefore the generator's own 44
quads, cropped from the page through the same crop path (the DB
postprocess still runs in full on every page).

A step is one page per reader in flight (`--readers`, each on its own host
thread and stream, weights shared). `value`: pages/s with the pages already
in HBM; `e2e`: the same through the C ABI from page-locked host pages, the
page's bytes copied in and every result (mask, scores, reads) copied out
inside the timed region. `--workload stream` is config 5: 800 pages of 20-60
lines sharded by page over the ranks (strong scaling). With N > 1 each rank
reads its own pages; ranks exchange nothing but the timing.

`--impl reference` times the reference CPU path on this host: the C
restatement of ppocr-native's CPU engine and host page steps (oracle/; the
reference itself is Rust and cannot be built here), all host threads.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import faulthandler
import importlib.util
import itertools
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
PKG_DIR = ROOT / "ppocr-native_b200"
sys.path.insert(0, str(ROOT))

L2_FLUSH_BYTES = 256 << 20  # larger than the 126 MB L2
# DRAM bytes (read + written) of one launch of each probed kernel, from one
# ncu capture of its probe command (dram__bytes_read.sum +
# dram__bytes_write.sum; writes still dirty in L2 at the kernel's end are not
# counted there): `bench.py --workload layer|conv3x3|dw3x3 --profile
# --steps 2 --warmup 1` under `ncu -k regex:<kernel> -c 1`.
TRAFFIC = {
    "layer": (94.74e6, "pw_tc_kernel, bench.py --workload layer"),
    "conv3x3": (78.19e6, "conv_tc_kernel, bench.py --workload conv3x3"),
    "dw3x3": (107.59e6, "dw_row_kernel, bench.py --workload dw3x3"),
}
METRIC = "synthetic-page pages/s (2550x3300 page -> det 1984x1536 -> DB boxes -> crops -> rec -> CTC decode) per B200 job"


def package():
    name = "ppocr_native_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


# ----------------------------------------------------------------- plumbing

class Dist:
    def __init__(self):
        self.rank = int(os.environ.get("RANK", 0))
        self.world = int(os.environ.get("WORLD_SIZE", 1))
        self.local = int(os.environ.get("LOCAL_RANK", 0))
        self.pg = None
        self.device = "cuda"

    def init(self, backend: str):
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=300))
            self.pg = dist
            self.device = "cuda" if backend == "nccl" else "cpu"

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch

        t = torch.tensor([v], dtype=torch.float64, device=self.device)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def gather(self, values: list[float]) -> list[list[float]]:
        """Every rank's `values` (same length on every rank), on every rank."""
        if not self.pg:
            return [values]
        import torch

        t = torch.tensor(values, dtype=torch.float64, device=self.device)
        out = [torch.empty_like(t) for _ in range(self.world)]
        self.pg.all_gather(out, t)
        return [o.tolist() for o in out]

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()

    def whole_job(self, units_per_rank: float, local_seconds: float) -> tuple[float, float]:
        """Units of all ranks per second over the slowest rank's time (every
        rank reads the same number of its own pages: weak scaling), and that
        time."""
        t = self.max(local_seconds)
        return self.world * units_per_rank / t, t


class Clocks:
    """nvidia-smi samples of SM clock and throttle reasons while running."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.device)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = max(mx, float(parts[1]))
            except ValueError:
                continue
            for name, val in zip(names, parts[4:8]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_threads() -> int:
    return len(os.sched_getaffinity(0))


def peaks() -> dict:
    p = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    hbm, bf16 = p.get("hbm_gbs"), p.get("bf16_tflops")
    out = {"hbm": hbm, "hbm_source": "measured: MEASURED_PEAKS.json hbm_gbs (copy, burst)",
           "bf16": bf16, "bf16_source": "measured: MEASURED_PEAKS.json bf16_tflops (cuBLAS, burst)"}
    if hbm is None:
        out["hbm"], out["hbm_source"] = 6650.0, "fallback: 6.65 TB/s"
    if bf16 is None:
        out["bf16"], out["bf16_source"] = 1590.0, "fallback: 1.59 PFLOP/s"
    return out


# ------------------------------------------------------------- the pages

def make_pages(seeds_lines, threads: int = 8):
    """Synthetic pages (config 4 generator) for (seed, lines) pairs, made on
    host threads: [(page (h, w, 3) uint8, quads (n, 4, 2) float32)]."""
    workload = package().workload
    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        return list(ex.map(lambda sl: workload.synthetic_page(sl[0], lines=sl[1]), seeds_lines))


class PagePool:
    """Pages in page-locked host memory and, for the device-resident run, in
    HBM; each with its line quads."""

    def __init__(self, torch, device: int, pages):
        self.host, self.dev, self.quads = [], [], []
        for page, quads in pages:
            h = torch.from_numpy(page).pin_memory()
            self.host.append(h)
            self.dev.append(h.to(f"cuda:{device}", non_blocking=False))
            self.quads.append(np.ascontiguousarray(quads.reshape(-1, 8), dtype=np.float32))
        self.h, self.w = pages[0][0].shape[:2]
        torch.cuda.synchronize()

    def __len__(self):
        return len(self.host)


def read_pages(torch, readers, pool: PagePool, total: int, on_device: bool, main):
    """`total` pages (pool pages in turn) over the readers, one host thread
    each; every page: detection (the full DB postprocess on the model's
    map), then the page's line quads recognised and their texts read on the
    host. Returns device seconds (CUDA events on `main`, every reader stream
    ordered between them), wall seconds, host CPU seconds, per-page wall
    latencies and kernel launches per page."""
    counter = itertools.count()
    lock = threading.Lock()
    errors, lat, launches = [], [], []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(main)
    streams = [torch.cuda.ExternalStream(r.stream) for r in readers]
    for st in streams:
        st.wait_event(e0)

    def work(r):
        try:
            while True:
                with lock:
                    i = next(counter)
                if i >= total:
                    return
                k = i % len(pool)
                t0 = time.perf_counter()
                if on_device:
                    r.detect_ptr(pool.dev[k].data_ptr(), pool.w, pool.h, on_device=True)
                else:
                    r.detect_ptr(pool.host[k].data_ptr(), pool.w, pool.h)
                q = pool.quads[k]
                r.recognise_ptr(q.ctypes.data, len(q))
                texts = r.texts()  # the page's result, read on the host
                if len(texts) != len(q):
                    raise RuntimeError("a read is missing")
                lat.append(time.perf_counter() - t0)
                launches.append(r.launches)
        except Exception as e:  # reported by the caller
            errors.append(e)

    cpu0, w0 = time.process_time(), time.perf_counter()
    threads = [threading.Thread(target=work, args=(r,)) for r in readers]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    wall = time.perf_counter() - w0
    cpu = time.process_time() - cpu0
    if errors:
        raise errors[0]
    for st in streams:
        ev = torch.cuda.Event()
        ev.record(st)
        main.wait_event(ev)
    e1.record(main)
    e1.synchronize()
    return e0.elapsed_time(e1) / 1e3, wall, cpu, lat, (statistics.median(launches) if launches else 0)


# ------------------------------------------------------ secondary measures

class NeuralPipeline:
    """The detector and the recogniser runs of one page's tensors (seeded
    N(0, 1) inputs of the page's shapes), queued on one stream: the neural
    hot path alone, device-resident."""

    def __init__(self, cuda, synth, workload, device: int, like=None):
        page = workload.Page(seed=7)
        self.det = like.det.share_weights() if like else cuda.Model(synth.det_plan(seed=0), device=device)
        h, w = page.det.shape[:2]
        self.det.set_input_size(h, w)
        rec = like.rec.share_weights() if like else cuda.Model(synth.rec_plan(seed=1), device=device)
        self.rec = rec
        for m in (self.det, self.rec):  # several pages in flight
            m.set_options(cuda.OPT_THROUGHPUT)
        self.stream = self.det.stream
        rec.set_stream(self.stream)
        rec.set_sizes([(48, wd) for wd in page.widths])  # all lines of the page: one run
        np.copyto(self.det.input_mut(), page.det.reshape(-1))
        for lane in range(len(page.widths)):
            np.copyto(rec.lane_input_mut(lane), page.lines[lane].reshape(-1))
        self.det.run(60_000)
        rec.run(60_000)

    def enqueue(self):
        self.det.enqueue_device()
        self.rec.enqueue_device()

    def close(self):
        self.rec.close()
        self.det.close()


def device_time(torch, stream_ptr: int, fn, reps: int, flush) -> float:
    """Median seconds of fn() on a stream, CUDA events, L2 flushed before each."""
    stream = torch.cuda.ExternalStream(stream_ptr)
    times = []
    for i in range(reps + 3):
        with torch.cuda.stream(stream):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        fn()
        with torch.cuda.stream(stream):
            e1.record(stream)
        e1.synchronize()
        if i >= 3:
            times.append(e0.elapsed_time(e1) / 1e3)
    return statistics.median(times)


def configs_1_to_3(cuda, synth, torch, device: int, flush) -> dict:
    """Benchmark configs 1-3 on the device, inputs resident, L2 flushed: the
    fused depthwise 5x5 + pointwise 96->192 layer at 240 x 240, the detector
    at 960 x 736, the recogniser over 16 lines of 48 x 320."""
    rng = np.random.default_rng(0)
    out = {}
    with cuda.Model(synth.fused_layer_plan(seed=0)) as m:
        m.input_mut()[:] = rng.uniform(-1, 1, 240 * 240 * 96).astype(np.float32)
        m.run(60_000)
        t = device_time(torch, m.stream, m.enqueue_device, 20, flush)
        out["config1_fused_layer_us"] = t * 1e6
        out["config1_tflops"] = 2.400e9 / t / 1e12
        out["config1_steps"] = m.steps()
    with cuda.Model(synth.det_plan(seed=0)) as m:
        m.set_input_size(960, 736)
        m.input_mut()[:] = rng.standard_normal(960 * 736 * 3).astype(np.float32)
        m.run(60_000)
        out["config2_det_960x736_ms"] = device_time(torch, m.stream, m.enqueue_device, 20, flush) * 1e3
        m.set_input_size(1984, 1536)
        m.input_mut()[:] = rng.standard_normal(1984 * 1536 * 3).astype(np.float32)
        m.run(60_000)
        out["det_1984x1536_ms"] = device_time(torch, m.stream, m.enqueue_device, 10, flush) * 1e3
    with cuda.Model(synth.rec_plan(seed=1)) as m:
        m.set_sizes([(48, 320)] * 16)
        for lane in range(16):
            m.lane_input_mut(lane)[:] = rng.standard_normal(48 * 320 * 3).astype(np.float32)
        m.run(60_000)
        out["config3_rec_16x320_ms"] = device_time(torch, m.stream, m.enqueue_device, 20, flush) * 1e3
    return out


# The probed layers: the page's dominant kernel (conv_tc_kernel, the
# tensor-core implicit GEMM for stride-1 windowed convolutions) at its most
# common launch, the detector's 3x3 96 -> 24 RSE convolution at a quarter of
# a 1984 x 1536 page; the pointwise kernel (pw_tc_kernel) at its largest
# launch, the detector's first 1x1 24 -> 24 + swish at half the page; the
# depthwise kernel (dw_row_kernel) at its largest launch, the detector's
# first 3x3 depthwise layer over 24 channels + swish at half the page.
LAYERS = {
    "conv3x3": dict(h=496, w=384, ic=96, oc=24, k=3, fused="none",
                    kernel="conv_tc_kernel: 3x3 96->24 @ 496x384 (3xTF32 tcgen05, the RSE neck's convolution)"),
    "layer": dict(h=992, w=768, ic=24, oc=24, k=1, fused="swish",
                  kernel="pw_tc_kernel: 1x1 24->24 + swish @ 992x768 (3xTF32 tcgen05, the detector's first pointwise)"),
    "dw3x3": dict(h=992, w=768, ic=24, oc=24, k=3, fused="swish", kind="dwconv",
                  kernel="dw_row_kernel: depthwise 3x3 24 channels + swish @ 992x768 (FP32 FMA, the detector's first "
                         "depthwise)"),
}


def layer_plan(name: str) -> bytes:
    from ppocr_native_b200.plan import Op, encode, window

    L = LAYERS[name]
    kind = L.get("kind", "conv")
    rng = np.random.default_rng(0)
    wt = rng.normal(0, 0.02, L["k"] * L["k"] * (1 if kind == "dwconv" else L["ic"]) * L["oc"]).astype(np.float32)
    b = rng.normal(0, 0.02, L["oc"]).astype(np.float32)
    op = window(Op(kind, x=0, y=1, ic=L["ic"], oc=L["oc"], fused=L["fused"], w=(0, wt.size), b=(wt.size, L["oc"])),
                (L["k"], L["k"]), 1, L["k"] // 2, L["k"] // 2)
    return encode((0, L["h"], L["w"], L["ic"]), 2, [1], [op], np.concatenate([wt, b]))


def probe_kernel(cuda, torch, device: int, name: str, flush, reps: int = 20) -> dict:
    """One probed layer alone, CUDA events on the model's stream, L2 flushed
    before each launch. Algorithmic bytes: the input and output maps once,
    the weights (for the tensor cores: two tf32 halves, K padded to 32) and
    the bias; FLOPs: 2 per multiply-add."""
    L = LAYERS[name]
    h, w, ic, oc, k = L["h"], L["w"], L["ic"], L["oc"], L["k"]
    dw = L.get("kind") == "dwconv"
    m = cuda.Model(layer_plan(name), device=device)
    assert m.steps() == ["dwconv" if dw else "conv"], m.steps()
    m.input_mut()[:] = np.random.default_rng(0).standard_normal(h * w * ic).astype(np.float32)
    m.run(60_000)
    t = device_time(torch, m.stream, m.enqueue_device, reps, flush)
    m.close()
    if dw:
        return {"kernel": L["kernel"], "seconds": t, "flops": 2 * h * w * k * k * ic,
                "bytes": 4 * (h * w * ic + h * w * oc + k * k * ic + ic)}
    kk = k * k * ic
    kpad = -(-kk // 32) * 32
    return {"kernel": L["kernel"], "seconds": t, "flops": 2 * h * w * kk * oc,
            "bytes": 4 * (h * w * ic + h * w * oc + 2 * oc * kpad + oc)}


def roofline_entry(probe: dict, name: str, pk: dict, tensor: bool) -> dict:
    traffic, source = TRAFFIC[name]
    if tensor:
        tc_peak = pk["bf16"] / 2 / 3  # 3xTF32: tf32 at half the bf16 rate, three MMAs per product
        achieved = probe["flops"] / probe["seconds"] / 1e12
        return {"bound": "tensor", "kernel": probe["kernel"], "achieved": achieved, "peak": tc_peak,
                "unit": "TFLOP/s", "frac": achieved / tc_peak,
                "peak_source": pk["bf16_source"] + " / 2 (tf32) / 3 (3xTF32 products): FP32-equivalent",
                "traffic": traffic, "traffic_source": "ncu, one launch: " + source,
                "algorithmic_flops": probe["flops"], "algorithmic_bytes": probe["bytes"],
                "hbm_frac": probe["bytes"] / probe["seconds"] / 1e9 / pk["hbm"],
                "seconds_per_launch": probe["seconds"]}
    achieved = probe["bytes"] / probe["seconds"] / 1e9
    return {"bound": "hbm", "kernel": probe["kernel"], "achieved": achieved, "peak": pk["hbm"], "unit": "GB/s",
            "frac": achieved / pk["hbm"], "peak_source": pk["hbm_source"], "traffic": traffic,
            "traffic_source": "ncu, one launch: " + source, "algorithmic_bytes": probe["bytes"],
            "seconds_per_launch": probe["seconds"]}


# --------------------------------------------------------------- CPU side

_CPU_MODELS: dict = {}


def _cpu_models(o, synth, threads: int, page, quads) -> dict:
    """The CPU path's models, kept from one sample to the next as the
    reference worker keeps its engines: the detector, one recogniser per
    thread and the dictionary. The first call runs each once, untimed, at the
    sample's sizes (the page's detector input, the detector and the DB
    postprocess; every recogniser at the widest line), so no timed run pays
    for first-touch allocation."""
    m = _CPU_MODELS.get(threads)
    if m is None:
        o.build()
        o.set_fast(True)  # the register-tiled loops (the same bits as the plain ones)
        rec_plan = synth.rec_plan(seed=1)
        m = {"det": o.Oracle(synth.det_plan(seed=0)), "recs": [o.Oracle(rec_plan) for _ in range(threads)],
             "classes": o.dictionary(synth.characters(synth.VOCAB))}
        dw, dh = o.det_size(page.shape[1], page.shape[0])
        m["det"].set_size(dh, dw)
        x = o.det_input_hwc(page, dw, dh, o.MEAN, o.STD)
        o.boxes_from_prob(m["det"].run(x.reshape(-1), threads=threads)[0].reshape(dh, dw), page.shape[1],
                          page.shape[0])
        o.det_input_hwc(page, dw, dh, o.MEAN, o.STD)
        widest = max(o.rec_input_hwc(o.crop_text(page, q)).shape[1] for q in quads)
        for r in m["recs"]:
            r.set_size(48, widest)
            r.run(np.zeros(48 * widest * 3, np.float32), threads=1)
        _CPU_MODELS[threads] = m
    return m


def cpu_page_sample(page, quads, budget_s: float = 10.0, threads: int = 0) -> dict:
    """The reference CPU path (oracle, all host threads) over one page: the
    detector input, the detector at 1984 x 1536, the DB postprocess, then
    crops, recogniser inputs, recogniser and CTC decode of the page's lines
    until the budget is spent; seconds per page, lines scaled to all."""
    pkg = package()
    from oracle import oracle as o

    synth = pkg.synth
    threads = threads or cpu_threads()
    m = _cpu_models(o, synth, threads, page, quads)
    det, recs, classes = m["det"], m["recs"], m["classes"]
    t0 = time.perf_counter()
    dw, dh = o.det_size(page.shape[1], page.shape[0])
    x = o.det_input_hwc(page, dw, dh, o.MEAN, o.STD)
    det.set_size(dh, dw)
    prob = det.run(x.reshape(-1), threads=threads)[0].reshape(dh, dw)
    o.boxes_from_prob(prob, page.shape[1], page.shape[0])
    t_det = time.perf_counter() - t0
    from ppocr_native_b200.plan import flops

    det_plan, rec_plan = synth.det_plan(seed=0), synth.rec_plan(seed=1)
    macs = flops(det_plan, dh, dw) // 2
    # the lines as the reference worker reads them on the CPU
    # (ocr.rs:380-422 recognise_on_cpu): one recogniser per thread, lines
    # claimed in order, each line on one thread; lines until the budget
    left = max(budget_s - t_det, 0.0)
    claimed = itertools.count()
    lock = threading.Lock()
    work_macs = [0] * threads
    done_lines = [0] * threads
    t0 = time.perf_counter()

    def reader(k):
        r = recs[k]
        while True:
            with lock:
                i = next(claimed)
            if i >= len(quads) or time.perf_counter() - t0 > left:
                return
            crop = o.crop_text(page, quads[i])
            xin = o.rec_input_hwc(crop)
            r.set_size(48, xin.shape[1])
            out = r.run(xin.reshape(-1), threads=1)[0].reshape(-1, 2)
            o.ctc_decode(out[:, 0].astype(np.uint32), out[:, 1], classes)
            work_macs[k] += flops(rec_plan, 48, xin.shape[1]) // 2
            done_lines[k] += 1

    pool = [threading.Thread(target=reader, args=(k,)) for k in range(threads)]
    for th in pool:
        th.start()
    for th in pool:
        th.join()
    t_rec = time.perf_counter() - t0
    done = max(1, sum(done_lines))
    macs += sum(work_macs)
    page_s = t_det + t_rec * len(quads) / done
    gmacs_core = macs / (t_det + t_rec) / threads / 1e9
    return {"seconds": page_s, "t_det": t_det, "t_rec": t_rec, "lines": done, "of": len(quads), "threads": threads,
            "gmacs_per_core": gmacs_core}


def cpu_tile_rate(reps: int = 20) -> float:
    """The CPU path's pointwise tile alone on one core, as the reference
    quotes its own (README: six pixels by sixteen channels, about 58 GMAC/s
    on one Zen 3 core): a 1x1 384->384 layer with bias over 32 x 32 pixels
    (1.5 MB in, 1.5 MB out, weights 0.6 MB: cache resident), one thread,
    the best of `reps` runs; GMAC/s."""
    package()
    from oracle import oracle as o
    from ppocr_native_b200.plan import Op, encode, window

    o.build()
    o.set_fast(True)
    h = w = 32
    c = 384
    rng = np.random.default_rng(0)
    wt = rng.normal(0, 0.02, c * c + c).astype(np.float32)
    op = window(Op("conv", x=0, y=1, ic=c, oc=c, w=(0, c * c), b=(c * c, c)), (1, 1), 1, 0, 0)
    m = o.Oracle(encode((0, h, w, c), 2, [1], [op], wt))
    x = rng.standard_normal(h * w * c).astype(np.float32)
    best = float("inf")
    for k in range(reps + 3):
        t0 = time.perf_counter()
        m.run(x, threads=1)
        if k >= 3:
            best = min(best, time.perf_counter() - t0)
    return h * w * c * c / best / 1e9


def cpu_sample_text(s: dict, tile: float) -> str:
    """What one CPU page sample was, for `cpu_baseline.sample`."""
    return (f"1 page: detector input + detector 1984x1536 + DB boxes ({s['t_det']:.2f} s), "
            f"{s['lines']} of {s['of']} lines cropped, recognised and decoded ({s['t_rec']:.2f} s, "
            "scaled to all); C restatement of the reference CPU engine and page steps (tier-3 FMA "
            "order; dense convolutions in register-tiled AVX2+FMA tiles of 4 pixels x 24 columns, "
            "the CTC head panel by panel over all time steps as the reference's, activations, "
            "softmax, attention and transposed convolutions vectorised, channel means summed by "
            "the layer that writes their input, input resizes through the reference's byte tables), "
            f"OpenMP over output rows; {s['gmacs_per_core']:.2f} GMAC/s per core over the whole page "
            "(every step's time, the networks' multiply-adds); its pointwise tile alone on one core: "
            f"{tile:.1f} GMAC/s, against about 58 for the reference's on one Zen 3 core (its README)")


def cpu_baseline(page, quads, budget_s: float = 15.0) -> dict:
    s = cpu_page_sample(page, quads, budget_s)
    tile = cpu_tile_rate()
    return {"value": 1.0 / s["seconds"], "unit": "pages/s", "cores": s["threads"], "kind": "port",
            "sample": cpu_sample_text(s, tile), "gmacs_per_core": s["gmacs_per_core"],
            "tile_gmacs_one_core": tile}


# ------------------------------------------------------------------ ours

def run_layer(args, d, cuda, device):
    """--workload layer | conv3x3 | dw3x3: the probed layer alone, warm-up then
    timed steps (the command ncu captures)."""
    L = LAYERS[args.workload]
    m = cuda.Model(layer_plan(args.workload), device=device)
    m.input_mut()[:] = np.random.default_rng(0).standard_normal(L["h"] * L["w"] * L["ic"]).astype(np.float32)
    m.run(60_000)
    for _ in range(args.warmup + args.steps):
        m.enqueue_device()
    m.wait(60_000)
    m.close()
    return {"profile": args.workload, "launches_per_step": 1} if d.rank == 0 else None


def run_neural(args, d, cuda, synth, workload, torch, device):
    """--workload neural|det|rec: the neural hot path alone, device-resident,
    k page pipelines in flight (the commands the launch lists come from)."""
    k = 1 if args.profile else max(1, args.readers)
    pipes = [NeuralPipeline(cuda, synth, workload, device)]
    pipes += [NeuralPipeline(cuda, synth, workload, device, like=pipes[0]) for _ in range(k - 1)]
    main = torch.cuda.Stream(device=device)
    streams = [torch.cuda.ExternalStream(p.stream) for p in pipes]
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=f"cuda:{device}")

    def one(p):
        if args.workload in ("neural", "det"):
            p.det.enqueue_device()
        if args.workload in ("neural", "rec"):
            p.rec.enqueue_device()

    for _ in range(args.warmup):
        for p in pipes:
            one(p)
    torch.cuda.synchronize()
    d.barrier()
    events = []
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(main):
            flush.zero_()
            e0.record(main)
        for p, st in zip(pipes, streams):
            st.wait_event(e0)
            one(p)
            done = torch.cuda.Event()
            done.record(st)
            main.wait_event(done)
        e1.record(main)
        events.append((e0, e1))
    torch.cuda.synchronize()
    local = sum(a.elapsed_time(b) for a, b in events) / 1e3
    value, total = d.whole_job(args.steps * k, local)
    launches = pipes[0].det.launches + pipes[0].rec.launches
    for p in reversed(pipes):
        p.close()
    if d.rank == 0:
        return {"profile": args.workload, "pages_per_s": value, "ms_per_step": total / args.steps * 1e3,
                "launches_per_page": launches}
    return None


def run_ours(args, d: Dist) -> dict | None:
    import torch

    pkg = package()
    cuda, synth, workload = pkg.cuda, pkg.synth, pkg.workload
    device = d.local
    torch.cuda.set_device(device)
    d.init("nccl")
    if args.workload in LAYERS:
        return run_layer(args, d, cuda, device)
    if args.workload in ("neural", "det", "rec"):
        return run_neural(args, d, cuda, synth, workload, torch, device)

    R = max(1, args.readers)
    # The pages: config 4 (44 lines each) or config 5's stream (20-60 lines),
    # a pool of distinct seeded pages per rank read in turn.
    if args.workload == "stream":
        stream = workload.page_stream(seed=5, pages=args.stream_pages)
        mine = stream[d.rank::d.world]
        total = len(mine)
        distinct = mine[:args.pool]
    else:
        total = args.steps * R
        distinct = [(1000 * d.rank + i, workload.LINES_PER_PAGE) for i in range(args.pool)]
    pages = make_pages(distinct, threads=min(16, cpu_threads()))
    pool = PagePool(torch, device, pages)
    text = synth.characters(synth.VOCAB)
    det = cuda.Model(synth.det_plan(seed=0), device=device)
    rec = cuda.Model(synth.rec_plan(seed=1), device=device)
    readers = [cuda.Reader(det, rec, text) for _ in range(R)]
    main = torch.cuda.Stream(device=device)

    # Warm-up: every reader reads every distinct page once (its buffers grow
    # to the largest page: no allocation, which would synchronize the
    # device, inside the timed passes), then the warm-up steps.
    def warm(r):
        for k in range(len(pool)):
            r.detect_ptr(pool.host[k].data_ptr(), pool.w, pool.h)
            q = pool.quads[k]
            r.recognise_ptr(q.ctypes.data, len(q))

    with cf.ThreadPoolExecutor(max_workers=R) as ex:
        list(ex.map(warm, readers))
    read_pages(torch, readers, pool, max(args.warmup, 1) * R, False, main)
    torch.cuda.synchronize()

    # value: the pages already in HBM.
    d.barrier()
    torch.cuda.synchronize()
    before = [r.host_times() for r in readers]
    with Clocks(device) as clocks:
        dev_s, dev_wall, dev_cpu, dev_lat, launches = read_pages(torch, readers, pool, total, True, main)
    after = [r.host_times() for r in readers]
    host_ms = {k: sum(a[k] - b[k] for a, b in zip(after, before)) / total * 1e3 for k in after[0]}
    d.barrier()
    # e2e: the pages in page-locked host memory, copied in by the reader.
    torch.cuda.synchronize()
    e2e_s, e2e_wall, e2e_cpu, e2e_lat, _ = read_pages(torch, readers, pool, total, False, main)
    d.barrier()
    boxes_found = readers[0].boxes().shape[0]
    scored, rescored = readers[0].stats()
    for r in readers:
        r.close()
    value, value_t = d.whole_job(total, dev_s)
    e2e, e2e_t = d.whole_job(total, e2e_s)
    page_bytes = pool.h * pool.w * 3
    # per rank: pages/s, median and max page latency, host CPU use (of all host threads)
    host_keys = list(host_ms)
    per_rank = d.gather([total / dev_s, statistics.median(dev_lat), max(dev_lat),
                         dev_cpu / dev_wall / cpu_threads(), total / e2e_s, statistics.median(e2e_lat), max(e2e_lat),
                         e2e_cpu / e2e_wall / cpu_threads(), dev_cpu / total * 1e3] + [host_ms[k] for k in host_keys])
    extra = {}
    if d.rank == 0 and not args.quick:
        flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=f"cuda:{device}")
        # the neural hot path alone (device-resident page tensors, R pages in flight)
        nargs = argparse.Namespace(**vars(args))
        nargs.workload, nargs.steps, nargs.warmup, nargs.profile = "neural", 20, 3, False
        extra["neural"] = run_neural(nargs, Dist(), cuda, synth, workload, torch, device)
        extra.update(configs_1_to_3(cuda, synth, torch, device, flush))
        pk = peaks()
        extra["probes"] = {n: probe_kernel(cuda, torch, device, n, flush) for n in LAYERS}
        extra["peaks"] = pk
    det.close()
    rec.close()
    if d.rank != 0:
        return None
    # bytes per page through the C ABI: in, the page and its quads; out, the
    # mask and the reads (2 floats per time step of every line; the box
    # scores are a few bytes)
    def steps_of(q):
        w = cuda.rec_input_width(int(np.rint(q[2] - q[0])), int(np.rint(q[5] - q[1])))
        return -(-w // 8)

    steps_per_page = float(np.mean([sum(steps_of(q) for q in pool.quads[k]) for k in range(len(pool))]))
    h2d = page_bytes + 32 * float(np.mean([len(q) for q in pool.quads]))
    d2h = 1984 * 1536 + 8 * steps_per_page
    result = {
        "metric": METRIC,
        "value": value,
        "unit": "pages/s",
        "n_gpus": d.world,
        "steps": args.steps if args.workload == "page" else total,
        "warmup": args.warmup,
        "ms_per_step": value_t / (total / R) * 1e3,
        "higher_is_better": True,
        "scaling": "strong" if args.workload == "stream" else "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic: seeded 2550x3300 pages (white, rows of dark glyph-like rectangles 20-40 px tall with "
                "1-3 px gaps, gray noise sigma 4); random-init weights N(0,0.02) of the PP-OCRv6-shaped det/rec plans",
        "config": {
            "workload": ("config 5: 800-page stream, 20-60 lines per page, sharded by page" if args.workload == "stream"
                         else "config 4: 2550x3300 page -> resize+normalize -> det 1984x1536 -> DB postprocess -> "
                              "crops of the page's 44 line quads -> rec inputs -> rec (all lines, one run) -> "
                              "CTC decode (18 710 classes)"),
            "boxes": f"DB postprocess of the random-init detector's map: {boxes_found} box(es) (a near-constant 0.5 "
                     "map); the generator's line quads are recognised",
            "pages_per_step": R,
            "readers": f"{R} readers per GPU, one host thread and one stream each, weights shared",
            "distinct_pages": len(pool),
            "l2": "inputs larger than L2: each page is 25 MB and the detector's tensors ~1.5 GB per page",
            "parallelism": f"replicas x{d.world} (pages sharded by rank, no collective)",
            "box_scores": {"gpu_scored": scored, "host_rescored": rescored},
            **extra,
        },
        "e2e": {"value": e2e, "unit": "pages/s", "h2d_bytes_per_step": int(h2d * R),
                "d2h_bytes_per_step": int(d2h * R),
                "method": "C ABI ppocr_reader_detect + ppocr_reader_recognise + texts read, page bytes in "
                          "page-locked host memory; per page: page H2D, kernels, mask/scores/reads D2H, host "
                          f"page steps; {R} readers in flight; CUDA events around all readers' streams"},
        "gpu_launches": int(launches * total),
        "per_rank": [{"rank": i, "pages_per_s": v[0], "page_ms_median": v[1] * 1e3, "page_ms_max": v[2] * 1e3,
                      "host_cpu_busy": v[3], "e2e_pages_per_s": v[4], "e2e_page_ms_median": v[5] * 1e3,
                      "e2e_page_ms_max": v[6] * 1e3, "e2e_host_cpu_busy": v[7], "host_cpu_ms_per_page": v[8],
                      "reader_host_ms_per_page": dict(zip(host_keys, v[9:])),
                      "host_cores": cpu_threads()} for i, v in enumerate(per_rank)],
        "clocks": clocks.summary(),
    }
    if extra.get("probes"):
        pr, pk = extra.pop("probes"), extra["peaks"]
        result["config"].pop("probes", None)
        result["roofline"] = roofline_entry(pr["conv3x3"], "conv3x3", pk, True)
        result["roofline_pointwise"] = roofline_entry(pr["layer"], "layer", pk, False)
        result["roofline_depthwise"] = roofline_entry(pr["dw3x3"], "dw3x3", pk, False)
    return result


# ------------------------------------------------------------- reference

def run_reference(args, d: Dist) -> dict | None:
    """The reference CPU path on this host, rank 0 only: each timed step one
    bounded sample (a page's detector and DB postprocess, and its lines
    until a budget, scaled); at most three timed samples so the run ends in
    minutes whatever --steps asks."""
    if d.rank != 0:
        return None
    pkg = package()
    page, quads = pkg.workload.synthetic_page(1000)
    samples, base = [], None
    n = min(max(args.steps, 1), 3)
    for step in range(min(args.warmup, 1) + n):
        s = cpu_page_sample(page, quads, budget_s=args.ref_budget)
        if step >= min(args.warmup, 1):
            samples.append(1.0 / s["seconds"])
            base = s
    value = statistics.median(samples)
    tile = cpu_tile_rate()
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": value, "unit": "pages/s", "n_gpus": d.world, "steps": n, "warmup": min(args.warmup, 1),
        "ms_per_step": 1e3 / value, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (the same page generator and weights as the GPU arm)",
        "config": {"workload": "config 4: 2550x3300 page -> det 1984x1536 -> DB boxes -> crops of the 44 line quads "
                               "-> rec -> CTC decode, on the host cores"},
        "cpu_baseline": {"value": value, "unit": "pages/s", "cores": base["threads"], "kind": "port",
                         "sample": "per step " + cpu_sample_text(base, tile), "gmacs_per_core": base["gmacs_per_core"],
                         "tile_gmacs_one_core": tile},
        "e2e": {"value": value, "unit": "pages/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    faulthandler.enable()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50, help="steps of `--readers` pages each")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--readers", type=int, default=8, help="readers (pages in flight) per GPU")
    ap.add_argument("--pool", type=int, default=16, help="distinct pages per rank")
    ap.add_argument("--stream-pages", type=int, default=800)
    ap.add_argument("--ref-budget", type=float, default=10.0, help="seconds of CPU work per reference sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--quick", action="store_true", help="the page run alone (no neural, config 1-3 or probe legs)")
    ap.add_argument("--workload", choices=["page", "stream", "neural", "det", "rec", *LAYERS], default="page")
    ap.add_argument("--profile", action="store_true",
                    help="only warm-up and timed steps (no e2e, probe, peak or CPU legs): for ncu launch lists")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    d = Dist()
    if args.impl == "reference":
        result = run_reference(args, d)
    else:
        result = run_ours(args, d)
        if result is not None and not args.profile and args.workload in ("page", "stream"):
            if args.no_cpu_baseline or args.quick:
                result["cpu_baseline"] = None
            else:
                page, quads = package().workload.synthetic_page(1000)
                result["cpu_baseline"] = cpu_baseline(page, quads)
    d.close()
    if result is not None:
        print(json.dumps(result))


if __name__ == "__main__":
    main()
