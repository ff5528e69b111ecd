"""Benchmark: synthetic 300-dpi pages through the PP-OCRv6 detector and
recogniser on B200, one process per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload page|det|rec|layer]

A step is one page's neural hot path: the detector at 1984 x 1536 and the
recogniser over the page's 44 lines (runs of up to 16 lanes, each line at
its own width). `value` is pages/s over all ranks with every input already
in HBM; `e2e` the same through the public C ABI from page-locked host
buffers, copies in and out included. With N > 1 each rank reads its own
pages (weak scaling); ranks exchange nothing but the timing.

`--impl reference` times the reference CPU path on this host: the C
restatement of ppocr-native's CPU engine (oracle/, the reference itself is
Rust and cannot be built here), all host threads, bounded samples.
"""

from __future__ import annotations

import argparse
import faulthandler
import importlib.util
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
# DRAM bytes (read + written) of one launch of the pointwise probe, from one
# ncu capture of `bench.py --workload layer`
# (profiles/pw_tc_kernel_1x1_24to24_992x768.md); writes still dirty in L2 when
# the kernel ends are not counted there.
TRAFFIC_PER_LAUNCH = 99.67e6
TRAFFIC_SOURCE = "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch (profiles/pw_tc_kernel_1x1_24to24_992x768.md)"
# The same for the dominant kernel's probe (`bench.py --workload conv3x3`).
CONV_TRAFFIC_PER_LAUNCH = 78.19e6
# The same for the depthwise probe (`bench.py --workload dw3x3`).
DW_TRAFFIC_PER_LAUNCH = 107.59e6
DW_TRAFFIC_SOURCE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch "
                     "(profiles/dw_row_kernel_3x3_c24_992x768.md)")
CONV_TRAFFIC_SOURCE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch "
                       "(profiles/conv_tc_kernel_3x3_96to24_496x384.md)")


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

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()

    def whole_job(self, units_per_rank: float, local_seconds: float) -> tuple[float, float]:
        """Units of all ranks per second over the slowest rank's time (every
        rank processes the same number of its own pages: weak scaling), and
        that time."""
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


# -------------------------------------------------------------- our path

class PagePipeline:
    """The detector and the recogniser runs of one page, queued on one stream."""

    def __init__(self, cuda, synth, page, device: int, workload: str = "page", like=None):
        """`like`: another pipeline whose weights this one shares (its own
        models, stream and buffers)."""
        self.det = like.det.share_weights() if like else cuda.Model(synth.det_plan(seed=0), device=device)
        h, w = page.det.shape[:2]
        self.det.set_input_size(h, w)
        rec = like.recs[0].share_weights() if like else cuda.Model(synth.rec_plan(seed=1), device=device)
        self.recs = [rec] + [rec.share_weights() for _ in page.runs[1:]]
        self.stream = self.det.stream
        for m, run in zip(self.recs, page.runs):
            m.set_stream(self.stream)
            m.set_sizes([(48, page.widths[i]) for i in run])
        self.page = page
        self.workload = workload

    def models(self):
        if self.workload == "det":
            return [self.det]
        if self.workload == "rec":
            return list(self.recs)
        return [self.det, *self.recs]

    def all_models(self):
        return [self.det, *self.recs]

    def fill_host(self):
        """Copy the page into the page-locked lane inputs."""
        np.copyto(self.det.input_mut(), self.page.det.reshape(-1))
        for m, run in zip(self.recs, self.page.runs):
            for lane, i in enumerate(run):
                np.copyto(m.lane_input_mut(lane), self.page.lines[i].reshape(-1))

    def enqueue_host(self):
        """The public call sequence, first half: every run queues the copy of
        its page-locked inputs in, its kernels and the copy of its outputs
        out."""
        for m in self.models():
            m.enqueue()

    def wait_host(self):
        """Second half: wait for the runs; the host reads each result."""
        for m in self.models():
            m.wait(0)
        outs = [self.det.output()]
        for m, run in zip(self.recs, self.page.runs):
            for lane in range(len(run)):
                outs.append(m.lane_output(lane))
        return outs

    def run_host(self):
        self.enqueue_host()
        return self.wait_host()

    def enqueue_device(self):
        for m in self.models():
            m.enqueue_device()

    def launches(self) -> int:
        return sum(m.launches for m in self.models())

    def io_bytes(self):
        h2d = self.page.input_bytes()
        d2h = self.det.output().nbytes
        for m, run in zip(self.recs, self.page.runs):
            d2h += sum(m.lane_output(lane).nbytes for lane in range(len(run)))
        return h2d, d2h

    def close(self):
        # the recogniser models run on the detector's stream: they go first
        for m in reversed(self.all_models()):
            m.close()


# The probed layers: the page's dominant kernel (conv_tc_kernel, the
# tensor-core implicit GEMM for stride-1 windowed convolutions, the largest
# share of a page's launch time) at its most common launch, the detector's
# 3x3 96 -> 24 RSE convolution at a quarter of a 1984 x 1536 page; and the
# pointwise kernel (pw_tc_kernel) at its largest launch, the detector's first
# 1x1 24 -> 24 + swish at half the page; and the depthwise kernel
# (dw_row_kernel) at its largest launch, the detector's first 3x3 depthwise
# layer over 24 channels + swish at half the page.
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


def run_layer(args, d, cuda, torch, device):
    """--workload layer | conv3x3 | dw3x3: the probed layer alone, warm-up then timed
    steps (the command ncu captures)."""
    L = LAYERS[args.workload]
    m = cuda.Model(layer_plan(args.workload), device=device)
    m.input_mut()[:] = np.random.default_rng(0).standard_normal(L["h"] * L["w"] * L["ic"]).astype(np.float32)
    m.run(60_000)
    for _ in range(args.warmup + args.steps):
        m.enqueue_device()
    m.wait(60_000)
    m.close()
    return {"profile": args.workload, "launches_per_step": 1} if d.rank == 0 else None


def probe_kernel(cuda, torch, device: int, name: str, reps: int = 20) -> dict:
    """Time one probed layer alone with CUDA events on the model's stream, L2
    flushed before each launch. Algorithmic bytes: the input and output maps
    once, the weights (for the tensor cores: two tf32 halves, K padded to 32)
    and the bias; FLOPs: 2 per multiply-add of the convolution."""
    L = LAYERS[name]
    h, w, ic, oc, k = L["h"], L["w"], L["ic"], L["oc"], L["k"]
    dw = L.get("kind") == "dwconv"
    rng = np.random.default_rng(0)
    m = cuda.Model(layer_plan(name), device=device)
    assert m.steps() == ["dwconv" if dw else "conv"], m.steps()
    m.input_mut()[:] = rng.standard_normal(h * w * ic).astype(np.float32)
    m.run(60_000)
    stream = torch.cuda.ExternalStream(m.stream)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=f"cuda:{device}")
    times = []
    for i in range(reps + 3):
        with torch.cuda.stream(stream):
            flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        m.enqueue_device()
        with torch.cuda.stream(stream):
            e1.record(stream)
        e1.synchronize()
        if i >= 3:
            times.append(e0.elapsed_time(e1) / 1e3)
    m.close()
    t = statistics.median(times)
    if dw:
        return {"kernel": L["kernel"], "seconds": t, "flops": 2 * h * w * k * k * ic,
                "bytes": 4 * (h * w * ic + h * w * oc + k * k * ic + ic)}
    kk = k * k * ic
    kpad = -(-kk // 32) * 32
    return {"kernel": L["kernel"], "seconds": t, "flops": 2 * h * w * kk * oc,
            "bytes": 4 * (h * w * ic + h * w * oc + 2 * oc * kpad + oc)}


def cpu_baseline(widths_seed: int = 0, budget_s: float = 20.0) -> dict:
    """The reference CPU path (C restatement, all host threads) on a bounded
    sample: one page's detector and as many of its lines as fit the budget,
    scaled to pages/s."""
    pkg = package()
    from oracle.oracle import Oracle, build

    build()
    synth, workload = pkg.synth, pkg.workload
    page = workload.Page(widths_seed)
    threads = cpu_threads()
    det = Oracle(synth.det_plan(seed=0))
    det.set_size(*page.det.shape[:2])
    t0 = time.perf_counter()
    det.run(page.det.reshape(-1), threads=threads)
    t_det = time.perf_counter() - t0
    rec = Oracle(synth.rec_plan(seed=1))
    t_rec, done = 0.0, 0
    for i, wd in enumerate(page.widths):
        rec.set_size(48, wd)
        t0 = time.perf_counter()
        rec.run(page.lines[i].reshape(-1), threads=threads)
        t_rec += time.perf_counter() - t0
        done += 1
        if t_det + t_rec > budget_s:
            break
    page_s = t_det + t_rec * len(page.widths) / done
    return {"value": 1.0 / page_s, "unit": "pages/s", "cores": threads, "kind": "port",
            "sample": f"1 page: detector 1984x1536 ({t_det:.2f} s) + {done} of {len(page.widths)} lines "
                      f"({t_rec:.2f} s, scaled to all); C restatement of the reference CPU engine "
                      "(tier-3 FMA order), OpenMP over output rows"}


def run_ours(args, d: Dist) -> dict | None:
    import torch

    pkg = package()
    cuda, synth, workload = pkg.cuda, pkg.synth, pkg.workload
    device = d.local
    torch.cuda.set_device(device)
    d.init("nccl")
    if args.workload in LAYERS:
        return run_layer(args, d, cuda, torch, device)
    page = workload.Page(seed=1000 + d.rank)
    pipe = PagePipeline(cuda, synth, page, device, args.workload)
    # Pages in flight: one pipeline each (own models, streams and buffers,
    # shared weights); launch lists (--profile) take one.
    k = 1 if args.profile else max(1, args.inflight)
    pipes = [pipe] + [PagePipeline(cuda, synth, page, device, args.workload, like=pipe) for _ in range(k - 1)]
    streams = [torch.cuda.ExternalStream(p.stream) for p in pipes]
    main = torch.cuda.Stream(device=device)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=f"cuda:{device}")

    # Inputs into HBM once through the public path (copies included).
    for p in pipes:
        p.fill_host()
        p.run_host()
        for _ in range(args.warmup):
            p.enqueue_device()
    torch.cuda.synchronize()

    # value: device-resident inputs; a step is k pages enqueued at once, each
    # on its own stream, L2 flushed before each step outside its events.
    events = []
    d.barrier()
    torch.cuda.synchronize()
    with Clocks(device) as clocks:
        for _ in range(args.steps):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(main):
                flush.zero_()
                e0.record(main)
            for p, st in zip(pipes, streams):
                st.wait_event(e0)
                p.enqueue_device()
                done = torch.cuda.Event()
                done.record(st)
                main.wait_event(done)
            e1.record(main)
            events.append((e0, e1))
        torch.cuda.synchronize()
    d.barrier()
    local_s = sum(a.elapsed_time(b) for a, b in events) / 1e3
    value, total_s = d.whole_job(args.steps * k, local_s)
    if args.profile:
        launches = pipe.launches()
        pipe.close()
        if d.rank == 0:
            return {"profile": args.workload, "ms_per_step": total_s / args.steps * 1e3,
                    "launches_per_step": launches}
        return None

    # e2e: the public call sequence with host buffers. The page sits in the
    # models' page-locked lane inputs (where a caller's preprocessing writes
    # it); every step copies its inputs in, runs, copies its outputs out and
    # the host reads the result. The k pipelines take the pages in turn, so
    # one page's copies and latency-bound kernels overlap the others', as
    # enqueue/wait allow any caller.
    d.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for step in range(args.steps):
        p = pipes[step % k]
        if step >= k:
            outs = p.wait_host()
            _ = float(outs[0][0])
        p.enqueue_host()
    for step in range(max(0, args.steps - k), args.steps):
        outs = pipes[step % k].wait_host()
        _ = float(outs[0][0])
    torch.cuda.synchronize()
    e2e_local = time.perf_counter() - t0
    e2e, _ = d.whole_job(args.steps, e2e_local)
    h2d, d2h = pipe.io_bytes()
    launches = pipe.launches()

    # det alone (ms), for the metric's "det fwd ms"
    stream = streams[0]
    det_times = []
    for _ in range(5):
        with torch.cuda.stream(stream):
            flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        pipe.det.enqueue_device()
        with torch.cuda.stream(stream):
            e1.record(stream)
        e1.synchronize()
        det_times.append(e0.elapsed_time(e1))
    for p in reversed(pipes):
        p.close()
    d.barrier()

    result = None
    if d.rank == 0:
        probe = probe_kernel(cuda, torch, device, "conv3x3")
        pw = probe_kernel(cuda, torch, device, "layer")
        dwp = probe_kernel(cuda, torch, device, "dw3x3")
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
        hbm, bf16 = peaks.get("hbm_gbs"), peaks.get("bf16_tflops")
        hbm_source = "measured: MEASURED_PEAKS.json hbm_gbs (copy, burst)"
        bf16_source = "measured: MEASURED_PEAKS.json bf16_tflops (cuBLAS, burst)"
        if hbm is None:
            hbm, hbm_source = 6650.0, "fallback: 6.65 TB/s"
        if bf16 is None:
            bf16, bf16_source = 1590.0, "fallback: 1.59 PFLOP/s"
        # 3xTF32: the tf32 rate is half the bf16 one, three MMAs per product
        tc_peak = bf16 / 2 / 3
        result = {
            "metric": "synthetic-page pages/s (det 1984x1536 + rec 44 lines) per B200 job",
            "value": value,
            "unit": "pages/s",
            "n_gpus": d.world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": total_s / args.steps * 1e3,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic: seeded N(0,1) page tensors with the reference's page/line shapes; "
                    "random-init weights N(0,0.02) of the synthetic PP-OCRv6-shaped det/rec plans",
            "config": {"workload": "page: det 1984x1536 + rec 44 lines (48 x 320..1600, runs of 16)",
                       "det_fwd_ms": statistics.median(det_times),
                       "pages_per_step": k,
                       "l2": "flushed (256 MB write) before every timed step, outside the step's events",
                       "parallelism": f"replicas x{d.world} (pages sharded by rank, no collective)"},
            "e2e": {"value": e2e, "unit": "pages/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "method": "C ABI enqueue/wait, inputs in the models' page-locked buffers, per step: H2D, "
                              f"kernels, D2H, host read; one page per step, {k} pages in flight on their own "
                              "streams"},
            "gpu_launches": launches * args.steps * k,
            "roofline": {"bound": "tensor", "kernel": probe["kernel"],
                         "achieved": probe["flops"] / probe["seconds"] / 1e12, "peak": tc_peak, "unit": "TFLOP/s",
                         "frac": probe["flops"] / probe["seconds"] / 1e12 / tc_peak,
                         "peak_source": bf16_source + " / 2 (tf32) / 3 (3xTF32 products): FP32-equivalent",
                         "traffic": CONV_TRAFFIC_PER_LAUNCH, "traffic_source": CONV_TRAFFIC_SOURCE,
                         "algorithmic_flops": probe["flops"], "algorithmic_bytes": probe["bytes"],
                         "hbm_frac": probe["bytes"] / probe["seconds"] / 1e9 / hbm,
                         "seconds_per_launch": probe["seconds"]},
            "roofline_pointwise": {"bound": "hbm", "kernel": pw["kernel"],
                                   "achieved": pw["bytes"] / pw["seconds"] / 1e9, "peak": hbm, "unit": "GB/s",
                                   "frac": pw["bytes"] / pw["seconds"] / 1e9 / hbm, "peak_source": hbm_source,
                                   "traffic": TRAFFIC_PER_LAUNCH, "traffic_source": TRAFFIC_SOURCE,
                                   "algorithmic_bytes": pw["bytes"], "seconds_per_launch": pw["seconds"]},
            "roofline_depthwise": {"bound": "hbm", "kernel": dwp["kernel"],
                                   "achieved": dwp["bytes"] / dwp["seconds"] / 1e9, "peak": hbm, "unit": "GB/s",
                                   "frac": dwp["bytes"] / dwp["seconds"] / 1e9 / hbm, "peak_source": hbm_source,
                                   "traffic": DW_TRAFFIC_PER_LAUNCH, "traffic_source": DW_TRAFFIC_SOURCE,
                                   "algorithmic_bytes": dwp["bytes"],
                                   "seconds_per_launch": dwp["seconds"]},
            "clocks": clocks.summary(),
        }
    return result


def run_reference(args, d: Dist) -> dict | None:
    if d.rank != 0:
        return None
    samples = []
    base = None
    for step in range(args.warmup + args.steps):
        b = cpu_baseline(widths_seed=step, budget_s=8.0)
        if step >= args.warmup:
            samples.append(b["value"])
            base = b
    value = statistics.median(samples)
    return {
        "impl": "reference",
        "metric": "synthetic-page pages/s (det 1984x1536 + rec 44 lines) per B200 job",
        "value": value, "unit": "pages/s", "n_gpus": d.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 / value, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (same pages and weights as the GPU arm)",
        "config": {"workload": "page: det 1984x1536 + rec 44 lines (48 x 320..1600, runs of 16)"},
        "cpu_baseline": {"value": value, "unit": "pages/s", "cores": base["cores"], "kind": "port",
                         "sample": base["sample"]},
        "e2e": {"value": value, "unit": "pages/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    faulthandler.enable()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--inflight", type=int, default=8,
                    help="pages in flight (own models and streams, shared weights): a step's pages")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["page", "det", "rec", *LAYERS], default="page",
                    help="page (the benchmark step); det or rec alone, for profiling")
    ap.add_argument("--profile", action="store_true",
                    help="only warm-up and timed steps (no e2e, probe, peak or CPU legs): for ncu launch lists")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    d = Dist()
    if args.impl == "reference":
        result = run_reference(args, d)
    else:
        result = run_ours(args, d)
        if result is not None and not args.profile and args.workload == "page":
            if args.no_cpu_baseline:
                result["cpu_baseline"] = None
            else:
                result["cpu_baseline"] = cpu_baseline()
    d.close()
    if result is not None:
        print(json.dumps(result))


if __name__ == "__main__":
    main()
