"""Parity of the CUDA path (through the C ABI) with the CPU oracle.

The kernels accumulate every convolution output in the oracle's order (bias
first or last as the reference's tiles do, taps and channels in order, one
fused multiply-add each) and evaluate the activations with the same IEEE
operations, so most outputs are expected to be bit-identical; the bar
`north_star` sets is 1e-4 absolute on probabilities and recogniser values
and identical CTC classes. Each test asserts the bar and, where the kernel
is built to be exact, exact equality too.
"""

from __future__ import annotations

import ctypes
import glob
import os

import numpy as np
import pytest

from common import Op, encode, max_gap, noise, single, window
from ppocr_native_b200 import synth

pytestmark = pytest.mark.gpu

TOL = 1e-4  # north_star: probabilities and recogniser values within 1e-4


def gpu_run(cuda, plan, x, hw=None, options=0):
    with cuda.Model(plan) as m:
        if options:
            m.set_options(options)
        if hw is not None:
            m.set_input_size(*hw)
        m.input_mut()[:] = x
        m.run(60_000)
        return [m.output(k).copy() for k in range(m.output_count())], m.steps()


def oracle_run(oracle_mod, plan, x, hw=None):
    o = oracle_mod.Oracle(plan)
    if hw is not None:
        o.set_size(*hw)
    return o.run(x)


def check(got, want, exact=True, tol=TOL):
    assert got.shape == want.shape
    gap = max_gap(got, want)
    assert gap <= tol, gap
    if exact:
        assert np.array_equal(got, want), f"max gap {gap}, {int(np.sum(got != want))} of {got.size} differ"


def check_both(cuda, oracle_mod, plan, x, hw=None, tol=TOL, scale=1.0):
    """The product path (pointwise layers on the tensor cores, 3xTF32)
    within `tol` (times the output's scale), and the FP32-only path
    bit-identical to the oracle."""
    want = oracle_run(oracle_mod, plan, x, hw)[0]
    got, steps = gpu_run(cuda, plan, x, hw)
    check(got[0], want, exact=False, tol=tol * max(1.0, scale * float(np.abs(want).max())))
    exact, _ = gpu_run(cuda, plan, x, hw, options=cuda.OPT_NO_TENSOR_CORES)
    check(exact[0], want)
    return steps


# ---------------------------------------------------------------- one op each

CONV_CASES = [
    # k, s, pads (t,b,l,r), ic, oc, fused
    (3, 2, (1, 1, 1, 1), 3, 24, "swish"),   # det stem
    (3, 2, (1, 1, 1, 1), 3, 48, "swish"),   # rec stem
    (3, 1, (1, 1, 1, 1), 96, 24, "none"),   # RSE 3x3
    (1, 1, (0, 0, 0, 0), 96, 192, "swish"),
    (1, 1, (0, 0, 0, 0), 192, 384, "relu"),
    (1, 1, (0, 0, 0, 0), 384, 96, "none"),
    (1, 1, (0, 0, 0, 0), 24, 48, "hardswish"),
    (1, 1, (0, 0, 0, 0), 120, 360, "none"),
    (1, 1, (0, 0, 0, 0), 20, 36, "gelu"),    # oc % 16 != 0: bias last
    (1, 1, (0, 0, 0, 0), 5, 4, "hardsigmoid"),
    (2, 1, (0, 1, 0, 1), 8, 8, "gelu"),
    (5, 2, (2, 2, 2, 2), 6, 10, "sigmoid"),
    (3, 1, (1, 1, 1, 1), 16, 64, "hardsigmoidfifth"),
    (3, 1, (1, 1, 1, 1), 7, 13, "none"),
    # 3-wide, 32-channel blocks: the tensor cores with the horizontal taps folded
    (3, 1, (1, 1, 1, 1), 64, 40, "relu"),    # a slice's second 16-channel group half empty
    (3, 1, (1, 1, 1, 1), 32, 4, "swish"),    # one 16-channel group, 4 live
    (3, 1, (1, 1, 1, 1), 32, 128, "none"),   # four slices
    (5, 1, (2, 2, 2, 2), 32, 24, "none"),    # 5x5: the unfolded windowed path
]


@pytest.mark.parametrize("k,s,pads,ic,oc,fused", CONV_CASES)
def test_conv(cuda_mod, oracle_mod, k, s, pads, ic, oc, fused):
    h, w = 19, 23
    x = noise(h * w * ic, 3, 1.0)
    wt = noise(k * k * ic * oc, 5, 0.3)
    b = noise(oc, 7, 0.5)
    op = Op("conv", x=0, y=1, ic=ic, oc=oc, fused=fused, w=(0, wt.size), b=(wt.size, oc), kh=k, kw=k, sh=s, sw=s,
            pt=pads[0], pb=pads[1], pl=pads[2], pr=pads[3])
    plan = single(op, (h, w, ic), np.concatenate([wt, b]))
    check_both(cuda_mod, oracle_mod, plan, x, scale=1.0)


def test_conv_two_inputs(cuda_mod, oracle_mod):
    # a windowed conv over the concatenation of its input and a second one
    h, w, c1, c2, oc = 11, 9, 8, 12, 16
    first = window(Op("conv", x=0, y=1, ic=c1, oc=c2, w=(0, c1 * c2), b=(c1 * c2, c2)), (1, 1), 1, 0, 0)
    at = c1 * c2 + c2
    conv = window(Op("conv", x=0, y=2, ic=c1, oc=oc, x2=1, n2=c2), (3, 3), 1, 1, 1)
    conv.w, conv.b = (at, 9 * (c1 + c2) * oc), (at + 9 * (c1 + c2) * oc, oc)
    weights = noise(at + 9 * (c1 + c2) * oc + oc, 9, 0.4)
    plan = encode((0, h, w, c1), 3, [2], [first, conv], weights)
    x = noise(h * w * c1, 1, 1.0)
    check_both(cuda_mod, oracle_mod, plan, x)


@pytest.mark.parametrize("k,s,c,fused", [(3, 1, 8, "swish"), (3, 2, 12, "none"), (5, 1, 16, "relu"),
                                         (7, 1, 8, "none"), (5, 2, 5, "hardswish"), (5, 1, 96, "hardswish")])
def test_depthwise(cuda_mod, oracle_mod, k, s, c, fused):
    h, w = 21, 17
    x = noise(h * w * c, 11, 1.0)
    wt = noise(k * k * c, 13, 0.5)
    b = noise(c, 17, 0.5)
    p = k // 2
    op = window(Op("dwconv", x=0, y=1, ic=c, oc=c, fused=fused, w=(0, wt.size), b=(wt.size, c)), (k, k), s, p, p)
    plan = single(op, (h, w, c), np.concatenate([wt, b]))
    check_both(cuda_mod, oracle_mod, plan, x)


def elementwise_plan(kind, h, w, c, **kw):
    """pointwise producer of a second tensor (buffer 1), then `kind` from the
    image (buffer 0) and it into buffer 2."""
    prod_oc = kw.pop("prod_oc", c)
    prod = window(Op("conv", x=0, y=1, ic=c, oc=prod_oc, w=(0, c * prod_oc), b=(c * prod_oc, prod_oc)), (1, 1), 1, 0, 0)
    at = c * prod_oc + prod_oc
    extra = kw.pop("weights", 0)
    op = Op(kind, x=0, y=2, ic=c, oc=kw.pop("oc", c), x2=1, **kw)
    if extra:
        op.w = (at, extra)
    weights = noise(at + extra, 23, 0.5)
    return encode((0, h, w, c), 3, [2], [prod, op], weights)


@pytest.mark.parametrize("fused", ["none", "relu", "swish"])
def test_add(cuda_mod, oracle_mod, fused):
    plan = elementwise_plan("add", 13, 7, 12, fused=fused)
    x = noise(13 * 7 * 12, 2, 2.0)
    check_both(cuda_mod, oracle_mod, plan, x)


def test_concat_and_upsample(cuda_mod, oracle_mod):
    h, w, c = 6, 5, 8
    x = noise(h * w * c, 4, 1.0)
    for cin, plan in ((c, elementwise_plan("concatc", h, w, c, prod_oc=12, oc=20, n2=12)),
                      (3, elementwise_plan("concatc", h, w, 3, prod_oc=5, oc=8, n2=5))):
        xx = noise(h * w * cin, 4, 1.0)
        check_both(cuda_mod, oracle_mod, plan, xx)
    up = Op("upsample", x=0, y=1, ic=c, oc=c, sh=2, sw=3)
    plan = single(up, (h, w, c), np.zeros(0, np.float32))
    check(gpu_run(cuda_mod, plan, x)[0][0], oracle_run(oracle_mod, plan, x)[0])
    # upsampleadd: y = x2 + up(x); x2 made at the upsampled size by a stride-1 conv of an upsample
    upx = Op("upsample", x=0, y=1, ic=c, oc=c, sh=2, sw=2)
    conv = window(Op("conv", x=1, y=2, ic=c, oc=c, w=(0, c * c), b=(c * c, c)), (1, 1), 1, 0, 0)
    add = Op("upsampleadd", x=0, y=3, ic=c, oc=c, x2=2, sh=2, sw=2)
    plan = encode((0, h, w, c), 4, [3], [upx, conv, add], noise(c * c + c, 6, 0.5))
    check_both(cuda_mod, oracle_mod, plan, x)


def test_pools_mean_gates(cuda_mod, oracle_mod):
    h, w, c = 14, 10, 12
    x = noise(h * w * c, 8, 1.5)
    mp = Op("maxpool", x=0, y=1, ic=c, oc=c, kh=2, kw=2, sh=1, sw=1, pb=1, pr=1)
    plan = single(mp, (h, w, c), np.zeros(0, np.float32))
    check(gpu_run(cuda_mod, plan, x)[0][0], oracle_run(oracle_mod, plan, x)[0])
    ap = Op("avgpool", x=0, y=1, ic=c, oc=c, kh=7, kw=2, sh=7, sw=2)
    plan = single(ap, (h, w, c), np.zeros(0, np.float32))
    check(gpu_run(cuda_mod, plan, x)[0][0], oracle_run(oracle_mod, plan, x)[0])
    mean = Op("mean", x=0, y=1, ic=c, oc=c)
    plan = single(mean, (h, w, c), np.zeros(0, np.float32))
    check(gpu_run(cuda_mod, plan, x)[0][0], oracle_run(oracle_mod, plan, x)[0])
    # a squeeze-and-excite gate: mean -> 1x1 -> channelmul
    m = Op("mean", x=0, y=1, ic=c, oc=c)
    g = window(Op("conv", x=1, y=2, ic=c, oc=c, fused="hardsigmoid", w=(0, c * c), b=(c * c, c)), (1, 1), 1, 0, 0)
    cm = Op("channelmul", x=0, y=3, ic=c, oc=c, x2=2)
    plan = encode((0, h, w, c), 4, [3], [m, g, cm], noise(c * c + c, 5, 0.5))
    check_both(cuda_mod, oracle_mod, plan, x)


def test_mean_on_a_page(cuda_mod, oracle_mod):
    # layers.rs:1208-1233: a large offset plus small noise over 300k pixels
    pixels, c = 300_000, 3
    x = noise(pixels * c, 13, 0.01).reshape(pixels, c)
    x = (x + np.float32(1000.0) + np.arange(c, dtype=np.float32)).astype(np.float32).reshape(-1)
    plan = single(Op("mean", x=0, y=1, ic=c, oc=c), (600, 500, c), np.zeros(0, np.float32))
    got = gpu_run(cuda_mod, plan, x)[0][0]
    want = oracle_run(oracle_mod, plan, x)[0]
    assert max_gap(got, want) <= 1e-4


@pytest.mark.parametrize("t", [1, 7, 37, 203])
def test_attention(cuda_mod, oracle_mod, t):
    """Exact on the FP32 path; beside the tensor cores (eight threads per
    query, __expf) within the tolerance."""
    c, heads = 120, 8
    x = noise(t * 3 * c, 21, 1.5)
    att = Op("attention", x=0, y=1, ic=3 * c, oc=c, n2=heads, w=(0, 1))
    plan = single(att, (1, t, 3 * c), np.float32([15 ** -0.5]))
    check_both(cuda_mod, oracle_mod, plan, x)


def test_layernorm_attention(cuda_mod, oracle_mod):
    t, c = 37, 120
    gamma, beta = noise(c, 3, 1.0) + 1, noise(c, 4, 0.5)
    ln = Op("layernorm", x=0, y=1, ic=c, oc=c, w=(0, 2 * c + 1))
    xs = noise(t * c, 9, 3.0)
    plan = single(ln, (1, t, c), np.concatenate([gamma, beta, np.float32([1e-6])]))
    # beside the tensor cores the sums are warp reductions (within tolerance);
    # on the FP32 cores the reference's order, bit for bit
    check_both(cuda_mod, oracle_mod, plan, xs)


def ctc_plan(kind, t, ci, vocab, seed=7):
    cols = -(-vocab // 16) * 16
    logical = noise(ci * vocab, seed, 0.8).reshape(ci, vocab)
    full = np.zeros((ci, cols), np.float32)
    full[:, :vocab] = logical
    w = full.reshape(ci, cols // 16, 16).transpose(1, 0, 2).copy()
    b = np.full(cols, -1e30, np.float32)
    b[:vocab] = noise(vocab, 11, 0.5)
    if kind == "ctchead":
        op = Op("ctchead", x=0, y=1, ic=ci, oc=vocab, w=(0, w.size), b=(w.size, cols))
    else:
        op = Op("ctcargmax", x=0, y=1, ic=ci, oc=2, n2=vocab, w=(0, w.size), b=(w.size, cols))
    return single(op, (1, t, ci), np.concatenate([w.reshape(-1), b]))


@pytest.mark.parametrize("t,ci,vocab", [(1, 19, 37), (13, 19, 64), (40, 120, 18710), (97, 120, 1000)])
def test_ctc_head(cuda_mod, oracle_mod, t, ci, vocab):
    x = noise(t * ci, t + 3, 2.0)
    plan = ctc_plan("ctcargmax", t, ci, vocab)
    got = gpu_run(cuda_mod, plan, x)[0][0].reshape(t, 2)
    want = oracle_run(oracle_mod, plan, x)[0].reshape(t, 2)
    assert np.array_equal(got[:, 0], want[:, 0])
    # The logits are bit-identical; 1/sum is summed over the columns in
    # another order (per column block, then merged) than the reference's one
    # online pass, so it carries its rounding: within the 1e-5 the
    # reference's own CTC test allows (layers.rs:1313).
    assert max_gap(got[:, 1], want[:, 1]) <= 1e-5
    if vocab <= 1000:
        plan = ctc_plan("ctchead", t, ci, vocab)
        got = gpu_run(cuda_mod, plan, x)[0][0]
        assert max_gap(got, oracle_run(oracle_mod, plan, x)[0]) <= 1e-6


@pytest.mark.parametrize("bump,winner", [(0.0, 5.0), (1.2e-5, 300.0)], ids=["tie", "near-tie"])
@pytest.mark.parametrize("options", [0, 4], ids=["tensor-cores", "fp32-cores"])
def test_ctc_head_ties(cuda_mod, oracle_mod, options, bump, winner):
    """Ties the tensor-core logits cannot order: columns 5, 300 and 700 share
    weights and dominate every row; 700 copies 5 (an exact tie: the first
    wins) and 300's bias is 5's plus `bump`, a few ulps of the logits, so
    each row's class comes from the exact FP32 recompute."""
    t, ci, vocab = 64, 120, 1000
    cols = -(-vocab // 16) * 16
    logical = noise(ci * vocab, 31, 0.05).reshape(ci, vocab)
    bias = noise(vocab, 37, 0.5)
    strong = np.abs(noise(ci, 41, 1.0)) + np.float32(0.5)
    for c in (5, 300, 700):
        logical[:, c] = strong
        bias[c] = bias[5]
    bias[300] = bias[5] + np.float32(bump)
    full = np.zeros((ci, cols), np.float32)
    full[:, :vocab] = logical
    w = full.reshape(ci, cols // 16, 16).transpose(1, 0, 2).copy()
    b = np.full(cols, -1e30, np.float32)
    b[:vocab] = bias
    op = Op("ctcargmax", x=0, y=1, ic=ci, oc=2, n2=vocab, w=(0, w.size), b=(w.size, cols))
    plan = single(op, (1, t, ci), np.concatenate([w.reshape(-1), b]))
    x = np.abs(noise(t * ci, 43, 1.0))
    got = gpu_run(cuda_mod, plan, x, options=options)[0][0].reshape(t, 2)
    want = oracle_run(oracle_mod, plan, x)[0].reshape(t, 2)
    assert set(want[:, 0].tolist()) == {winner}
    assert np.array_equal(got[:, 0], want[:, 0])
    assert max_gap(got[:, 1], want[:, 1]) <= 1e-5


@pytest.mark.parametrize("ic,oc,k,fused", [(5, 3, 2, "none"), (24, 24, 2, "relu"), (24, 1, 2, "sigmoid"),
                                           (16, 4, 3, "swish")])
def test_convtranspose(cuda_mod, oracle_mod, ic, oc, k, fused):
    h, w = 9, 7
    x = noise(h * w * ic, 5, 1.0)
    wt = noise(ic * k * k * oc, 7, 0.6)
    b = noise(k * k * oc, 9, 0.5)
    op = Op("convtranspose", x=0, y=1, ic=ic, oc=oc, kh=k, kw=k, sh=k, sw=k, fused=fused,
            w=(0, wt.size), b=(wt.size, b.size))
    plan = single(op, (h, w, ic), np.concatenate([wt, b]))
    check_both(cuda_mod, oracle_mod, plan, x)


# ---------------------------------------------------------- fused layers, nets

def test_fused_layer_config1(cuda_mod, oracle_mod):
    """Benchmark config 1 at full size: dw 5x5 + hardswish -> pw 96->192 +
    hardswish, fused into one kernel."""
    plan = synth.fused_layer_plan(seed=0)
    x = np.random.default_rng(1).uniform(-1, 1, 240 * 240 * 96).astype(np.float32)
    steps = check_both(cuda_mod, oracle_mod, plan, x)
    assert steps == ["dw+pw"]


@pytest.mark.parametrize("h,w", [(64, 48), (40, 8), (16, 16), (8, 36), (4, 4)])
def test_page_model(cuda_mod, oracle_mod, h, w):
    plan = synth.page_model_plan(16, 16)
    x = synth.ramp_input(h * w * 3)
    check_both(cuda_mod, oracle_mod, plan, x, hw=(h, w))


@pytest.mark.parametrize("width", [3, 17, 40, 64, 1001])
def test_line_model(cuda_mod, oracle_mod, width):
    plan = synth.line_model_plan(40)
    x = synth.ramp_input(2 * width * 3)
    want = oracle_run(oracle_mod, plan, x, hw=(2, width))[0].reshape(-1, 2)
    for options in (0, cuda_mod.OPT_NO_TENSOR_CORES):
        got = gpu_run(cuda_mod, plan, x, hw=(2, width), options=options)[0][0].reshape(-1, 2)
        assert np.array_equal(got[:, 0], want[:, 0])
        assert max_gap(got[:, 1], want[:, 1]) <= 1e-5


@pytest.mark.parametrize("std", [None, 0.02], ids=["busy", "baseline-init"])
def test_detector_960x736(cuda_mod, oracle_mod, std):
    """Benchmark config 2: probabilities within 1e-4 with the pointwise
    layers on the tensor cores (3xTF32), bit-identical with every
    contraction on the FP32 cores. The neck's RSE outputs read only by an
    upsample-add are never written (their gate-add runs inside it): three
    such steps."""
    plan = synth.det_plan(seed=3, std=std)
    x = np.random.default_rng(4).normal(0, 1, 960 * 736 * 3).astype(np.float32)
    want = oracle_run(oracle_mod, plan, x)[0]
    got, steps = gpu_run(cuda_mod, plan, x)
    assert "dw+pw" in steps and "gate_add" in steps and any("sources" in s for s in steps)
    assert steps.count("gate_add+upsample_add") == 3, steps
    check(got[0], want, exact=False)
    got, _ = gpu_run(cuda_mod, plan, x, options=cuda_mod.OPT_NO_TENSOR_CORES)
    check(got[0], want)


def test_detector_lanes(cuda_mod, oracle_mod):
    """Three pages of different sizes in one detector run (lane-packed
    windowed convs, transposed convs and gates on the tensor cores): each
    within the tolerance of the oracle, and bit-identical to the oracle with
    every contraction on the FP32 cores."""
    plan = synth.det_plan(seed=11, std=None, size=(96, 64))
    sizes = [(96, 64), (64, 128), (32, 96)]
    xs = [synth.stripes(h, w, phase=7 * i) for i, (h, w) in enumerate(sizes)]
    o = oracle_mod.Oracle(plan)
    wants = []
    for (h, w), x in zip(sizes, xs):
        o.set_size(h, w)
        wants.append(o.run(x)[0])
    for options in (0, cuda_mod.OPT_NO_TENSOR_CORES):
        with cuda_mod.Model(plan) as m:
            if options:
                m.set_options(options)
            m.set_sizes(sizes)
            for i, x in enumerate(xs):
                m.lane_input_mut(i)[:] = x
            m.run(60_000)
            for i, want in enumerate(wants):
                check(m.lane_output(i).copy(), want, exact=bool(options))


def test_folded_conv_lanes(cuda_mod, oracle_mod):
    """A 3x3 96 -> 24 conv (horizontal taps folded into the tensor cores'
    columns, 120-pixel tiles of 30-pixel lane quadrants) over lanes whose
    widths and sizes fall on every tile and quadrant edge: 1, 2, 29..31,
    120, 121 pixels wide, one pixel high, and more tiles than SMs."""
    ic, oc = 96, 24
    wt = noise(9 * ic * oc, 5, 0.1)
    b = noise(oc, 7, 0.5)
    op = window(Op("conv", x=0, y=1, ic=ic, oc=oc, fused="swish", w=(0, wt.size), b=(wt.size, oc)), (3, 3), 1, 1, 1)
    plan = single(op, (8, 8, ic), np.concatenate([wt, b]))
    sizes = [(5, 1), (3, 2), (7, 29), (1, 30), (4, 31), (2, 120), (3, 121), (1, 1), (181, 97)]
    xs = [noise(h * w * ic, 11 + i, 1.0) for i, (h, w) in enumerate(sizes)]
    o = oracle_mod.Oracle(plan)
    wants = []
    for (h, w), x in zip(sizes, xs):
        o.set_size(h, w)
        wants.append(o.run(x)[0])
    for options in (0, cuda_mod.OPT_NO_TENSOR_CORES):
        with cuda_mod.Model(plan) as m:
            if options:
                m.set_options(options)
            m.set_sizes(sizes)
            for i, x in enumerate(xs):
                m.lane_input_mut(i)[:] = x
            m.run(60_000)
            for i, want in enumerate(wants):
                check(m.lane_output(i).copy(), want, exact=bool(options),
                      tol=TOL * max(1.0, float(np.abs(want).max())))


@pytest.mark.parametrize("k,s,c,oc", [(3, 1, 24, 24), (3, 2, 48, 96), (5, 1, 96, 192), (5, 2, 40, 24)])
def test_depthwise_pointwise_step_on_tensor_cores(cuda_mod, oracle_mod, k, s, c, oc):
    """A depthwise layer feeding a 1x1 layer, as one step beside the tensor
    cores, within the tolerance of the oracle; strides 1 and 2, 3x3 and 5x5,
    channel counts that leave part of a K block, several lanes of different
    sizes. Beside the tensor cores the pair runs as the row-run depthwise
    kernel then the pointwise tensor-core kernel: the same bits as the two
    layers run as separate steps."""
    rng = np.random.default_rng(k * 100 + s * 10 + c)
    dw_w = rng.normal(0, 0.3, k * k * c).astype(np.float32)
    dw_b = rng.normal(0, 0.2, c).astype(np.float32)
    pw_w = rng.normal(0, 0.2, c * oc).astype(np.float32)
    pw_b = rng.normal(0, 0.2, oc).astype(np.float32)
    dw = window(Op("dwconv", x=0, y=1, ic=c, oc=c, fused="hardswish", w=(0, dw_w.size), b=(dw_w.size, c)),
                (k, k), s, k // 2, k // 2)
    at = dw_w.size + c
    pw = window(Op("conv", x=1, y=2, ic=c, oc=oc, fused="swish", w=(at, pw_w.size), b=(at + pw_w.size, oc)),
                (1, 1), 1, 0, 0)
    plan = encode((0, 16, 16, c), 3, [2], [dw, pw], np.concatenate([dw_w, dw_b, pw_w, pw_b]))
    sizes = [(37, 41), (8, 130), (3, 5)]
    xs = [rng.uniform(-1, 1, h * w * c).astype(np.float32) for h, w in sizes]
    o = oracle_mod.Oracle(plan)
    wants = []
    for (h, w), x in zip(sizes, xs):
        o.set_size(h, w)
        wants.append(o.run(x)[0])
    outs = []
    for options in (0, cuda_mod.OPT_NO_FUSION):
        with cuda_mod.Model(plan) as m:
            if options:
                m.set_options(options)
            m.set_sizes(sizes)
            for i, x in enumerate(xs):
                m.lane_input_mut(i)[:] = x
            m.run(60_000)
            if not options:
                assert m.steps() == ["dw+pw"]
            outs.append([m.lane_output(i).copy() for i in range(len(sizes))])
    for fused, apart, want in zip(outs[0], outs[1], wants):
        assert np.array_equal(fused, apart), max_gap(fused, apart)
        assert max_gap(fused, want) <= TOL * max(1.0, float(np.abs(want).max()))


def test_detector_unfused_matches_fused(cuda_mod):
    plan = synth.det_plan(seed=5, std=None, size=(320, 256))
    x = synth.stripes(320, 256)
    fp32 = cuda_mod.OPT_NO_TENSOR_CORES
    fused, _ = gpu_run(cuda_mod, plan, x, options=fp32)
    plain, steps = gpu_run(cuda_mod, plan, x, options=fp32 | cuda_mod.OPT_NO_FUSION | cuda_mod.OPT_NO_GRAPH)
    assert "dw+pw" not in steps
    assert np.array_equal(fused[0], plain[0])


@pytest.mark.parametrize("fp32", [False, True], ids=["tensor-cores", "fp32-cores"])
def test_recogniser_16_lanes(cuda_mod, oracle_mod, fp32):
    """Benchmark config 3: 16 lines of 48 x 320 in one batch; classes
    identical and probabilities within 1e-4 of the oracle, lane by lane."""
    plan = synth.rec_plan(seed=2, std=None)
    rng = np.random.default_rng(6)
    xs = [rng.normal(0, 1, 48 * 320 * 3).astype(np.float32) for _ in range(16)]
    with cuda_mod.Model(plan) as m:
        if fp32:
            m.set_options(cuda_mod.OPT_NO_TENSOR_CORES)
        m.set_sizes([(48, 320)] * 16)
        for i, x in enumerate(xs):
            m.lane_input_mut(i)[:] = x
        m.run(60_000)
        outs = [m.lane_output(i).copy().reshape(-1, 2) for i in range(16)]
    o = oracle_mod.Oracle(plan)
    classes = set()
    for x, got in zip(xs, outs):
        want = o.run(x)[0].reshape(-1, 2)
        assert np.array_equal(got[:, 0], want[:, 0])
        assert max_gap(got[:, 1], want[:, 1]) <= TOL
        classes |= set(want[:, 0].tolist())
    assert len(classes) > 5  # the busy weights make varied classes


def test_lanes_of_different_sizes(cuda_mod, oracle_mod):
    """gpu.rs:57-84: lanes of several widths in one run each match the CPU,
    and a lane alone gives the bits it gives alongside others."""
    plan = synth.rec_plan(seed=1, std=None, vocab=500)
    widths = [640, 96, 1280, 96, 320]
    xs = [synth.stripes(48, wd, phase=i * 31) for i, wd in enumerate(widths)]
    with cuda_mod.Model(plan) as m:
        m.set_sizes([(48, wd) for wd in widths])
        for i, x in enumerate(xs):
            m.lane_input_mut(i)[:] = x
        m.run(60_000)
        together = [m.lane_output(i).copy() for i in range(len(widths))]
        m.set_sizes([(48, widths[1])])
        m.input_mut()[:] = xs[1]
        m.run(60_000)
        alone = m.output().copy()
    assert np.array_equal(alone, together[1])
    o = oracle_mod.Oracle(plan)
    for wd, x, got in zip(widths, xs, together):
        o.set_size(48, wd)
        want = o.run(x)[0].reshape(-1, 2)
        got = got.reshape(-1, 2)
        assert np.array_equal(got[:, 0], want[:, 0])
        assert max_gap(got[:, 1], want[:, 1]) <= TOL


def test_bad_size_keeps_model(cuda_mod):
    plan = synth.page_model_plan(16, 16)
    x = synth.ramp_input(16 * 16 * 3)
    with cuda_mod.Model(plan) as m:
        m.input_mut()[:] = x
        m.run(60_000)
        before = m.output().copy()
        for h, w in [(10, 16), (16, 22), (0, 16), (1 << 20, 1 << 20)]:
            with pytest.raises(cuda_mod.PpocrError) as e:
                m.set_input_size(h, w)
            assert e.value.code == cuda_mod.E_SIZE
        assert m.input_mut().size == 16 * 16 * 3
        m.input_mut()[:] = x
        m.run(60_000)
        assert np.array_equal(m.output(), before)


def test_share_weights_and_graph_replay(cuda_mod):
    plan = synth.det_plan(seed=8, std=None, size=(256, 192))
    x = synth.stripes(256, 192)
    with cuda_mod.Model(plan) as m:
        m.input_mut()[:] = x
        m.run(60_000)
        first = m.output().copy()
        m.run(60_000)  # graph replay
        assert np.array_equal(m.output(), first)
        with m.share_weights() as m2:
            m2.input_mut()[:] = x
            m2.run(60_000)
            assert np.array_equal(m2.output(), first)
        m.set_options(cuda_mod.OPT_NO_GRAPH)
        m.input_mut()[:] = x
        m.run(60_000)
        assert np.array_equal(m.output(), first)


def test_wait_times_out_and_recovers(cuda_mod):
    """A wait shorter than the run returns PPOCR_E_TIMEOUT; the run itself
    completes and a later wait returns it (no kernel is harmed)."""
    plan = synth.det_plan(seed=0, size=(1984, 1536))
    with cuda_mod.Model(plan) as m:
        m.set_sizes([(1984, 1536)] * 4)
        m.enqueue()
        try:
            m.wait(1)
            timed_out = False
        except cuda_mod.PpocrError as e:
            assert e.code == cuda_mod.E_TIMEOUT
            timed_out = True
        m.wait(0)
        assert timed_out, "four 1984x1536 pages finished within 1 ms"
        assert np.isfinite(m.lane_output(3)).all()


def _cudart():
    pats = glob.glob(os.path.join(os.path.dirname(np.__file__), "..", "nvidia", "cuda_runtime", "lib",
                                  "libcudart.so*"))
    for p in pats + ["libcudart.so.12", "/usr/local/cuda/lib64/libcudart.so"]:
        try:
            return ctypes.CDLL(p)
        except OSError:
            continue
    pytest.fail("no libcudart to copy device memory with")


def test_device_resident_path(cuda_mod, oracle_mod):
    """Inputs written straight to device memory, a run that copies nothing,
    the output read from device memory."""
    rt = _cudart()
    rt.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    plan = synth.page_model_plan(32, 24)
    x = synth.ramp_input(32 * 24 * 3)
    with cuda_mod.Model(plan) as m:
        m.set_options(cuda_mod.OPT_NO_TENSOR_CORES)
        dptr, n = m.lane_device_input(0)
        assert n == x.size
        assert rt.cudaMemcpy(dptr, x.ctypes.data, x.nbytes, 1) == 0
        m.enqueue_device()
        m.wait(60_000)
        optr, on = m.lane_device_output(0, 0)
        out = np.empty(on, np.float32)
        assert rt.cudaMemcpy(out.ctypes.data, optr, out.nbytes, 2) == 0
    check(out, oracle_run(oracle_mod, plan, x)[0])


def test_models_sharing_a_stream(cuda_mod):
    """Two models queued on one stream give what they give apart, and can be
    freed in either order (the borrowed stream is never touched on free)."""
    det = synth.det_plan(seed=9, std=None, size=(128, 96))
    rec = synth.rec_plan(seed=9, std=None, vocab=300)
    xd, xr = synth.stripes(128, 96), synth.stripes(48, 200)
    apart = []
    for plan, x, hw in ((det, xd, None), (rec, xr, (48, 200))):
        apart.append(gpu_run(cuda_mod, plan, x, hw=hw)[0][0])
    for first_closed in (0, 1):
        a = cuda_mod.Model(det)
        b = cuda_mod.Model(rec)
        b.set_stream(a.stream)
        b.set_input_size(48, 200)
        a.input_mut()[:] = xd
        b.input_mut()[:] = xr
        a.enqueue()
        b.enqueue()
        b.wait(60_000)
        a.wait(60_000)
        assert np.array_equal(a.output(), apart[0])
        assert np.array_equal(b.output(), apart[1])
        models = [a, b]
        models[first_closed].close()
        models[1 - first_closed].close()


@pytest.mark.parametrize("k,n", [(24, 24), (48, 96), (96, 192), (192, 192), (384, 384), (120, 360), (36, 20),
                                 (240, 120), (13, 40)])
def test_pointwise_tensor_cores(cuda_mod, oracle_mod, k, n):
    """A pointwise layer large enough for the tensor cores (3xTF32): within
    a few units of the FP32 result, relative to the output's scale, and the
    same kernel bit for bit from run to run."""
    h, w = 37, 91  # 3367 pixels: 27 tiles of 128, the last one partial
    x = noise(h * w * k, 3, 1.0)
    wt = noise(k * n, 5, float(k) ** -0.5)
    b = noise(n, 7, 0.5)
    op = window(Op("conv", x=0, y=1, ic=k, oc=n, fused="relu", w=(0, wt.size), b=(wt.size, n)), (1, 1), 1, 0, 0)
    plan = single(op, (h, w, k), np.concatenate([wt, b]))
    got, _ = gpu_run(cuda_mod, plan, x)
    again, _ = gpu_run(cuda_mod, plan, x)
    assert np.array_equal(got[0], again[0])
    want = oracle_run(oracle_mod, plan, x)[0]
    assert max_gap(got[0], want) <= 2e-5 * max(1.0, float(np.abs(want).max()))
    exact, _ = gpu_run(cuda_mod, plan, x, options=cuda_mod.OPT_NO_TENSOR_CORES)
    check(exact[0], want)


def test_throughput_grids_give_the_same_bits(cuda_mod):
    """PPOCR_OPT_THROUGHPUT sizes the tensor-core grids for several runs in
    flight (small layers on few SMs, no narrowed slices): every output's sum
    is formed the same way, so the detector and a multi-lane recogniser give
    the same bits as with the default grids."""
    rng = np.random.default_rng(9)
    det = synth.det_plan(seed=11, std=None, size=(256, 192))
    x = rng.standard_normal(256 * 192 * 3).astype(np.float32)
    outs = []
    for opts in (0, cuda_mod.OPT_THROUGHPUT):
        with cuda_mod.Model(det) as m:
            m.set_options(opts)
            m.input_mut()[:] = x
            m.run(60_000)
            outs.append(m.output().copy())
    assert np.array_equal(outs[0], outs[1])
    rec = synth.rec_plan(seed=12, std=None, vocab=2000)
    widths = [320, 96, 800, 48 * 9]
    xs = [rng.standard_normal(48 * w * 3).astype(np.float32) for w in widths]
    outs = []
    for opts in (0, cuda_mod.OPT_THROUGHPUT):
        with cuda_mod.Model(rec) as m:
            m.set_options(opts)
            m.set_sizes([(48, w) for w in widths])
            for i, xi in enumerate(xs):
                m.lane_input_mut(i)[:] = xi
            m.run(60_000)
            outs.append([m.lane_output(i).copy() for i in range(len(widths))])
    for a, b in zip(*outs):
        assert np.array_equal(a, b)


TILE_SHAPES = [(24, 24, 3, 1), (24, 48, 3, 2), (48, 48, 3, 1), (48, 96, 3, 2), (96, 96, 3, 1), (96, 192, 3, 2),
               (48, 96, 5, 1), (24, 24, 5, 2), (96, 192, 5, 1)]


@pytest.mark.parametrize("c,n,k,s", TILE_SHAPES)
def test_fused_dw_pw_row_tiles(cuda_mod, oracle_mod, c, n, k, s):
    """The fused depthwise -> pointwise row-tile kernel (narrow layers, both
    modes): lanes of different sizes (rows shorter and longer than a tile,
    a one-pixel row), swish after both layers; bit for
    bit against the oracle in the exact mode, within 1e-4 of the output's
    scale with the tensor-core mode's activation quotient."""
    rng = np.random.default_rng(c * 7 + n + k + s)
    dww = rng.normal(0, 0.2, k * k * c).astype(np.float32)
    dwb = rng.normal(0, 0.1, c).astype(np.float32)
    pww = rng.normal(0, 0.2, c * n).astype(np.float32)
    pwb = rng.normal(0, 0.1, n).astype(np.float32)
    blob = np.concatenate([dww, dwb, pww, pwb])
    at = np.cumsum([0, dww.size, dwb.size, pww.size])
    dw = window(Op("dwconv", x=0, y=1, ic=c, oc=c, fused="swish", w=(int(at[0]), dww.size), b=(int(at[1]), c)),
                (k, k), s, k // 2, k // 2)
    pw = window(Op("conv", x=1, y=2, ic=c, oc=n, fused="swish", w=(int(at[2]), pww.size), b=(int(at[3]), n)),
                (1, 1), 1, 0, 0)
    plan = encode((0, 40, 300, c), 3, [2], [dw, pw], blob)
    sizes = [(40, 300), (7, 13), (1, 1), (33, 129), (12, 64)]
    xs = [rng.uniform(-1, 1, h * w * c).astype(np.float32) for h, w in sizes]
    o = oracle_mod.Oracle(plan)
    wants = []
    for (h, w), x in zip(sizes, xs):
        o.set_size(h, w)
        wants.append(o.run(x)[0])
    for opts in (cuda_mod.OPT_NO_TENSOR_CORES, 0):
        with cuda_mod.Model(plan) as m:
            m.set_options(opts)
            m.set_sizes(sizes)
            for i, x in enumerate(xs):
                m.lane_input_mut(i)[:] = x
            m.run(60_000)
            assert m.steps() == ["dw+pw"]
            for i, want in enumerate(wants):
                got = m.lane_output(i)
                if opts:
                    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (sizes[i], opts)
                else:
                    assert max_gap(got, want) <= 1e-4 * max(1.0, float(np.abs(want).max())), sizes[i]


def test_lane_layouts_back_to_back(cuda_mod):
    """A model whose lanes change run after run (more, fewer, wider,
    narrower; its buffers are kept and its lane tables rewritten) gives each
    run the bits a fresh model gives it."""
    plan = synth.rec_plan(seed=12, std=None, vocab=600)
    rng = np.random.default_rng(3)
    layouts = [[320, 800, 96, 1280, 48 * 9], [96], [1600, 320], [48 * 7] * 12, [640]]
    inputs = [[rng.standard_normal(48 * w * 3).astype(np.float32) for w in ws] for ws in layouts]
    fresh = []
    for ws, xs in zip(layouts, inputs):
        with cuda_mod.Model(plan) as m:
            m.set_sizes([(48, w) for w in ws])
            for i, x in enumerate(xs):
                m.lane_input_mut(i)[:] = x
            m.run(60_000)
            fresh.append([m.lane_output(i).copy() for i in range(len(ws))])
    with cuda_mod.Model(plan) as m:
        for _ in range(2):
            for ws, xs, want in zip(layouts, inputs, fresh):
                m.set_sizes([(48, w) for w in ws])
                for i, x in enumerate(xs):
                    m.lane_input_mut(i)[:] = x
                m.run(60_000)
                for i in range(len(ws)):
                    assert np.array_equal(m.lane_output(i), want[i])



def test_narrow_pointwise_rows(cuda_mod, oracle_mod):
    """Narrow pointwise layers in both modes: a layer gated by a
    squeeze-and-excite vector (the gate folded into its input loads), one
    with a residual add folded in, lanes whose widths are not multiples of
    four, a one-pixel lane; bit for bit against the oracle with every
    contraction on the FP32 cores, within 1e-4 beside the tensor cores."""
    rng = np.random.default_rng(21)
    blobs, at = [], 0

    def weights(n):
        nonlocal at
        v = rng.normal(0, 0.3, n).astype(np.float32)
        blobs.append(v)
        at += n
        return (at - n, n)

    ops = [Op("mean", x=0, y=1, ic=24, oc=24)]
    op = window(Op("conv", x=1, y=2, ic=24, oc=24, fused="hardsigmoid"), (1, 1), 1, 0, 0)
    op.w, op.b = weights(24 * 24), weights(24)
    ops.append(op)
    ops.append(Op("channelmul", x=0, y=3, ic=24, oc=24, x2=2))
    op = window(Op("conv", x=3, y=4, ic=24, oc=48, fused="swish"), (1, 1), 1, 0, 0)
    op.w, op.b = weights(24 * 48), weights(48)
    ops.append(op)
    op = window(Op("conv", x=4, y=5, ic=48, oc=48, fused="none"), (1, 1), 1, 0, 0)
    op.w, op.b = weights(48 * 48), weights(48)
    ops.append(op)
    ops.append(Op("add", x=5, y=6, ic=48, oc=48, x2=4))
    plan = encode((0, 16, 16, 24), 7, [6], ops, np.concatenate(blobs))
    sizes = [(7, 13), (1, 1), (33, 129), (12, 66)]
    xs = [rng.uniform(-1, 1, h * w * 24).astype(np.float32) for h, w in sizes]
    o = oracle_mod.Oracle(plan)
    wants = []
    for (h, w), x in zip(sizes, xs):
        o.set_size(h, w)
        wants.append(o.run(x)[0])
    for opts in (cuda_mod.OPT_NO_TENSOR_CORES, 0):
        with cuda_mod.Model(plan) as m:
            m.set_options(opts)
            m.set_sizes(sizes)
            for i, x in enumerate(xs):
                m.lane_input_mut(i)[:] = x
            m.run(60_000)
            assert "gate+conv" in m.steps() and "conv+add" in m.steps(), m.steps()
            for i, want in enumerate(wants):
                got = m.lane_output(i)
                if opts:
                    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), sizes[i]
                else:
                    assert max_gap(got, want) <= 1e-4 * max(1.0, float(np.abs(want).max())), sizes[i]


@pytest.mark.parametrize("k", [3, 5], ids=["folded-3x3", "5x5"])
def test_conv_sources(cuda_mod, oracle_mod, k):
    """A windowed conv over four sources, three of them nearest-upsampled
    by 8, 4 and 2 (an upsample + concat chain, the DB head's shape) and the
    second input at full size, folded into the conv as sources: on the FP32
    cores read in place, bit for bit against the oracle; on the tensor cores
    (their nearest-upsampled copy side by side, then the conv: 3-wide with
    its horizontal taps folded, 5x5 not) within 1e-4 of the output's scale;
    lanes of different sizes."""
    from ppocr_native_b200.plan import Builder

    b = Builder(64, 96, 24, np.random.default_rng(40 + k), None)
    s8, s4, s2 = b.avgpool(0, (8, 8), (8, 8)), b.avgpool(0, (4, 4), (4, 4)), b.avgpool(0, (2, 2), (2, 2))
    cat = b.concat(b.concat(b.upsample(s8, 8), b.upsample(s4, 4)), b.upsample(s2, 2))
    y = b.conv(cat, 24, k=k, act="relu", x2=0)
    plan = b.build([y])
    sizes = [(64, 96), (32, 40), (8, 8), (48, 128)]
    rng = np.random.default_rng(k)
    xs = [rng.uniform(-1, 1, h * w * 24).astype(np.float32) for h, w in sizes]
    o = oracle_mod.Oracle(plan)
    wants = []
    for (h, w), x in zip(sizes, xs):
        o.set_size(h, w)
        wants.append(o.run(x)[0])
    for options in (0, cuda_mod.OPT_NO_TENSOR_CORES):
        with cuda_mod.Model(plan) as m:
            if options:
                m.set_options(options)
            m.set_sizes(sizes)
            for i, x in enumerate(xs):
                m.lane_input_mut(i)[:] = x
            m.run(60_000)
            assert any("sources" in st for st in m.steps()), m.steps()
            for i, want in enumerate(wants):
                check(m.lane_output(i).copy(), want, exact=bool(options),
                      tol=TOL * max(1.0, float(np.abs(want).max())))
