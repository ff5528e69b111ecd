"""Pinning the CPU oracle (oracle/ppocr_oracle.c) to the reference's own
known-answer tests. The reference ships no network-level golden vectors for
the engine; its engine tests compare each layer with an f64 definition under
stated bounds, and its plan/size tests name the malformed files and sizes it
refuses. The same definitions, bounds, inputs (the xorshift `noise`, the
`sin(0.37 i)` ramp, the `cos` fills) and cases are checked here against the
oracle. Each test cites the reference test it restates.
"""

from __future__ import annotations

import math
import struct

import numpy as np
import pytest

from common import Op, encode, max_gap, noise, single, window
from ppocr_native_b200 import synth
from ppocr_native_b200.plan import ACT


def act_plan(code: str, xs: np.ndarray) -> bytes:
    """An add of the values and zeros with a folded activation."""
    n = xs.size
    add = Op("add", x=0, y=2, ic=1, oc=1, x2=1, fused=code)
    zero = Op("conv", x=0, y=1, ic=1, oc=1, kh=1, kw=1, sh=1, sw=1, w=(0, 1))
    return encode((0, 1, n, 1), 3, [2], [zero, add], np.zeros(1, np.float32))


def activation_values(oracle_mod, code: str, xs: np.ndarray) -> np.ndarray:
    return np.array([oracle_mod.activation(ACT[code], float(v)) for v in xs], np.float32)


@pytest.mark.parametrize("n", [1003, 70001])
@pytest.mark.parametrize("code", ["relu", "sigmoid", "gelu", "swish", "hardsigmoid", "hardsigmoidfifth",
                                  "hardswish"])
def test_layer_activations_match_the_scalar_definition(oracle_mod, code, n):
    """A layer's fused activation (eight lanes at a time, the rest one by
    one, spans past 64 Ki values split over threads) gives orc_activation's
    bits on every value: signed zeros, infinities, NaN, the exp cut-off and
    the clamp edges among seeded normals of several scales."""
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 87.3, -87.3, 88.8, -88.8, 104.0, -104.0, 3.0, -3.0,
                        2.9999998, -2.9999998, 5.5, -5.5, 6.0, -6.0, 2.5, -2.5, 1e-30, -1e-30, 1e-7, -1e-7],
                       np.float32)
    rng = np.random.default_rng(n)
    xs = np.concatenate([special, (rng.standard_normal(n - special.size) *
                                   rng.choice([0.1, 1.0, 10.0, 100.0], n - special.size)).astype(np.float32)])
    got = oracle_mod.Oracle(act_plan(code, xs)).run(xs)[0]
    with np.errstate(invalid="ignore", over="ignore"):
        zero_conv = xs * np.float32(0.0) + np.float32(0.0)  # the plan's zero-weight conv: NaN at the infinities
        want = activation_values(oracle_mod, code, xs + zero_conv)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    ok = ~np.isnan(want)
    assert np.array_equal(got[ok].view(np.uint32), want[ok].view(np.uint32))


# activation.rs:241-300 (sigmoid_tiers_match_scalar_and_libm)
def test_sigmoid_within_1e7_of_float64(oracle_mod):
    xs = np.concatenate([(np.arange(4000, dtype=np.float32) - 2000) * np.float32(0.0517),
                         np.float32([0, -0.0, 3.0, -3.0, -87.33654, 87.33654, 1e-40, -1e-40])]).astype(np.float32)
    got = activation_values(oracle_mod, "sigmoid", xs)
    for g, v in zip(got, xs):
        exact = 1.0 / (1.0 + math.exp(-float(v)))
        gap = abs(float(g) - exact)
        assert gap <= 1e-7, (v, g, exact)
        assert exact < np.finfo(np.float32).tiny or gap <= 4 * np.finfo(np.float32).eps * exact, (v, g)
    ends = activation_values(oracle_mod, "sigmoid", np.float32([-np.inf, -100, 0, -0.0, 100, np.inf]))
    assert list(ends) == [0.0, 0.0, 0.5, 0.5, 1.0, 1.0]


# layers.rs:1098-1130 (activation_tiers_match_scalar)
def test_gelu_and_swish_match_float64(oracle_mod):
    xs = (np.arange(-4000, 4000, dtype=np.float32) * np.float32(0.0025)).astype(np.float32)
    gelu = activation_values(oracle_mod, "gelu", xs)
    swish = activation_values(oracle_mod, "swish", xs)
    for x, g, s in zip(xs.astype(np.float64), gelu, swish):
        bound = 2e-6 * max(abs(x), 1.0)
        want = 0.5 * x * (1.0 + math.erf(x / math.sqrt(2.0)))
        assert abs(float(g) - want) < bound / 4, (x, g, want)
        want = x / (1.0 + math.exp(-x))
        assert abs(float(s) - want) < bound, (x, s, want)


def test_exp_neg_matches_float64(oracle_mod):
    for z in np.linspace(-87, 0, 2001, dtype=np.float32):
        e = oracle_mod.exp_neg(float(z))
        exact = math.exp(float(z))
        # XNNPACK documents the p5 exp to within a few ulp
        assert abs(e - exact) <= 4e-7 * exact + 1e-38, (z, e, exact)
    assert oracle_mod.exp_neg(-100.0) == 0.0
    assert oracle_mod.exp_neg(0.0) == 1.0


def test_hard_activations(oracle_mod):
    xs = np.linspace(-6, 6, 97, dtype=np.float32)
    alpha = np.float32(struct.unpack("<f", struct.pack("<I", 0x3E2AAAAD))[0])
    hs = np.clip(xs * alpha + np.float32(0.5), 0, 1).astype(np.float32)
    assert np.array_equal(activation_values(oracle_mod, "hardsigmoid", xs), hs)
    h5 = np.clip(xs * np.float32(0.2) + np.float32(0.5), 0, 1).astype(np.float32)
    assert np.array_equal(activation_values(oracle_mod, "hardsigmoidfifth", xs), h5)
    assert np.array_equal(activation_values(oracle_mod, "hardswish", xs), (xs * hs).astype(np.float32))
    assert np.array_equal(activation_values(oracle_mod, "relu", xs), np.maximum(xs, 0))


# layers.rs:1163-1206 (transposed_convolution_matches_float64), with relu in
# place of the test's (-0.25, 0.75) clamp, which no plan activation expresses.
@pytest.mark.parametrize("fused", ["none", "relu"])
def test_transposed_convolution_matches_float64(oracle_mod, fused):
    ih, iw, ic, kh, kw, oc = 3, 4, 5, 2, 3, 3
    x = noise(ih * iw * ic, 5, 1.0)
    w = noise(ic * kh * kw * oc, 7, 1.0)
    b = noise(kh * kw * oc, 9, 0.5)
    op = Op("convtranspose", x=0, y=1, ic=ic, oc=oc, kh=kh, kw=kw, sh=kh, sw=kw, fused=fused,
            w=(0, w.size), b=(w.size, b.size))
    got = oracle_mod.Oracle(single(op, (ih, iw, ic), np.concatenate([w, b]))).run(x)[0]
    ow = iw * kw
    X = x.reshape(ih, iw, ic).astype(np.float64)
    Wt = w.reshape(ic, kh, kw, oc).astype(np.float64)
    for i, g in enumerate(got):
        pixel, o = divmod(i, oc)
        r, col = divmod(pixel, ow)
        want = float(X[r // kh, col // kw] @ Wt[:, r % kh, col % kw, o]) + float(b[(r % kh * kw + col % kw) * oc + o])
        if fused == "relu":
            want = max(want, 0.0)
        assert abs(float(g) - want) < 1e-5, (i, g, want)


# layers.rs:1208-1233 (channel_mean_holds_on_pages)
def test_channel_mean_holds_on_pages(oracle_mod):
    pixels, c = 300_000, 3
    x = noise(pixels * c, 13, 0.01).reshape(pixels, c)
    x = (x + np.float32(1000.0) + np.arange(c, dtype=np.float32)).astype(np.float32)
    op = Op("mean", x=0, y=1, ic=c, oc=c)
    got = oracle_mod.Oracle(single(op, (600, 500, c), np.zeros(0, np.float32))).run(x.reshape(-1))[0]
    want = x.astype(np.float64).sum(0) / pixels
    assert np.all(np.abs(got.astype(np.float64) - want) < 1e-4)


# layers.rs:1257-1318 (ctc_head_tiers_match_scalar): argmax exact, every
# probability and 1/sum within 1e-5 of the f64 softmax.
@pytest.mark.parametrize("vocab", [37, 64])
@pytest.mark.parametrize("t", [1, 4, 6, 7, 13])
def test_ctc_head_matches_float64(oracle_mod, vocab, t):
    ci = 19
    cols = -(-vocab // 16) * 16
    logical = noise(ci * vocab, 7, 0.8).reshape(ci, vocab)
    w = np.zeros((cols // 16, ci, 16), np.float32)
    full = np.zeros((ci, cols), np.float32)
    full[:, :vocab] = logical
    w[:] = full.reshape(ci, cols // 16, 16).transpose(1, 0, 2)
    b = np.full(cols, -1e30, np.float32)
    b[:vocab] = noise(vocab, 11, 0.5)
    x = noise(t * ci, t + 3, 2.0)
    logits = x.reshape(t, ci).astype(np.float64) @ logical.astype(np.float64) + b[:vocab].astype(np.float64)
    mx = logits.max(1, keepdims=True)
    e = np.exp(logits - mx)
    probs_want = e / e.sum(1, keepdims=True)
    weights = np.concatenate([w.reshape(-1), b])
    head = Op("ctchead", x=0, y=1, ic=ci, oc=vocab, w=(0, w.size), b=(w.size, cols))
    probs = oracle_mod.Oracle(single(head, (1, t, ci), weights)).run(x)[0].reshape(t, vocab)
    assert np.max(np.abs(probs - probs_want)) < 1e-5
    arg = Op("ctcargmax", x=0, y=1, ic=ci, oc=2, n2=vocab, w=(0, w.size), b=(w.size, cols))
    out = oracle_mod.Oracle(single(arg, (1, t, ci), weights)).run(x)[0].reshape(t, 2)
    assert np.array_equal(out[:, 0], logits.argmax(1).astype(np.float32))
    assert np.max(np.abs(out[:, 1] - 1.0 / e.sum(1))) < 1e-5


def conv_f64(x, w, b, kh, kw, s, pads, oc):
    """Dense conv in f64 over an HWC image, w [kh][kw][c][oc]."""
    h, wd, c = x.shape
    pt, pb, pl, pr = pads
    xp = np.zeros((h + pt + pb, wd + pl + pr, c))
    xp[pt:pt + h, pl:pl + wd] = x
    oh = (h + pt + pb - kh) // s + 1
    ow = (wd + pl + pr - kw) // s + 1
    y = np.zeros((oh, ow, oc)) + b
    for ky in range(kh):
        for kx in range(kw):
            patch = xp[ky:ky + s * (oh - 1) + 1:s, kx:kx + s * (ow - 1) + 1:s]
            y += patch @ w[ky, kx]
    return y


# dense.rs:547-623 and depthwise.rs:528-648 compare kernels with their
# definitions; here the oracle's convolutions against f64.
@pytest.mark.parametrize("k,s,pads,ic,oc", [(3, 2, (1, 1, 1, 1), 3, 24), (3, 1, (1, 1, 1, 1), 12, 16),
                                            (1, 1, (0, 0, 0, 0), 20, 36), (2, 1, (0, 1, 0, 1), 8, 8),
                                            (5, 2, (2, 2, 2, 2), 6, 10)])
def test_conv_matches_float64(oracle_mod, k, s, pads, ic, oc):
    h, w = 13, 17
    x = noise(h * w * ic, 3, 1.0)
    wt = noise(k * k * ic * oc, 5, 0.5)
    b = noise(oc, 7, 0.5)
    op = window(Op("conv", x=0, y=1, ic=ic, oc=oc, w=(0, wt.size), b=(wt.size, oc)), (k, k), s, pads[0], pads[1])
    got = oracle_mod.Oracle(single(op, (h, w, ic), np.concatenate([wt, b]))).run(x)[0]
    want = conv_f64(x.reshape(h, w, ic).astype(np.float64), wt.reshape(k, k, ic, oc).astype(np.float64),
                    b.astype(np.float64), k, k, s, pads, oc)
    assert max_gap(got, want.reshape(-1).astype(np.float32)) < 2e-5


@pytest.mark.parametrize("k,s,c", [(3, 1, 8), (3, 2, 12), (5, 1, 16), (7, 1, 8), (5, 2, 5)])
def test_depthwise_matches_float64(oracle_mod, k, s, c):
    h, w = 15, 11
    x = noise(h * w * c, 11, 1.0)
    wt = noise(k * k * c, 13, 0.5)
    b = noise(c, 17, 0.5)
    p = k // 2
    op = window(Op("dwconv", x=0, y=1, ic=c, oc=c, w=(0, wt.size), b=(wt.size, c)), (k, k), s, p, p)
    got = oracle_mod.Oracle(single(op, (h, w, c), np.concatenate([wt, b]))).run(x)[0]
    X = x.reshape(h, w, c).astype(np.float64)
    Wt = wt.reshape(k, k, c).astype(np.float64)
    xp = np.zeros((h + 2 * p, w + 2 * p, c))
    xp[p:p + h, p:p + w] = X
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    want = np.zeros((oh, ow, c)) + b
    for ky in range(k):
        for kx in range(k):
            want += xp[ky:ky + s * (oh - 1) + 1:s, kx:kx + s * (ow - 1) + 1:s] * Wt[ky, kx]
    assert max_gap(got, want.reshape(-1).astype(np.float32)) < 1e-5


def test_layernorm_and_attention_match_float64(oracle_mod):
    t, c, heads = 23, 24, 4
    hd = c // heads
    x = noise(t * 3 * c, 21, 1.5)
    scale = np.float32(hd ** -0.5)
    att = Op("attention", x=0, y=1, ic=3 * c, oc=c, n2=heads, w=(0, 1))
    got = oracle_mod.Oracle(single(att, (1, t, 3 * c), np.float32([scale]))).run(x)[0].reshape(t, c)
    X = x.reshape(t, 3, heads, hd).astype(np.float64)
    for h in range(heads):
        q, k, v = X[:, 0, h] * float(scale), X[:, 1, h], X[:, 2, h]
        s = q @ k.T
        p = np.exp(s - s.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        assert np.max(np.abs(got[:, h * hd:(h + 1) * hd] - p @ v)) < 1e-5
    gamma, beta = noise(c, 3, 1.0) + 1, noise(c, 4, 0.5)
    ln = Op("layernorm", x=0, y=1, ic=c, oc=c, w=(0, 2 * c + 1))
    xs = noise(t * c, 9, 3.0)
    got = oracle_mod.Oracle(single(ln, (1, t, c), np.concatenate([gamma, beta, np.float32([1e-6])]))).run(xs)[0]
    X = xs.reshape(t, c).astype(np.float64)
    m = X.mean(1, keepdims=True)
    want = (X - m) / np.sqrt(((X - m) ** 2).mean(1, keepdims=True) + 1e-6) * gamma + beta
    assert max_gap(got, want.reshape(-1).astype(np.float32)) < 1e-5


# plan.rs:959-995 (malformed_files_refused) and :1008-1036 (malformed_operations_refused)
def pointwise_op():
    return Op("conv", x=0, y=1, ic=4, oc=4, kh=1, kw=1, sh=1, sw=1, w=(0, 16), b=(16, 4))


def good_file(ops=None, weights=20):
    return encode((0, 2, 2, 4), 2, [1], ops or [pointwise_op()], np.arange(weights, dtype=np.float32))


def malformed_files():
    good = good_file()
    header = 8 + 4 * 8
    cases = [("not a plan", b"not a plan at all, really"), ("truncated description", good[:header + 10]),
             ("no weights", good[:128]), ("truncated weights", good[:-2])]

    def edit(what, at, v):
        b = bytearray(good)
        b[at:at + 4] = struct.pack("<I", v)
        cases.append((what, bytes(b)))

    def field(k):
        return header + 4 * k

    edit("unknown kind", field(0), 99)
    edit("unknown activation", field(1), 99)
    edit("missing buffer", field(4), 7)
    edit("weights past the end", field(16), 8)
    edit("weights the shape contradicts", field(17), 12)
    edit("a zero-sized image", 8 + 4, 0)
    edit("no buffers", 8 + 16, 0)
    edit("an operation count past the file", 8 + 24, 0xFFFFFFFF)
    nan = bytearray(good)
    nan[-4:] = struct.pack("<f", float("nan"))
    cases.append(("a weight that is not a number", bytes(nan)))

    def op_edit(what, f):
        op = pointwise_op()
        f(op)
        cases.append((what, good_file([op], 80)))

    op_edit("zero input channels", lambda op: setattr(op, "ic", 0))
    op_edit("zero stride", lambda op: setattr(op, "sw", 0))
    op_edit("padding past the window limit", lambda op: setattr(op, "pl", 1 << 20))
    op_edit("bias of the wrong length", lambda op: setattr(op, "b", (16, 3)))
    op_edit("output over its input", lambda op: setattr(op, "y", 0))

    def mean_relu(op):
        op.kind, op.fused, op.w, op.b = "mean", "relu", (0, 0), (0, 0)
    op_edit("folded activation on a mean", mean_relu)
    op_edit("unused weights on an addition", lambda op: setattr(op, "kind", "add"))
    op_edit("second input on a pointwise layer", lambda op: setattr(op, "n2", 4))

    def overlap(op):
        op.kind, op.kh, op.kw, op.sh, op.sw, op.w, op.b = "convtranspose", 2, 2, 1, 1, (0, 64), (0, 0)
    op_edit("overlapping transposed windows", overlap)
    return cases


@pytest.mark.parametrize("what,data", malformed_files(), ids=[c[0] for c in malformed_files()])
def test_malformed_plans_refused(oracle_mod, what, data):
    with pytest.raises(oracle_mod.OracleError):
        oracle_mod.Oracle(data)


def test_good_plan_loads_and_subnormals_flush(oracle_mod):
    o = oracle_mod.Oracle(good_file())
    assert o.output_len(0) == 16
    # plan.rs:997-1006 (subnormal_weights_load_as_zero): a subnormal last
    # bias loads, and acts as a zero.
    data = bytearray(good_file())
    data[-4:] = struct.pack("<I", 0x80000001)
    zero = bytearray(good_file())
    zero[-4:] = struct.pack("<f", 0.0)
    x = np.full(16, 1e-3, np.float32)
    out = oracle_mod.Oracle(bytes(data)).run(x)[0]
    assert np.array_equal(out, oracle_mod.Oracle(bytes(zero)).run(x)[0])


# plan.rs:1038-1059 (sizes_follow_the_input)
def test_sizes_follow_the_input(oracle_mod):
    stem = window(Op("conv", x=0, y=1, ic=3, oc=4, w=(0, 108), b=(108, 4)), (3, 3), 2, 1, 1)
    up = Op("upsample", x=1, y=0, ic=4, oc=4, sh=2, sw=2)
    o = oracle_mod.Oracle(encode((0, 8, 8, 3), 2, [0], [stem, up], np.full(112, 0.5, np.float32)))
    o.set_size(6, 10)
    assert o.output_len(0) == 240
    with pytest.raises(oracle_mod.OracleError):
        o.set_size(1 << 20, 1 << 20)
    assert o.input_len == 6 * 10 * 3


def ramp_run(o):
    return o.run(synth.ramp_input(o.input_len))[0]


# mod.rs:1478-1494 (threads_match_one_thread)
@pytest.mark.parametrize("make", [lambda: synth.page_model_plan(64, 48), lambda: synth.page_model_plan(40, 8),
                                  lambda: synth.line_model_plan(1001)], ids=["page64x48", "page40x8", "line1001"])
def test_threads_match_one_thread(oracle_mod, make):
    o = oracle_mod.Oracle(make())
    want = o.run(synth.ramp_input(o.input_len), threads=1)[0]
    for threads in (2, 3, 8):
        got = o.run(synth.ramp_input(o.input_len), threads=threads)[0]
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# mod.rs:1496-1507 (page_size_matches_fresh_load)
def test_page_size_matches_fresh_load(oracle_mod):
    o = oracle_mod.Oracle(synth.page_model_plan(16, 16))
    for h, w in [(16, 24), (40, 8), (8, 36), (4, 4), (16, 16), (64, 48)]:
        o.set_size(h, w)
        assert o.input_len == h * w * 3 and o.output_len(0) == h * w
        fresh = oracle_mod.Oracle(synth.page_model_plan(h, w))
        assert np.array_equal(ramp_run(o).view(np.uint32), ramp_run(fresh).view(np.uint32))


# mod.rs:1509-1526 (bad_page_size_refused)
def test_bad_page_size_refused(oracle_mod):
    o = oracle_mod.Oracle(synth.page_model_plan(16, 16))
    before = ramp_run(o)
    for h, w in [(10, 16), (16, 22), (0, 16), (2 ** 64 - 1, 16), (1 << 20, 1 << 20)]:
        with pytest.raises(oracle_mod.OracleError):
            o.set_size(h, w)
        assert o.input_len == 16 * 16 * 3
        assert np.array_equal(ramp_run(o), before)


# mod.rs:1528-1554 (width_matches_fresh_load, bad_width_keeps_model_size)
def test_line_width_matches_fresh_load(oracle_mod):
    o = oracle_mod.Oracle(synth.line_model_plan(40))
    for width in [3, 40, 1001, 17, 3, 64]:
        o.set_size(2, width)
        t = ((width - 1) // 2 + 1 - 2) // 2 + 1
        assert o.output_len(0) == 2 * t
        fresh = oracle_mod.Oracle(synth.line_model_plan(width))
        assert np.array_equal(ramp_run(o).view(np.uint32), ramp_run(fresh).view(np.uint32))
    o.set_size(2, 40)
    before = ramp_run(o)
    for width in [2, 1, 0, 2 ** 64 - 1, 1 << 40]:
        with pytest.raises(oracle_mod.OracleError):
            o.set_size(2, width)
        assert np.array_equal(ramp_run(o), before)


def test_timed_path_gives_the_plain_loops_bits(oracle_mod):
    """The register-tiled AVX2+FMA loops bench.py times (dense convolutions
    and depthwise layers in 6-pixel tiles, the CTC head's logits six time
    steps at a time) keep every output's chain of fused multiply-adds in the
    plain loops' order: the same bits on the detector, the recogniser (argmax
    and logits heads) and the fused benchmark layer, at sizes with border and
    interior tiles and widths that are not multiples of six."""
    from ppocr_native_b200 import synth

    rng = np.random.default_rng(21)
    cases = [(synth.det_plan(seed=5, std=None, size=(160, 128)), (160, 128)),
             (synth.det_plan(seed=5, std=None, size=(160, 128)), (96, 224)),
             (synth.rec_plan(seed=3, std=None, vocab=700), (48, 328)),
             (synth.rec_plan(seed=3, std=None, vocab=300, logits=True), (48, 100)),
             (synth.fused_layer_plan(seed=0, h=23, w=31), (23, 31))]
    # dense convolutions whose widths reach the 16- and 8-column tiles (the
    # networks' widths are all multiples of 24), bias first and last, one
    # over a second input, one strided
    h, w, c1, c2 = 13, 29, 5, 7
    for oc, fused, two, stride in [(40, "swish", False, 1), (32, "relu", True, 1), (16, "none", False, 2)]:
        taps, ch = 9, c1 + (c2 if two else 0)
        first = window(Op("conv", x=0, y=1, ic=c1, oc=c2, w=(0, c1 * c2), b=(c1 * c2, c2)), (1, 1), 1, 0, 0)
        at = c1 * c2 + c2
        conv = window(Op("conv", x=0, y=2, ic=c1, oc=oc, fused=fused, x2=1 if two else 0, n2=c2 if two else 0),
                      (3, 3), stride, 1, 1)
        conv.w, conv.b = (at, taps * ch * oc), (at + taps * ch * oc, oc)
        weights = noise(at + taps * ch * oc + oc, 9 + oc, 0.4)
        cases.append((encode((0, h, w, c1), 3, [2], [first, conv], weights), (h, w)))
    for oc, fused in [(1, "sigmoid"), (4, "relu"), (8, "swish")]:  # 4-, 16- and 32-column blocks
        w = noise(5 * 4 * oc, 3, 0.5)
        bias = noise(4 * oc, 4, 0.5)
        op = Op("convtranspose", x=0, y=1, ic=5, oc=oc, kh=2, kw=2, sh=2, sw=2, fused=fused,
                w=(0, w.size), b=(w.size, bias.size))
        cases.append((single(op, (3, 7, 5), np.concatenate([w, bias])), (3, 7)))
    try:
        for plan, (h, w) in cases:
            p = oracle_mod.Oracle(plan)
            p.set_size(h, w)
            x = rng.standard_normal(p.input_len).astype(np.float32)
            oracle_mod.set_fast(False)
            plain = p.run(x)[0]
            oracle_mod.set_fast(True)
            fast = p.run(x)[0]
            assert np.array_equal(plain.view(np.uint32), fast.view(np.uint32))
    finally:
        oracle_mod.set_fast(False)
