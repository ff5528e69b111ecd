"""Synthetic PP-OCRv6-shaped plans: the single fused layer, the detector and
the recogniser, plus the reference engine's own test miniatures.

No trained weights exist here (the reference exports its plans from
RapidOCR's ONNX models at package-build time, `pkgbuild/PKGBUILD:49-56`), so
the networks are random-init with the architecture the reference's hints
pin down:

- det: an LCNet-style backbone at PP-LCNet x0.75 widths with the det stem of
  24 channels (`src/engine/kernels/dense.rs:416-419`), depthwise 3x3 then 5x5
  in the last seven blocks, squeeze-and-excite in the last two; an RSE-FPN
  neck at 96 channels with slope-0.2 hard sigmoids (`layers.rs:43`), the
  top-down upsample-adds, a 3x3 96->24 RSE per level; a DB head whose 3x3
  conv reads the four levels upsampled in place (`schedule.rs:902-954`) and
  two chained 2x2 transposed convs, relu then sigmoid (`schedule.rs:828-853`).
- rec: stem 3x3 s2 3->48 (`dense.rs:416-419`), depthwise-separable blocks to
  6 x W/8 x 384, an average pool over the height, 1x1 to 120, two SVTR
  blocks (LayerNorm, qkv 120->360, 8-head attention of head size 15
  (`tools/export_ocr.py:654`), projection, MLP 120->240->120, residual adds),
  a final LayerNorm and the CTC argmax over 18 710 classes
  (`layers.rs:699-700`, `tests/parity.rs:218`).

Only fused codes 0-6 appear in det and rec, so both stay plans the
reference itself would load; swish stands where LCNet has hardswish.
"""

from __future__ import annotations

import numpy as np

from .plan import Builder, Op, encode, window

VOCAB = 18710  # blank + 18 707 characters + space, tests/parity.rs:218
DET_SIZE = (960, 736)
PAGE_DET_SIZE = (1984, 1536)
REC_HEIGHT = 48


def fused_layer_plan(seed: int = 0, h: int = 240, w: int = 240, c: int = 96, oc: int = 192) -> bytes:
    """Benchmark config 1: depthwise 5x5 s1 pad 2 + hardswish feeding a
    pointwise 96->192 + bias + hardswish. Weights ~N(0, 0.05), biases
    ~U(-0.1, 0.1), numpy default_rng(seed)."""
    rng = np.random.default_rng(seed)
    dw_w = rng.normal(0, 0.05, size=(5, 5, c)).astype(np.float32)
    dw_b = rng.uniform(-0.1, 0.1, size=c).astype(np.float32)
    pw_w = rng.normal(0, 0.05, size=(c, oc)).astype(np.float32)
    pw_b = rng.uniform(-0.1, 0.1, size=oc).astype(np.float32)
    at = 0
    blocks = []
    for v in (dw_w, dw_b, pw_w, pw_b):
        blocks.append((at, v.size))
        at += v.size
    dw = window(Op("dwconv", x=0, y=1, ic=c, oc=c, fused="hardswish"), (5, 5), 1, 2, 2)
    dw.w, dw.b = blocks[0], blocks[1]
    pw = window(Op("conv", x=1, y=2, ic=c, oc=oc, fused="hardswish"), (1, 1), 1, 0, 0)
    pw.w, pw.b = blocks[2], blocks[3]
    weights = np.concatenate([v.reshape(-1) for v in (dw_w, dw_b, pw_w, pw_b)])
    return encode((0, h, w, c), 3, [2], [dw, pw], weights)


def _block(b: Builder, x: int, oc: int, k: int, s: int, se: bool) -> int:
    d = b.dw(x, k=k, s=s, act="swish")
    if se:
        c = b.channels[d]
        m = b.mean(d)
        g = b.conv(m, c // 4, act="relu")
        g = b.conv(g, c, act="hardsigmoid")
        d = b.channelmul(d, g)
    return b.conv(d, oc, act="swish")


def _rse(b: Builder, x: int, oc: int, k: int) -> int:
    """RSE layer: conv, then x + x * SE(x) with the slope-0.2 hard sigmoid."""
    y = b.conv(x, oc, k=k)
    m = b.mean(y)
    g = b.conv(m, oc // 4, act="relu")
    g = b.conv(g, oc, act="hardsigmoidfifth")
    gated = b.channelmul(y, g)
    return b.add(y, gated)


def det_plan(seed: int = 0, std: float | None = 0.02, size: tuple[int, int] = DET_SIZE) -> bytes:
    """Benchmark config 2's detector; input HWC f32, output the probability
    map. `std` None scales each block by its fan-in (see `Builder`)."""
    b = Builder(size[0], size[1], 3, np.random.default_rng(seed), std)
    x = b.conv(0, 24, k=3, s=2, act="swish")  # 1/2
    x = _block(b, x, 24, 3, 1, False)
    x = _block(b, x, 48, 3, 2, False)  # 1/4
    c2 = _block(b, x, 48, 3, 1, False)
    x = _block(b, c2, 96, 3, 2, False)  # 1/8
    c3 = _block(b, x, 96, 3, 1, False)
    x = _block(b, c3, 192, 3, 2, False)  # 1/16
    for _ in range(5):
        x = _block(b, x, 192, 5, 1, False)
    c4 = x
    x = _block(b, c4, 384, 5, 2, True)  # 1/32
    c5 = _block(b, x, 384, 5, 1, True)
    in2, in3, in4, in5 = (_rse(b, c, 96, 1) for c in (c2, c3, c4, c5))
    out4 = b.upsampleadd(in5, in4, 2)
    out3 = b.upsampleadd(out4, in3, 2)
    out2 = b.upsampleadd(out3, in2, 2)
    p5, p4, p3, p2 = (_rse(b, t, 24, 3) for t in (in5, out4, out3, out2))
    u5 = b.upsample(p5, 8)
    u4 = b.upsample(p4, 4)
    u3 = b.upsample(p3, 2)
    cat = b.concat(b.concat(u5, u4), u3)
    h = b.conv(cat, 24, k=3, act="relu", x2=p2)
    h = b.convtranspose(h, 24, 2, act="relu")
    # In fan-in mode the last layer is damped so the probabilities spread over
    # (0, 1) instead of saturating.
    prob = b.convtranspose(h, 1, 2, act="sigmoid", std=None if std is not None else 0.0004)
    return b.build([prob])


def rec_plan(seed: int = 0, std: float | None = 0.02, width: int = 320, argmax: bool = True,
             vocab: int = VOCAB, logits: bool = False) -> bytes:
    """Benchmark config 3's recogniser; input HWC 48 x W x 3, output
    `[T][2]` = (best class as f32, 1 / sum exp) with T = ceil(W / 8). With
    `logits` the network ends in the head's logits instead: a 1x1 conv
    120 -> vocab, output `[T][vocab]` (the tap the logits parity test reads)."""
    b = Builder(REC_HEIGHT, width, 3, np.random.default_rng(seed), std)
    x = b.conv(0, 48, k=3, s=2, act="swish")  # 24 x W/2
    x = _block(b, x, 96, 3, 1, False)
    x = _block(b, x, 192, 3, 2, False)  # 12 x W/4
    x = _block(b, x, 192, 3, 1, False)
    x = _block(b, x, 384, 3, 2, False)  # 6 x W/8
    x = _block(b, x, 384, 5, 1, False)
    x = _block(b, x, 384, 5, 1, True)
    x = b.avgpool(x, (6, 1), (6, 1))  # 1 x W/8
    x = b.conv(x, 120, act="swish")
    for _ in range(2):
        n = b.layernorm(x)
        qkv = b.conv(n, 360)
        a = b.attention(qkv, 8, 15 ** -0.5)
        x = b.add(x, b.conv(a, 120))
        n = b.layernorm(x)
        m = b.conv(b.conv(n, 240, act="gelu"), 120)
        x = b.add(x, m)
    x = b.layernorm(x)
    out = b.conv(x, vocab) if logits else b.ctc(x, vocab, argmax=argmax)
    return b.build([out])


# -- the reference engine's test miniatures (src/engine/mod.rs:1327-1468) ---

def _ramp(n: int, scale: float) -> np.ndarray:
    i = np.arange(n, dtype=np.float32)
    return (np.sin(i * np.float32(0.37)) * np.float32(scale)).astype(np.float32)


def _weigh(op: Op, at: int) -> int:
    taps = op.kh * op.kw
    if op.kind == "dwconv":
        w, bl = taps * op.oc, op.oc
    elif op.kind == "convtranspose":
        w, bl = taps * op.ic * op.oc, taps * op.oc
    else:
        w, bl = taps * (op.ic + op.n2) * op.oc, op.oc
    op.w, op.b = (at, w), (at + w, bl)
    return w + bl


def line_model_plan(stored: int) -> bytes:
    """A recogniser-shaped model with every width rule: padded stride-2 stem,
    right-padded max pool, SE gate from a mean, width-halving average pool,
    attention and the CTC argmax (`src/engine/mod.rs:1374-1413`)."""
    at = 0
    stem = window(Op("conv", 0, 1, 3, 4, fused="relu"), (3, 3), 2, 1, 1)
    at += _weigh(stem, at)
    pool = Op("maxpool", 1, 2, 4, 4, kh=1, kw=2, sh=1, sw=1, pr=1)
    mean = Op("mean", 2, 1, 4, 4)
    gate = window(Op("conv", 1, 3, 4, 4, fused="hardsigmoid"), (1, 1), 1, 0, 0)
    at += _weigh(gate, at)
    scale = Op("channelmul", 2, 1, 4, 4, x2=3)
    average = Op("avgpool", 1, 2, 4, 4, kh=1, kw=2, sh=1, sw=2)
    qkv = window(Op("conv", 2, 1, 4, 12, fused="gelu"), (1, 1), 1, 0, 0)
    at += _weigh(qkv, at)
    attention = Op("attention", 1, 2, 12, 4, n2=2, w=(at, 1))
    at += 1
    head = Op("ctcargmax", 2, 3, 4, 2, n2=37, w=(at, 4 * 48), b=(at + 4 * 48, 48))
    at += 5 * 48
    values = _ramp(at, 0.5)
    values[at - 48 + 37:] = np.float32(-1e30)
    ops = [stem, pool, mean, gate, scale, average, qkv, attention, head]
    return encode((0, 2, stored, 3), 4, [3], ops, values)


def page_model_plan(h: int, w: int) -> bytes:
    """A detector-shaped model with every size rule along both axes
    (`src/engine/mod.rs:1415-1468`): padded stride-2 stem, max pool, a 2x2
    conv padded below and right, 7x7 depthwise, a gate from a mean, a
    stride-2 conv upsampled back onto the pool, a two-input conv, a channel
    concatenation and a transposed conv to full size."""
    at = 0
    ops: list[Op] = []

    def layer(kind, xy, ioc, k, s, pads, fused):
        nonlocal at
        op = window(Op(kind, xy[0], xy[1], ioc[0], ioc[1], fused=fused), (k, k), s, *pads)
        if kind in ("conv", "dwconv"):
            at += _weigh(op, at)
        ops.append(op)

    layer("conv", (0, 1), (3, 8), 3, 2, (1, 1), "relu")
    layer("maxpool", (1, 2), (8, 8), 2, 1, (0, 1), "none")
    layer("conv", (1, 3), (8, 8), 2, 1, (0, 1), "gelu")
    layer("dwconv", (3, 4), (8, 8), 7, 1, (3, 3), "none")
    layer("mean", (4, 5), (8, 8), 0, 0, (0, 0), "none")
    layer("conv", (5, 6), (8, 8), 1, 1, (0, 0), "hardsigmoidfifth")
    layer("channelmul", (4, 5), (8, 8), 0, 0, (0, 0), "none")
    layer("conv", (5, 4), (8, 8), 3, 2, (1, 1), "swish")
    layer("upsampleadd", (4, 6), (8, 8), 1, 2, (0, 0), "none")
    ops[6].x2 = 6
    ops[8].x2 = 2
    two = window(Op("conv", 6, 4, 8, 8), (3, 3), 1, 1, 1)
    two.x2, two.n2 = 3, 8
    at += _weigh(two, at)
    concat = Op("concatc", 4, 6, 8, 16, x2=5, n2=8)
    out = Op("convtranspose", 6, 1, 16, 1, kh=2, kw=2, sh=2, sw=2, fused="sigmoid")
    at += _weigh(out, at)
    ops.extend([two, concat, out])
    return encode((0, h, w, 3), 7, [1], ops, _ramp(at, 0.4))


def ramp_input(n: int, step: float = 0.013) -> np.ndarray:
    """The reference tests' input fill `cos(i * 0.013)` (`mod.rs:1470-1476`)."""
    return np.cos(np.arange(n, dtype=np.float32) * np.float32(step)).astype(np.float32)


def stripes(h: int, w: int, c: int = 3, phase: int = 0) -> np.ndarray:
    """The reference GPU tests' input `sin(((i + phase) % 977) * 0.37) * 2`
    (`tests/gpu.rs:18-22`)."""
    i = np.arange(h * w * c, dtype=np.int64)
    return (np.sin(((i + phase) % 977).astype(np.float32) * np.float32(0.37)) * 2).astype(np.float32)


def darkness_det_plan(size: tuple[int, int] = (480, 640), blur: int = 7, gain: float = 3.0) -> bytes:
    """A detector-shaped plan with set (not random) weights whose map marks
    dark ink: a depthwise blur of `blur` x `blur` over the normalized page,
    then a 1x1 conv 3 -> 1 of weight -gain/3 per channel and a sigmoid, so
    dark glyph rows with small gaps become blobs of probability near 1 on a
    near-0 background. It gives the page reader real text boxes to find
    (a random-init detector maps a page to a near-constant 0.5); it is a
    test input, not a model."""
    k = blur
    b = Builder(size[0], size[1], 3, np.random.default_rng(0), 0.0)
    d = b.new(3)
    op = Op("dwconv", x=0, y=d, ic=3, oc=3, fused="none", kh=k, kw=k, sh=1, sw=1,
            pt=k // 2, pb=k // 2, pl=k // 2, pr=k // 2)
    op.w = b.put(np.full((k, k, 3), 1.0 / (k * k), np.float32))
    op.b = b.put(np.zeros(3, np.float32))
    b.ops.append(op)
    y = b.new(1)
    pw = Op("conv", x=d, y=y, ic=3, oc=1, fused="sigmoid", kh=1, kw=1, sh=1, sw=1)
    pw.w = b.put(np.full((1, 1, 3, 1), -gain / 3.0, np.float32))
    pw.b = b.put(np.zeros(1, np.float32))
    b.ops.append(pw)
    return encode(b.input, b.buffers, [y], b.ops, np.concatenate(b.blob))


def characters(vocab: int = VOCAB) -> str:
    """Dictionary metadata for a `vocab`-class recogniser: vocab - 2 lines
    (blank and space are added by the dictionary), distinct CJK code points
    from U+4E00 (characters.txt of the real model is 18 707 such lines)."""
    return "".join(chr(0x4E00 + i) + "\n" for i in range(vocab - 2))
