"""PPOCRPL1 plan files: the operation records and a numpy writer.

A plan is the reference engine's model format (ppocr-native
`src/engine/plan.rs:9-28`): the magic ``PPOCRPL1``, seven little-endian u32
(input buffer, input height, width, channels, buffer count, output count,
operation count), one u32 per output, twenty u32 per operation, zero padding
to a 64-byte boundary, then the weights as f32 to the end of the file.

This module writes such files for synthetic networks and the test models
(the same layout as the reference's test writer, `plan.rs:848-898`, and its
exporter, `tools/export_ocr.py:839-870`). Reading and checking a plan is the
CUDA library's job (`csrc/plan.cpp`); ``describe`` here only decodes records
for tests.
"""

from __future__ import annotations

import dataclasses
import struct

import numpy as np

MAGIC = b"PPOCRPL1"
OP_FIELDS = 20

# Operation kinds by file code, `plan.rs:130-146`.
KINDS = [
    "conv",
    "dwconv",
    "add",
    "maxpool",
    "avgpool",
    "channelmul",
    "concatc",
    "layernorm",
    "attention",
    "mean",
    "ctchead",
    "ctcargmax",
    "upsample",
    "upsampleadd",
    "convtranspose",
]
# Folded activations by file code, `plan.rs:167-175`. Code 7, hardswish, is an
# extension of this library: x * clamp(x * 0x3e2aaaad + 0.5, 0, 1). The
# reference refuses it (`plan.rs:776-778`); only the single-layer benchmark
# plan uses it.
FUSED = [
    "none",
    "relu",
    "sigmoid",
    "gelu",
    "swish",
    "hardsigmoid",
    "hardsigmoidfifth",
    "hardswish",
]
KIND = {k: i for i, k in enumerate(KINDS)}
ACT = {a: i for i, a in enumerate(FUSED)}


@dataclasses.dataclass
class Op:
    """One operation record, in the field order of `plan.rs:15-18`."""

    kind: str
    x: int
    y: int
    ic: int
    oc: int
    fused: str = "none"
    x2: int = 0
    kh: int = 0
    kw: int = 0
    sh: int = 0
    sw: int = 0
    pt: int = 0
    pb: int = 0
    pl: int = 0
    pr: int = 0
    n2: int = 0
    w: tuple[int, int] = (0, 0)
    b: tuple[int, int] = (0, 0)

    def fields(self) -> list[int]:
        return [
            KIND[self.kind],
            ACT[self.fused],
            self.x,
            self.x2,
            self.y,
            self.ic,
            self.oc,
            self.kh,
            self.kw,
            self.sh,
            self.sw,
            self.pt,
            self.pb,
            self.pl,
            self.pr,
            self.n2,
            self.w[0],
            self.w[1],
            self.b[0],
            self.b[1],
        ]


def window(op: Op, k: tuple[int, int], s: int, before: int, after: int) -> Op:
    """Kernel, stride and padding of a windowed op (as the reference tests'
    `window`, `src/engine/mod.rs:1344-1347`)."""
    op.kh, op.kw = k
    op.sh = op.sw = s
    op.pt = op.pl = before
    op.pb = op.pr = after
    return op


def encode(
    input: tuple[int, int, int, int],
    buffers: int,
    outputs: list[int],
    ops: list[Op],
    weights: np.ndarray,
) -> bytes:
    """A plan file: `input` is (buffer, height, width, channels)."""
    slot, h, w, c = input
    words = [slot, h, w, c, buffers, len(outputs), len(ops), *outputs]
    for op in ops:
        words.extend(op.fields())
    head = MAGIC + struct.pack(f"<{len(words)}I", *words)
    head += b"\0" * (-len(head) % 64)
    return head + np.ascontiguousarray(weights, dtype="<f4").tobytes()


def describe(data: bytes) -> dict:
    """Decode a plan's records without checking them (test helper)."""
    if data[:8] != MAGIC:
        raise ValueError("not a plan")
    head = struct.unpack_from("<7I", data, 8)
    slot, h, w, c, buffers, nout, nops = head
    at = 8 + 28
    outputs = list(struct.unpack_from(f"<{nout}I", data, at))
    at += 4 * nout
    ops = []
    for _ in range(nops):
        f = struct.unpack_from(f"<{OP_FIELDS}I", data, at)
        at += 4 * OP_FIELDS
        ops.append(
            Op(
                kind=KINDS[f[0]],
                fused=FUSED[f[1]],
                x=f[2],
                x2=f[3],
                y=f[4],
                ic=f[5],
                oc=f[6],
                kh=f[7],
                kw=f[8],
                sh=f[9],
                sw=f[10],
                pt=f[11],
                pb=f[12],
                pl=f[13],
                pr=f[14],
                n2=f[15],
                w=(f[16], f[17]),
                b=(f[18], f[19]),
            )
        )
    start = -(-at // 64) * 64
    weights = np.frombuffer(data[start:], dtype="<f4")
    return {
        "input": (slot, h, w, c),
        "buffers": buffers,
        "outputs": outputs,
        "ops": ops,
        "weights": weights,
    }


class Builder:
    """Appends operations and their weight blocks; buffers are numbered as
    they are made. Weight blocks are laid out as `tools/export_ocr.py` packs
    them: dense conv `[kh][kw][ic+n2][oc]` (:316), depthwise `[kh][kw][c]`
    (:312), transposed conv `[ic][kh][kw][oc]` with the bias tiled kh*kw
    times (:517-518), LayerNorm `[gamma, beta, eps]` (:551), attention
    `[scale]` (:819), CTC head `[cols/16][ic][16]` panels with -1e30 bias
    past the vocabulary (:719-724)."""

    def __init__(self, h: int, w: int, c: int, rng: np.random.Generator, std: float | None = 0.02):
        """`std` None draws each weight block ~N(0, 4/fan_in) and each bias
        ~N(0, 0.02) instead, which keeps activations O(1) through the depth
        (busy maps for parity tests); a number draws every block ~N(0, std)."""
        self.input = (0, h, w, c)
        self.buffers = 1
        self.ops: list[Op] = []
        self.blob: list[np.ndarray] = []
        self.at = 0
        self.rng = rng
        self.std = std
        self.channels = {0: c}

    # -- weights -----------------------------------------------------------
    def put(self, values: np.ndarray) -> tuple[int, int]:
        v = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
        block = (self.at, v.size)
        self.blob.append(v)
        self.at += v.size
        return block

    def normal(self, *shape: int, std: float | None = None, fan_in: int = 1) -> np.ndarray:
        if std is None:
            std = self.std if self.std is not None else float(np.sqrt(3.0 / fan_in))
        return self.rng.normal(0.0, std, size=shape).astype(np.float32)

    def new(self, c: int) -> int:
        slot = self.buffers
        self.buffers += 1
        self.channels[slot] = c
        return slot

    # -- layers ------------------------------------------------------------
    def conv(self, x, oc, k=1, s=1, pad=None, act="none", x2=None, n2=0, std=None, stride_hw=None) -> int:
        ic = self.channels[x]
        kh, kw = (k, k) if isinstance(k, int) else k
        pad = (kh // 2 if pad is None else pad)
        y = self.new(oc)
        op = Op("conv", x=x, y=y, ic=ic, oc=oc, fused=act, kh=kh, kw=kw, sh=s, sw=s,
                pt=pad, pb=pad, pl=pad, pr=pad)
        if stride_hw is not None:
            op.sh, op.sw = stride_hw
        if x2 is not None:
            op.x2, op.n2 = x2, n2 or self.channels[x2]
        op.w = self.put(self.normal(kh, kw, ic + op.n2, oc, std=std, fan_in=kh * kw * (ic + op.n2)))
        op.b = self.put(self.normal(oc, std=std, fan_in=10000))
        self.ops.append(op)
        return y

    def dw(self, x, k=3, s=1, act="none", std=None) -> int:
        c = self.channels[x]
        y = self.new(c)
        op = Op("dwconv", x=x, y=y, ic=c, oc=c, fused=act, kh=k, kw=k, sh=s, sw=s,
                pt=k // 2, pb=k // 2, pl=k // 2, pr=k // 2)
        op.w = self.put(self.normal(k, k, c, std=std, fan_in=k * k))
        op.b = self.put(self.normal(c, std=std, fan_in=10000))
        self.ops.append(op)
        return y

    def simple(self, kind, x, x2=None, oc=None, act="none", **kw) -> int:
        ic = self.channels[x]
        oc = ic if oc is None else oc
        y = self.new(oc)
        op = Op(kind, x=x, y=y, ic=ic, oc=oc, fused=act, **kw)
        if x2 is not None:
            op.x2 = x2
        self.ops.append(op)
        return y

    def mean(self, x) -> int:
        return self.simple("mean", x)

    def channelmul(self, x, gate) -> int:
        return self.simple("channelmul", x, x2=gate)

    def add(self, a, b, act="none") -> int:
        return self.simple("add", a, x2=b, act=act)

    def upsample(self, x, f) -> int:
        return self.simple("upsample", x, sh=f, sw=f)

    def upsampleadd(self, x, x2, f) -> int:
        return self.simple("upsampleadd", x, x2=x2, sh=f, sw=f)

    def concat(self, a, b) -> int:
        n2 = self.channels[b]
        return self.simple("concatc", a, x2=b, oc=self.channels[a] + n2, n2=n2)

    def layernorm(self, x, eps=1e-6) -> int:
        c = self.channels[x]
        y = self.new(c)
        gamma = 1.0 + self.normal(c, fan_in=10000)
        beta = self.normal(c, fan_in=10000)
        op = Op("layernorm", x=x, y=y, ic=c, oc=c)
        op.w = self.put(np.concatenate([gamma, beta, np.float32([eps])]))
        self.ops.append(op)
        return y

    def attention(self, qkv, heads, scale) -> int:
        ic = self.channels[qkv]
        c = ic // 3
        y = self.new(c)
        op = Op("attention", x=qkv, y=y, ic=ic, oc=c, n2=heads)
        op.w = self.put(np.float32([scale]))
        self.ops.append(op)
        return y

    def ctc(self, x, vocab, argmax=True, std=None) -> int:
        ci = self.channels[x]
        cols = -(-vocab // 16) * 16
        logical = self.normal(ci, vocab, std=std, fan_in=ci)
        panels = np.zeros((cols // 16, ci, 16), np.float32)
        full = np.zeros((ci, cols), np.float32)
        full[:, :vocab] = logical
        panels[:] = full.reshape(ci, cols // 16, 16).transpose(1, 0, 2)
        bias = np.full(cols, -1e30, np.float32)
        bias[:vocab] = self.normal(vocab, std=std, fan_in=10000)
        oc = 2 if argmax else vocab
        y = self.new(oc)
        op = Op("ctcargmax" if argmax else "ctchead", x=x, y=y, ic=ci, oc=oc,
                n2=vocab if argmax else 0)
        op.w = self.put(panels)
        op.b = self.put(bias)
        self.ops.append(op)
        return y

    def convtranspose(self, x, oc, k=2, act="none", std=None) -> int:
        ic = self.channels[x]
        y = self.new(oc)
        op = Op("convtranspose", x=x, y=y, ic=ic, oc=oc, fused=act, kh=k, kw=k, sh=k, sw=k)
        op.w = self.put(self.normal(ic, k, k, oc, std=std, fan_in=ic))
        op.b = self.put(np.tile(self.normal(oc, std=std, fan_in=10000), k * k))
        self.ops.append(op)
        return y

    def avgpool(self, x, k, s) -> int:
        kh, kw = k
        sh, sw = s
        return self.simple("avgpool", x, kh=kh, kw=kw, sh=sh, sw=sw)

    def maxpool(self, x, k=2) -> int:
        return self.simple("maxpool", x, kh=k, kw=k, sh=1, sw=1, pb=k - 1, pr=k - 1)

    def build(self, outputs: list[int]) -> bytes:
        weights = np.concatenate(self.blob) if self.blob else np.zeros(0, np.float32)
        return encode(self.input, self.buffers, outputs, self.ops, weights)


def shapes(data: bytes, h: int, w: int) -> list[Op]:
    """Every op of a plan with its sizes at an input of h x w, as
    `plan.rs:414-494` derives them (no checks: for cost accounting). Each
    returned op carries ih, iw, oh, ow attributes."""
    d = describe(data)
    slot, _, _, c = d["input"]
    ops = d["ops"]
    made: dict[int, tuple[int, int, int]] = {slot: (h, w, c)}
    for op in ops:
        ih, iw, _ = made[op.x]
        if op.kind in ("conv", "dwconv", "maxpool", "avgpool"):
            oh = (ih + op.pt + op.pb - op.kh) // op.sh + 1
            ow = (iw + op.pl + op.pr - op.kw) // op.sw + 1
        elif op.kind in ("upsample", "upsampleadd"):
            oh, ow = ih * op.sh, iw * op.sw
        elif op.kind == "convtranspose":
            oh, ow = ih * op.kh, iw * op.kw
        elif op.kind == "mean":
            oh, ow = 1, 1
        else:
            oh, ow = ih, iw
        op.ih, op.iw, op.oh, op.ow = ih, iw, oh, ow
        made[op.y] = (oh, ow, op.oc)
    return ops


def macs(op: Op) -> int:
    """Multiply-adds of one op, as the reference's profiler counts them
    (`examples/plan.rs:140-152`)."""
    spatial = op.oh * op.ow
    if op.kind == "conv":
        return op.kh * op.kw * (op.ic + op.n2) * op.oc * spatial
    if op.kind == "dwconv":
        return op.kh * op.kw * op.oc * spatial
    if op.kind == "attention":
        return 2 * op.iw * op.iw * op.oc
    if op.kind == "ctchead":
        return op.iw * op.ic * op.oc
    if op.kind == "ctcargmax":
        return op.iw * op.ic * -(-op.n2 // 16) * 16
    if op.kind == "convtranspose":
        return op.kh * op.kw * op.ic * op.oc * op.ih * op.iw
    return 0


def flops(data: bytes, h: int, w: int) -> int:
    """Floating-point operations (2 per multiply-add) of a whole plan."""
    return 2 * sum(macs(op) for op in shapes(data, h, w))
