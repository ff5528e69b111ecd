// PPOCRPL1 parsing and checks, following ppocr-native `src/engine/plan.rs`.
#include "plan.hpp"

#include <cmath>
#include <cstdio>
#include <cstring>
#include <limits>

namespace ppocr {

namespace {

constexpr size_t OP_FIELDS = 20;                   // plan.rs:68
constexpr size_t MAX_SCRATCH_FLOATS = size_t(1) << 30;  // plan.rs:73
constexpr size_t MAX_WINDOW = size_t(1) << 16;     // plan.rs:77

std::string fmt(const char *f, size_t a = 0, size_t b = 0, size_t c = 0) {
    char buf[256];
    std::snprintf(buf, sizeof buf, f, a, b, c);
    return buf;
}

bool shape_len(size_t a, size_t b, size_t c, size_t &out) {
    if (!a || !b || !c) return false;
    if (a > std::numeric_limits<size_t>::max() / b) return false;
    size_t ab = a * b;
    if (ab > std::numeric_limits<size_t>::max() / c) return false;
    out = ab * c;
    return true;
}

bool window_len(size_t n, long before, long after, size_t k, size_t s, size_t &out) {
    if (before < 0 || after < 0 || s == 0) return false;
    size_t span = n + size_t(before) + size_t(after);
    if (span < k) return false;
    out = (span - k) / s + 1;
    return true;
}

}  // namespace

const char *kind_name(int kind) {
    static const char *names[] = {"conv", "dwconv", "add", "maxpool", "avgpool", "channelmul",
                                  "concatc", "layernorm", "attention", "mean", "ctchead",
                                  "ctcargmax", "upsample", "upsampleadd", "convtranspose"};
    return kind >= 0 && kind < K_COUNT ? names[kind] : "?";
}

bool Plan::produced(size_t before, size_t s, size_t &oh, size_t &ow, size_t &oc) const {
    for (size_t i = before; i-- > 0;)
        if (ops[i].y == s) {
            oh = ops[i].oh; ow = ops[i].ow; oc = ops[i].oc;
            return true;
        }
    if (s == slot) { oh = h; ow = w; oc = c; return true; }
    return false;
}

// plan.rs:414-494
bool Plan::derive_shapes(size_t height, size_t width, std::string &err) {
    h = height; w = width;
    for (size_t i = 0; i < ops.size(); i++) {
        size_t ih, iw, ic;
        if (!produced(i, ops[i].x, ih, iw, ic)) { err = fmt("op %zu reads a buffer nothing wrote", i); return false; }
        Op &op = ops[i];
        if (ic != op.ic) { err = fmt("op %zu reads a tensor of another shape", i); return false; }
        size_t oh = ih, ow = iw;
        switch (op.kind) {
        case K_CONV: case K_DWCONV: case K_MAXPOOL: case K_AVGPOOL:
            if (!window_len(ih, op.pt, op.pb, op.kh, op.sh, oh) || !window_len(iw, op.pl, op.pr, op.kw, op.sw, ow)) {
                err = fmt("op %zu has a window larger than its padded input", i);
                return false;
            }
            break;
        case K_UPSAMPLE: case K_UPSAMPLEADD:
            if ((op.sh && ih > std::numeric_limits<size_t>::max() / op.sh) ||
                (op.sw && iw > std::numeric_limits<size_t>::max() / op.sw)) {
                err = fmt("op %zu output size overflows", i);
                return false;
            }
            oh = ih * op.sh; ow = iw * op.sw;
            break;
        case K_CONVTRANSPOSE:
            if ((op.kh && ih > std::numeric_limits<size_t>::max() / op.kh) ||
                (op.kw && iw > std::numeric_limits<size_t>::max() / op.kw)) {
                err = fmt("op %zu output size overflows", i);
                return false;
            }
            oh = ih * op.kh; ow = iw * op.kw;
            break;
        case K_MEAN: oh = 1; ow = 1; break;
        default: break;
        }
        bool two = true;
        size_t wh = 0, ww = 0, wc = 0;
        switch (op.kind) {
        case K_ADD: case K_UPSAMPLEADD: wh = oh; ww = ow; wc = op.oc; break;
        case K_CONCATC: wh = oh; ww = ow; wc = op.n2; break;
        case K_CHANNELMUL: wh = 1; ww = 1; wc = op.oc; break;
        case K_CONV:
            if (op.n2 > 0) { wh = ih; ww = iw; wc = op.n2; } else two = false;
            break;
        default: two = false;
        }
        if (two) {
            size_t h2, w2, c2;
            if (!produced(i, op.x2, h2, w2, c2) || h2 != wh || w2 != ww || c2 != wc) {
                err = fmt("op %zu reads a second tensor of another shape", i);
                return false;
            }
        }
        op.ih = ih; op.iw = iw; op.oh = oh; op.ow = ow;
    }
    std::fill(pool.begin(), pool.end(), 0);
    size_t image;
    if (!shape_len(height, width, c, image)) { err = "input shape is zero or overflows"; return false; }
    auto grow = [&](size_t s, size_t n) {
        if (s >= pool.size()) { err = fmt("buffer %zu does not exist", s); return false; }
        if (pool[s] < n) pool[s] = n;
        return true;
    };
    if (!grow(slot, image)) return false;
    for (size_t i = 0; i < ops.size(); i++) {
        size_t n;
        if (!shape_len(ops[i].oh, ops[i].ow, ops[i].oc, n)) { err = fmt("op %zu output shape is zero or overflows", i); return false; }
        if (!grow(ops[i].y, n)) return false;
    }
    out_n.assign(outputs.size(), 0);
    for (size_t k = 0; k < outputs.size(); k++) {
        size_t oh, ow, oc;
        if (!produced(ops.size(), outputs[k], oh, ow, oc)) { err = fmt("output %zu is never written", k); return false; }
        out_n[k] = oh * ow * oc;
    }
    return true;
}

// plan.rs:498-767
bool Plan::check(size_t weight_floats, std::string &err) const {
    for (size_t n : pool)
        if (n > MAX_SCRATCH_FLOATS) { err = fmt("a buffer wants %zu floats, ceiling is %zu", n, MAX_SCRATCH_FLOATS); return false; }
    size_t input_len;
    if (!shape_len(h, w, c, input_len)) { err = "input shape is zero or overflows"; return false; }
    if (slot >= pool.size()) { err = fmt("the input names buffer %zu, only %zu exist", slot, pool.size()); return false; }
    if (pool[slot] < input_len) { err = "the input buffer is smaller than the image"; return false; }
    for (size_t k = 0; k < outputs.size(); k++) {
        if (outputs[k] >= pool.size()) { err = fmt("an output names buffer %zu, only %zu exist", outputs[k], pool.size()); return false; }
        if (pool[outputs[k]] < out_n[k]) { err = fmt("output %zu claims %zu elements, its buffer holds fewer", k, out_n[k]); return false; }
    }
    for (size_t i = 0; i < ops.size(); i++) {
        const Op &op = ops[i];
        auto bad = [&](const char *what) {
            char buf[256];
            std::snprintf(buf, sizeof buf, "op %zu (%s) %s", i, kind_name(op.kind), what);
            err = buf;
            return false;
        };
        size_t in_len, out_len;
        if (!shape_len(op.ih, op.iw, op.ic, in_len)) return bad("input shape is zero or overflows");
        if (!shape_len(op.oh, op.ow, op.oc, out_len)) return bad("output shape is zero or overflows");
        switch (op.kind) {
        case K_CONV: case K_DWCONV: case K_AVGPOOL: case K_MAXPOOL: {
            size_t dims[4] = {op.kh, op.kw, op.sh, op.sw};
            long pads[4] = {op.pt, op.pb, op.pl, op.pr};
            for (size_t d : dims)
                if (d == 0 || d > MAX_WINDOW) return bad("has an unsupported kernel, stride or padding");
            for (long p : pads)
                if (p < 0 || size_t(p) > MAX_WINDOW) return bad("has an unsupported kernel, stride or padding");
            if (op.oh > size_t(std::numeric_limits<long>::max()) / op.sh ||
                op.ow > size_t(std::numeric_limits<long>::max()) / op.sw)
                return bad("window coordinates overflow");
            if (op.ic > std::numeric_limits<size_t>::max() / op.sw) return bad("pixel stride overflows");
            break;
        }
        case K_MEAN:
            if (op.oh != 1 || op.ow != 1 || op.ic != op.oc) return bad("invalid channel mean");
            break;
        case K_CONCATC:
            if (op.ih != op.oh || op.iw != op.ow || op.ic + op.n2 != op.oc) return bad("invalid channel concatenation");
            break;
        case K_CTCHEAD: case K_CTCARGMAX: {
            size_t vocab = op.kind == K_CTCHEAD ? op.oc : op.n2;
            size_t cols = (vocab + 15) / 16 * 16;
            if (op.ih != 1 || op.oh != 1 || op.iw != op.ow || vocab == 0 ||
                (op.kind == K_CTCARGMAX && op.oc != 2) || cols * op.ic != op.w1 || op.b1 != cols)
                return bad("invalid CTC head");
            break;
        }
        case K_LAYERNORM:
            if (op.oc * 2 + 1 != op.w1) return bad("needs gamma, beta and epsilon");
            break;
        case K_ATTENTION:
            if (op.ih != 1 || op.oh != 1 || op.iw != op.ow || op.oc * 3 != op.ic || op.n2 == 0 || op.oc % op.n2 ||
                op.w1 != 1 || op.iw > MAX_SCRATCH_FLOATS / op.iw)
                return bad("invalid attention shape");
            break;
        case K_UPSAMPLE: case K_UPSAMPLEADD:
            if (op.ic != op.oc || !op.sh || !op.sw || op.ih * op.sh != op.oh || op.iw * op.sw != op.ow)
                return bad("invalid upsampling");
            break;
        case K_CONVTRANSPOSE: {
            size_t cols = op.kh * op.kw * op.oc;
            if (!op.kh || !op.kw || op.sh != op.kh || op.sw != op.kw || op.pt || op.pb || op.pl || op.pr ||
                op.ih * op.kh != op.oh || op.iw * op.kw != op.ow || cols * op.ic != op.w1 || (op.b1 && op.b1 != cols))
                return bad("invalid transposed convolution");
            break;
        }
        default: break;
        }
        if ((op.kind == K_ADD || op.kind == K_CHANNELMUL || op.kind == K_LAYERNORM) &&
            (op.ih != op.oh || op.iw != op.ow || op.ic != op.oc))
            return bad("elementwise input/output shapes differ");
        if (op.kind == K_AVGPOOL &&
            (op.ic != op.oc || op.pt || op.pb || op.pl || op.pr || op.kh > op.ih || op.kw > op.iw ||
             op.oh != (op.ih - op.kh) / op.sh + 1 || op.ow != (op.iw - op.kw) / op.sw + 1))
            return bad("average pool requires complete valid windows");
        if (op.kind == K_MAXPOOL) {
            if (op.ic != op.oc || op.pt || op.pl) return bad("maxpool changes channels or requests unsupported padding");
            if ((op.oh - 1) * op.sh >= op.ih || (op.ow - 1) * op.sw >= op.iw) return bad("maxpool contains an empty output window");
        }
        if (op.pointwise() && (op.ih != op.oh || op.iw != op.ow)) return bad("unit-stride pointwise changes spatial dimensions");
        if (op.x >= pool.size()) return bad("input names a missing buffer");
        if (pool[op.x] < in_len) return bad("reads past its input buffer");
        if (op.y >= pool.size()) return bad("output names a missing buffer");
        if (pool[op.y] < out_len) return bad("writes past its output buffer");
        if (op.y == op.x || (op.has_second() && op.x2 == op.y)) return bad("writes the buffer it reads");
        if (op.has_second()) {
            size_t need = op.oc;
            if (op.kind == K_ADD || op.kind == K_UPSAMPLEADD) need = out_len;
            else if (op.kind == K_CONCATC) need = op.oh * op.ow * op.n2;
            else if (op.kind == K_CONV && !shape_len(op.ih, op.iw, op.n2, need)) return bad("second input overflows");
            if (op.x2 >= pool.size()) return bad("second input names a missing buffer");
            if (pool[op.x2] < need) return bad("reads past its second input buffer");
        }
        if (op.kind == K_CONV || op.kind == K_DWCONV) {
            size_t taps = op.kh * op.kw, want;
            if (op.n2 > 0 && (op.kind == K_DWCONV || op.pointwise())) return bad("reads a second input it cannot");
            if (op.kind == K_DWCONV) {
                if (op.ic != op.oc) return bad("is depthwise but changes channel count");
                want = taps * op.oc;
            } else {
                want = (op.ic + op.n2) * taps * op.oc;
            }
            if (op.w1 != want) return bad("has weights its shape contradicts");
            if (op.b1 && op.b1 != op.oc) return bad("has a bias of the wrong length");
        }
        bool weighted = op.kind == K_CONV || op.kind == K_DWCONV || op.kind == K_LAYERNORM || op.kind == K_ATTENTION ||
                        op.kind == K_CTCHEAD || op.kind == K_CTCARGMAX || op.kind == K_CONVTRANSPOSE;
        if (!weighted && (op.w1 || op.b1)) return bad("has weights it does not use");
        if (op.fused != A_NONE &&
            !(op.kind == K_CONV || op.kind == K_DWCONV || op.kind == K_ADD || op.kind == K_CONVTRANSPOSE))
            return bad("has an invalid folded activation");
        if (op.w1 && (op.w0 > weight_floats || op.w1 > weight_floats - op.w0)) return bad("weights reach past the end");
        if (op.b1 && (op.b0 > weight_floats || op.b1 > weight_floats - op.b0)) return bad("bias reaches past the end");
    }
    return true;
}

bool Plan::parse(const uint8_t *bytes, size_t len, Plan &p, std::vector<float> &weights, std::string &err) {
    if (len < 8 || std::memcmp(bytes, "PPOCRPL1", 8) != 0) { err = "not a ppocr-native plan"; return false; }
    size_t at = 8;
    auto next = [&](size_t &v) {
        if (at + 4 > len) { err = "the description is truncated"; return false; }
        uint32_t word;
        std::memcpy(&word, bytes + at, 4);
        at += 4;
        v = word;
        return true;
    };
    size_t buffers, nout, nops;
    if (!next(p.slot) || !next(p.h) || !next(p.w) || !next(p.c) || !next(buffers) || !next(nout) || !next(nops))
        return false;
    // A count larger than the file fails on the first missing word; do not
    // reserve memory for it (plan.rs:324-333).
    if (nout > len / 4 || nops > len / (4 * OP_FIELDS)) { err = "the description is truncated"; return false; }
    p.outputs.resize(nout);
    for (size_t k = 0; k < nout; k++)
        if (!next(p.outputs[k])) return false;
    p.ops.resize(nops);
    for (size_t i = 0; i < nops; i++) {
        size_t f[OP_FIELDS];
        for (size_t j = 0; j < OP_FIELDS; j++)
            if (!next(f[j])) return false;
        if (f[0] >= K_COUNT) { err = fmt("operation kind %zu is unknown", f[0]); return false; }
        if (f[1] >= A_COUNT) { err = fmt("activation %zu is unknown", f[1]); return false; }
        Op &op = p.ops[i];
        op.kind = int(f[0]); op.fused = int(f[1]);
        op.x = f[2]; op.x2 = f[3]; op.y = f[4]; op.ic = f[5]; op.oc = f[6];
        op.kh = f[7]; op.kw = f[8]; op.sh = f[9]; op.sw = f[10];
        op.pt = long(f[11]); op.pb = long(f[12]); op.pl = long(f[13]); op.pr = long(f[14]);
        op.n2 = f[15]; op.w0 = f[16]; op.w1 = f[17]; op.b0 = f[18]; op.b1 = f[19];
    }
    if (buffers == 0 || buffers > nops + 1) { err = fmt("%zu buffers for %zu operations", buffers, nops); return false; }
    size_t start = (at + 63) / 64 * 64;
    if (start > len) { err = "the plan ends before its weights"; return false; }
    size_t raw = len - start;
    if (raw % 4) { err = fmt("the weights are %zu bytes, not a whole number of floats", raw); return false; }
    weights.resize(raw / 4);
    for (size_t i = 0; i < weights.size(); i++) {
        float v;
        std::memcpy(&v, bytes + start + 4 * i, 4);
        if (!std::isfinite(v)) { err = fmt("the weights hold a non-finite value at float %zu", i); return false; }
        if (std::fpclassify(v) == FP_SUBNORMAL) v = std::copysign(0.0f, v);  // plan.rs:819-842
        weights[i] = v;
    }
    p.pool.assign(buffers, 0);
    if (!p.derive_shapes(p.h, p.w, err) || !p.check(weights.size(), err)) return false;
    for (const Op &op : p.ops)  // plan.rs:367-377
        if (op.kind == K_LAYERNORM && !(weights[op.w0 + 2 * op.oc] > 0.0f)) {
            err = "layer normalization epsilon is not positive";
            return false;
        }
    return true;
}

bool Plan::set_size(size_t height, size_t width, size_t weight_floats, std::string &err) {
    size_t oh = h, ow = w;
    if (derive_shapes(height, width, err) && check(weight_floats, err)) return true;
    std::string ignored;
    derive_shapes(oh, ow, ignored);
    return false;
}

}  // namespace ppocr
