/* TEST INFRASTRUCTURE ONLY (see ppocr_oracle.h): the CPU oracle.
 *
 * Arithmetic follows the reference's tier 3 (AVX2+FMA) scalar definitions:
 * every convolution output adds its taps in kernel row-major order, each
 * tap's channels in order, one fused multiply-add each
 * (`kernels/dense.rs:104-141`, `kernels/depthwise.rs:12-45`,
 * `kernels/pointwise.rs:20-44`), with the bias first or last where the
 * reference's tiles put it (`bias_first` below). One detail is not
 * restated: the reference's pointwise kernels also add the bias last on the
 * few pixels a call leaves after its 12- and 4-pixel tiles
 * (`pointwise.rs:131-185`), which depends on how its executor splits rows;
 * those outputs differ from this restatement by at most one rounding.
 *
 * Compiled with -ffp-contract=off: a product and a sum written apart stay two
 * roundings, as Rust keeps them; fmaf() marks every fused one.
 */
#include "ppocr_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

enum {
    K_CONV, K_DWCONV, K_ADD, K_MAXPOOL, K_AVGPOOL, K_CHANNELMUL, K_CONCATC,
    K_LAYERNORM, K_ATTENTION, K_MEAN, K_CTCHEAD, K_CTCARGMAX, K_UPSAMPLE,
    K_UPSAMPLEADD, K_CONVTRANSPOSE, K_COUNT
};
enum { A_NONE, A_RELU, A_SIGMOID, A_GELU, A_SWISH, A_HARDSIGMOID, A_HARDSIGMOIDFIFTH,
       A_HARDSWISH, A_COUNT };

#define OP_FIELDS 20
#define MAX_SCRATCH_FLOATS ((size_t)1 << 30) /* plan.rs:73 */
#define MAX_WINDOW ((size_t)1 << 16)         /* plan.rs:77 */

typedef struct {
    int kind, fused;
    size_t x, x2, y, ih, iw, ic, oh, ow, oc, kh, kw, sh, sw;
    long pt, pb, pl, pr;
    size_t n2, w0, w1, b0, b1;
} orc_op;

struct orc_plan {
    size_t slot, h, w, c;
    size_t nbuf, nout, nops;
    size_t *outputs, *out_n, *pool;
    orc_op *ops;
    float *weights;
    size_t nweights;
    /* buffers kept from run to run (the reference's arena is allocated once
     * per size, src/engine/schedule.rs:528-620), grown when a size needs more */
    float **kept;
    size_t *kept_n;
};

/* ---------------------------------------------------------------- errors */

static int fail(char *err, size_t len, const char *fmt, ...) {
    if (err && len) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(err, len, fmt, ap);
        va_end(ap);
    }
    return -1;
}

/* ------------------------------------------------------------ activations */

static inline float f_of(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t u_of(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* XNNPACK f32-vsigmoid "p5-div" exp constants, kernels/activation.rs:10-21. */
#define EXP_MAGIC_BIAS f_of(0x4b40007fu)
#define LOG2E f_of(0x3fb8aa3bu)
#define MINUS_LN2 f_of(0xbf317218u)
#define EXP_C5 f_of(0x3c07cfceu)
#define EXP_C4 f_of(0x3d2b9d0du)
#define EXP_C3 f_of(0x3e2aad40u)
#define EXP_C2 f_of(0x3efffee3u)
#define EXP_C1 f_of(0x3f7ffffbu)
#define EXP_CUTOFF f_of(0xc2aeac4fu)

/* exp(z) for z <= 0, the FMA (tier 3) form: activation.rs:37-60. */
float orc_exp_neg(float z) {
    float n = fmaf(z, LOG2E, EXP_MAGIC_BIAS);
    float s = f_of(u_of(n) << 23);
    n = n - EXP_MAGIC_BIAS;
    float t = fmaf(n, MINUS_LN2, z);
    float p = fmaf(fmaf(fmaf(fmaf(EXP_C5, t, EXP_C4), t, EXP_C3), t, EXP_C2), t, EXP_C1);
    if (z < EXP_CUTOFF) return 0.0f;
    return fmaf(t * s, p, s);
}

/* exp_neg over eight lanes: orc_exp_neg's operations, one lane each (the
 * same fused multiply-adds, shift, subtraction and cut-off). */
static inline __m256 exp_neg8(__m256 z) {
    __m256 n = _mm256_fmadd_ps(z, _mm256_set1_ps(LOG2E), _mm256_set1_ps(EXP_MAGIC_BIAS));
    __m256 sc = _mm256_castsi256_ps(_mm256_slli_epi32(_mm256_castps_si256(n), 23));
    n = _mm256_sub_ps(n, _mm256_set1_ps(EXP_MAGIC_BIAS));
    __m256 t = _mm256_fmadd_ps(n, _mm256_set1_ps(MINUS_LN2), z);
    __m256 q = _mm256_fmadd_ps(_mm256_set1_ps(EXP_C5), t, _mm256_set1_ps(EXP_C4));
    q = _mm256_fmadd_ps(q, t, _mm256_set1_ps(EXP_C3));
    q = _mm256_fmadd_ps(q, t, _mm256_set1_ps(EXP_C2));
    q = _mm256_fmadd_ps(q, t, _mm256_set1_ps(EXP_C1));
    __m256 r = _mm256_fmadd_ps(_mm256_mul_ps(t, sc), q, sc);
    return _mm256_andnot_ps(_mm256_cmp_ps(z, _mm256_set1_ps(EXP_CUTOFF), _CMP_LT_OQ), r);
}

/* Rust's f32::clamp: NaN passes through. */
static inline float clampf(float v, float lo, float hi) {
    if (v < lo) v = lo;
    if (v > hi) v = hi;
    return v;
}

/* activation.rs:151-159 */
static inline float sigmoid_one(float x) {
    float e = orc_exp_neg(f_of(u_of(x) | 0x80000000u));
    float f = e / (e + 1.0f);
    return (u_of(x) >> 31) ? f : 1.0f - f;
}

/* layers.rs:20-40, 54-67 */
static const uint32_t PHI_P[6] = {0x3ecc4228u, 0x3d0aa93cu, 0x3b9943c9u,
                                  0x39310738u, 0x36d52462u, 0x32c36a3cu};
static const uint32_t PHI_Q[5] = {0x3e80c788u, 0x3ceaaaeeu, 0x3af6ffc6u,
                                  0x389a737au, 0x35a0b9e3u};
static inline float gelu_one(float x) {
    float c = clampf(x, -5.5f, 5.5f);
    float s = c * c;
    float p = f_of(PHI_P[5]);
    for (int k = 4; k >= 0; k--) p = fmaf(p, s, f_of(PHI_P[k]));
    float q = f_of(PHI_Q[4]);
    for (int k = 3; k >= 0; k--) q = fmaf(q, s, f_of(PHI_Q[k]));
    q = fmaf(q, s, 1.0f);
    return x * clampf(fmaf(c, p / q, 0.5f), 0.0f, 1.0f);
}

#define HARDSIGMOID_ALPHA f_of(0x3e2aaaadu) /* layers.rs:42 */

/* conv.rs:36-72 (Tail::apply) with the clamp of relu folded in. */
float orc_activation(int code, float v) {
    switch (code) {
    case A_RELU: return clampf(v, 0.0f, INFINITY);
    case A_SIGMOID: return sigmoid_one(v);
    case A_GELU: return gelu_one(v);
    case A_SWISH: return v * sigmoid_one(v); /* layers.rs:70 */
    case A_HARDSIGMOID: return clampf(v * HARDSIGMOID_ALPHA + 0.5f, 0.0f, 1.0f); /* :215 */
    case A_HARDSIGMOIDFIFTH: return clampf(v * 0.2f + 0.5f, 0.0f, 1.0f);        /* :222 */
    case A_HARDSWISH: /* extension code 7: x * hardsigmoid(x) */
        return v * clampf(v * HARDSIGMOID_ALPHA + 0.5f, 0.0f, 1.0f);
    default: return v;
    }
}

/* The activation over a span, one loop per code so that each one vectorises;
 * every element takes the same operations as orc_activation. */
/* clampf over eight lanes: below lo gives lo, then above hi gives hi, NaN
 * passes through. */
static inline __m256 clamp8(__m256 v, float lo, float hi) {
    __m256 l = _mm256_set1_ps(lo), h = _mm256_set1_ps(hi);
    v = _mm256_blendv_ps(v, l, _mm256_cmp_ps(v, l, _CMP_LT_OQ));
    return _mm256_blendv_ps(v, h, _mm256_cmp_ps(v, h, _CMP_GT_OQ));
}

/* sigmoid_one over eight lanes; the sign bit of x picks f or 1 - f. */
static inline __m256 sigmoid8(__m256 x) {
    __m256 e = exp_neg8(_mm256_or_ps(x, _mm256_set1_ps(-0.0f)));
    __m256 f = _mm256_div_ps(e, _mm256_add_ps(e, _mm256_set1_ps(1.0f)));
    return _mm256_blendv_ps(_mm256_sub_ps(_mm256_set1_ps(1.0f), f), f, x);
}

/* gelu_one over eight lanes. */
static inline __m256 gelu8(__m256 x) {
    __m256 c = clamp8(x, -5.5f, 5.5f), sq = _mm256_mul_ps(c, c);
    __m256 p = _mm256_set1_ps(f_of(PHI_P[5]));
    for (int k = 4; k >= 0; k--) p = _mm256_fmadd_ps(p, sq, _mm256_set1_ps(f_of(PHI_P[k])));
    __m256 q = _mm256_set1_ps(f_of(PHI_Q[4]));
    for (int k = 3; k >= 0; k--) q = _mm256_fmadd_ps(q, sq, _mm256_set1_ps(f_of(PHI_Q[k])));
    q = _mm256_fmadd_ps(q, sq, _mm256_set1_ps(1.0f));
    __m256 g = _mm256_fmadd_ps(c, _mm256_div_ps(p, q), _mm256_set1_ps(0.5f));
    return _mm256_mul_ps(x, clamp8(g, 0.0f, 1.0f));
}

/* Eight activations at a time with orc_activation's operations per lane. */
static inline __m256 activation8(int code, __m256 v) {
    switch (code) {
    case A_RELU: return clamp8(v, 0.0f, INFINITY);
    case A_SIGMOID: return sigmoid8(v);
    case A_GELU: return gelu8(v);
    case A_SWISH: return _mm256_mul_ps(v, sigmoid8(v));
    case A_HARDSIGMOID:
        return clamp8(_mm256_add_ps(_mm256_mul_ps(v, _mm256_set1_ps(HARDSIGMOID_ALPHA)), _mm256_set1_ps(0.5f)),
                      0.0f, 1.0f);
    case A_HARDSIGMOIDFIFTH:
        return clamp8(_mm256_add_ps(_mm256_mul_ps(v, _mm256_set1_ps(0.2f)), _mm256_set1_ps(0.5f)), 0.0f, 1.0f);
    case A_HARDSWISH:
        return _mm256_mul_ps(v, clamp8(_mm256_add_ps(_mm256_mul_ps(v, _mm256_set1_ps(HARDSIGMOID_ALPHA)),
                                                     _mm256_set1_ps(0.5f)),
                                       0.0f, 1.0f));
    default: return v;
    }
}

/* The activation over a span, eight lanes at a time, the rest one by one;
 * every element takes the same operations as orc_activation. */
static void tail_span(float *y, size_t n, int code) {
    size_t i = 0;
#define TAIL_CASE(c)                                                                                               \
    case c:                                                                                                        \
        for (; i + 8 <= n; i += 8) _mm256_storeu_ps(y + i, activation8(c, _mm256_loadu_ps(y + i)));               \
        break;
    switch (code) {
        TAIL_CASE(A_RELU)
        TAIL_CASE(A_SIGMOID)
        TAIL_CASE(A_GELU)
        TAIL_CASE(A_SWISH)
        TAIL_CASE(A_HARDSIGMOID)
        TAIL_CASE(A_HARDSIGMOIDFIFTH)
        TAIL_CASE(A_HARDSWISH)
    default: break;
    }
#undef TAIL_CASE
    for (; i < n; i++) y[i] = orc_activation(code, y[i]);
}

/* The fused activation of a layer's outputs. Spans of up to 64 Ki values
 * (the per-pixel and per-tile calls, made from inside the layers' own
 * parallel loops) run on the calling thread: opening a nested parallel
 * region for each of them cost more than the activation itself. */
static void tail(float *y, size_t n, int code) {
    if (code == A_NONE) return;
    if (n <= 65536) {
        tail_span(y, n, code);
        return;
    }
    const size_t chunk = 16384, chunks = (n + chunk - 1) / chunk;
#pragma omp parallel for schedule(static)
    for (size_t k = 0; k < chunks; k++) tail_span(y + k * chunk, k + 1 < chunks ? chunk : n - k * chunk, code);
}

/* ------------------------------------------------------------------ parse */

static int shape_len(size_t a, size_t b, size_t c, size_t *out) {
    if (!a || !b || !c) return 0;
    if (a > SIZE_MAX / b) return 0;
    size_t ab = a * b;
    if (ab > SIZE_MAX / c) return 0;
    *out = ab * c;
    return 1;
}

static int produced(const orc_plan *p, size_t before, size_t slot, size_t *h, size_t *w, size_t *c) {
    for (size_t i = before; i-- > 0;) {
        if (p->ops[i].y == slot) {
            *h = p->ops[i].oh; *w = p->ops[i].ow; *c = p->ops[i].oc;
            return 1;
        }
    }
    if (slot == p->slot) { *h = p->h; *w = p->w; *c = p->c; return 1; }
    return 0;
}

static int window_len(size_t n, long before, long after, size_t k, size_t s, size_t *out) {
    if (before < 0 || after < 0 || s == 0) return 0;
    size_t span = n + (size_t)before + (size_t)after;
    if (span < k) return 0;
    *out = (span - k) / s + 1;
    return 1;
}

/* plan.rs:414-494 */
static int derive_shapes(orc_plan *p, size_t height, size_t width, char *err, size_t el) {
    p->h = height; p->w = width;
    for (size_t i = 0; i < p->nops; i++) {
        size_t h, w, c;
        if (!produced(p, i, p->ops[i].x, &h, &w, &c))
            return fail(err, el, "op %zu reads a buffer nothing wrote", i);
        orc_op *op = &p->ops[i];
        if (c != op->ic) return fail(err, el, "op %zu reads a tensor of another shape", i);
        size_t oh = h, ow = w;
        switch (op->kind) {
        case K_CONV: case K_DWCONV: case K_MAXPOOL: case K_AVGPOOL:
            if (!window_len(h, op->pt, op->pb, op->kh, op->sh, &oh) ||
                !window_len(w, op->pl, op->pr, op->kw, op->sw, &ow))
                return fail(err, el, "op %zu has a window larger than its padded input", i);
            break;
        case K_UPSAMPLE: case K_UPSAMPLEADD:
            if ((op->sh && h > SIZE_MAX / op->sh) || (op->sw && w > SIZE_MAX / op->sw))
                return fail(err, el, "op %zu output size overflows", i);
            oh = h * op->sh; ow = w * op->sw; break;
        case K_CONVTRANSPOSE:
            if ((op->kh && h > SIZE_MAX / op->kh) || (op->kw && w > SIZE_MAX / op->kw))
                return fail(err, el, "op %zu output size overflows", i);
            oh = h * op->kh; ow = w * op->kw; break;
        case K_MEAN: oh = 1; ow = 1; break;
        default: break;
        }
        int has2 = 1;
        size_t wh = 0, ww = 0, wc = 0;
        switch (op->kind) {
        case K_ADD: case K_UPSAMPLEADD: wh = oh; ww = ow; wc = op->oc; break;
        case K_CONCATC: wh = oh; ww = ow; wc = op->n2; break;
        case K_CHANNELMUL: wh = 1; ww = 1; wc = op->oc; break;
        case K_CONV: if (op->n2 > 0) { wh = h; ww = w; wc = op->n2; } else has2 = 0; break;
        default: has2 = 0;
        }
        if (has2) {
            size_t h2, w2, c2;
            if (!produced(p, i, op->x2, &h2, &w2, &c2) || h2 != wh || w2 != ww || c2 != wc)
                return fail(err, el, "op %zu reads a second tensor of another shape", i);
        }
        op->ih = h; op->iw = w; op->oh = oh; op->ow = ow;
    }
    memset(p->pool, 0, p->nbuf * sizeof(size_t));
    size_t image;
    if (!shape_len(height, width, p->c, &image)) return fail(err, el, "input shape is zero or overflows");
    if (p->slot >= p->nbuf) return fail(err, el, "buffer %zu does not exist", p->slot);
    if (p->pool[p->slot] < image) p->pool[p->slot] = image;
    for (size_t i = 0; i < p->nops; i++) {
        size_t n;
        if (!shape_len(p->ops[i].oh, p->ops[i].ow, p->ops[i].oc, &n))
            return fail(err, el, "op %zu output shape is zero or overflows", i);
        if (p->ops[i].y >= p->nbuf) return fail(err, el, "buffer %zu does not exist", p->ops[i].y);
        if (p->pool[p->ops[i].y] < n) p->pool[p->ops[i].y] = n;
    }
    for (size_t k = 0; k < p->nout; k++) {
        size_t h, w, c;
        if (!produced(p, p->nops, p->outputs[k], &h, &w, &c))
            return fail(err, el, "output %zu is never written", k);
        p->out_n[k] = h * w * c;
    }
    return 0;
}

static int has_second(const orc_op *op) {
    return op->kind == K_ADD || op->kind == K_CHANNELMUL || op->kind == K_CONCATC ||
           op->kind == K_UPSAMPLEADD || (op->kind == K_CONV && op->n2 > 0);
}
static int is_pointwise(const orc_op *op) {
    return op->kind == K_CONV && op->kh == 1 && op->kw == 1 && op->sh == 1 && op->sw == 1 &&
           !op->pt && !op->pb && !op->pl && !op->pr;
}

/* plan.rs:498-767, the rules the executor relies on. */
static int check(const orc_plan *p, char *err, size_t el) {
    for (size_t b = 0; b < p->nbuf; b++)
        if (p->pool[b] > MAX_SCRATCH_FLOATS)
            return fail(err, el, "a buffer wants %zu floats", p->pool[b]);
    size_t input_len;
    if (!shape_len(p->h, p->w, p->c, &input_len)) return fail(err, el, "input shape is zero");
    if (p->pool[p->slot] < input_len) return fail(err, el, "input buffer smaller than the image");
    for (size_t k = 0; k < p->nout; k++) {
        if (p->outputs[k] >= p->nbuf) return fail(err, el, "an output names a missing buffer");
        if (p->pool[p->outputs[k]] < p->out_n[k]) return fail(err, el, "output %zu too large", k);
    }
    for (size_t i = 0; i < p->nops; i++) {
        const orc_op *op = &p->ops[i];
        size_t in_len, out_len;
        if (!shape_len(op->ih, op->iw, op->ic, &in_len)) return fail(err, el, "op %zu input shape is zero", i);
        if (!shape_len(op->oh, op->ow, op->oc, &out_len)) return fail(err, el, "op %zu output shape is zero", i);
        switch (op->kind) {
        case K_CONV: case K_DWCONV: case K_AVGPOOL: case K_MAXPOOL:
            if (!op->kh || !op->kw || !op->sh || !op->sw || op->kh > MAX_WINDOW || op->kw > MAX_WINDOW ||
                op->sh > MAX_WINDOW || op->sw > MAX_WINDOW || op->pt < 0 || op->pb < 0 || op->pl < 0 ||
                op->pr < 0 || (size_t)op->pt > MAX_WINDOW || (size_t)op->pb > MAX_WINDOW ||
                (size_t)op->pl > MAX_WINDOW || (size_t)op->pr > MAX_WINDOW)
                return fail(err, el, "op %zu has an unsupported kernel, stride or padding", i);
            break;
        case K_MEAN:
            if (op->oh != 1 || op->ow != 1 || op->ic != op->oc) return fail(err, el, "op %zu invalid mean", i);
            break;
        case K_CONCATC:
            if (op->ih != op->oh || op->iw != op->ow || op->ic + op->n2 != op->oc)
                return fail(err, el, "op %zu invalid concatenation", i);
            break;
        case K_CTCHEAD: case K_CTCARGMAX: {
            size_t vocab = op->kind == K_CTCHEAD ? op->oc : op->n2;
            size_t cols = (vocab + 15) / 16 * 16;
            if (op->ih != 1 || op->oh != 1 || op->iw != op->ow || !vocab ||
                (op->kind == K_CTCARGMAX && op->oc != 2) || cols * op->ic != op->w1 || op->b1 != cols)
                return fail(err, el, "op %zu invalid CTC head", i);
            break;
        }
        case K_LAYERNORM:
            if (op->oc * 2 + 1 != op->w1) return fail(err, el, "op %zu needs gamma, beta and epsilon", i);
            break;
        case K_ATTENTION:
            if (op->ih != 1 || op->oh != 1 || op->iw != op->ow || op->oc * 3 != op->ic || !op->n2 ||
                op->oc % op->n2 || op->w1 != 1 || op->iw * op->iw > MAX_SCRATCH_FLOATS)
                return fail(err, el, "op %zu invalid attention shape", i);
            break;
        case K_UPSAMPLE: case K_UPSAMPLEADD:
            if (op->ic != op->oc || !op->sh || !op->sw || op->ih * op->sh != op->oh || op->iw * op->sw != op->ow)
                return fail(err, el, "op %zu invalid upsampling", i);
            break;
        case K_CONVTRANSPOSE: {
            size_t cols = op->kh * op->kw * op->oc;
            if (!op->kh || !op->kw || op->sh != op->kh || op->sw != op->kw || op->pt || op->pb || op->pl ||
                op->pr || op->ih * op->kh != op->oh || op->iw * op->kw != op->ow || cols * op->ic != op->w1 ||
                (op->b1 && op->b1 != cols))
                return fail(err, el, "op %zu invalid transposed convolution", i);
            break;
        }
        default: break;
        }
        if ((op->kind == K_ADD || op->kind == K_CHANNELMUL || op->kind == K_LAYERNORM) &&
            (op->ih != op->oh || op->iw != op->ow || op->ic != op->oc))
            return fail(err, el, "op %zu elementwise shapes differ", i);
        if (op->kind == K_AVGPOOL &&
            (op->ic != op->oc || op->pt || op->pb || op->pl || op->pr || op->kh > op->ih || op->kw > op->iw ||
             op->oh != (op->ih - op->kh) / op->sh + 1 || op->ow != (op->iw - op->kw) / op->sw + 1))
            return fail(err, el, "op %zu average pool requires complete valid windows", i);
        if (op->kind == K_MAXPOOL) {
            if (op->ic != op->oc || op->pt || op->pl) return fail(err, el, "op %zu maxpool padding", i);
            if ((op->oh - 1) * op->sh >= op->ih || (op->ow - 1) * op->sw >= op->iw)
                return fail(err, el, "op %zu maxpool contains an empty output window", i);
        }
        if (is_pointwise(op) && (op->ih != op->oh || op->iw != op->ow))
            return fail(err, el, "op %zu pointwise changes spatial dimensions", i);
        if (op->x >= p->nbuf || p->pool[op->x] < in_len) return fail(err, el, "op %zu reads past its input", i);
        if (op->y >= p->nbuf || p->pool[op->y] < out_len) return fail(err, el, "op %zu writes past its output", i);
        if (op->y == op->x || (has_second(op) && op->x2 == op->y))
            return fail(err, el, "op %zu writes the buffer it reads", i);
        if (has_second(op)) {
            size_t need = op->oc;
            if (op->kind == K_ADD || op->kind == K_UPSAMPLEADD) need = out_len;
            else if (op->kind == K_CONCATC) need = op->oh * op->ow * op->n2;
            else if (op->kind == K_CONV) need = op->ih * op->iw * op->n2;
            if (op->x2 >= p->nbuf || p->pool[op->x2] < need) return fail(err, el, "op %zu reads past its second input", i);
        }
        if (op->kind == K_CONV || op->kind == K_DWCONV) {
            size_t taps = op->kh * op->kw, want;
            if (op->n2 > 0 && (op->kind == K_DWCONV || is_pointwise(op)))
                return fail(err, el, "op %zu reads a second input it cannot", i);
            if (op->kind == K_DWCONV) {
                if (op->ic != op->oc) return fail(err, el, "op %zu depthwise changes channels", i);
                want = taps * op->oc;
            } else {
                want = (op->ic + op->n2) * taps * op->oc;
            }
            if (op->w1 != want) return fail(err, el, "op %zu: %zu weights for a shape needing %zu", i, op->w1, want);
            if (op->b1 && op->b1 != op->oc) return fail(err, el, "op %zu has a bias of the wrong length", i);
        }
        int weighted = op->kind == K_CONV || op->kind == K_DWCONV || op->kind == K_LAYERNORM ||
                       op->kind == K_ATTENTION || op->kind == K_CTCHEAD || op->kind == K_CTCARGMAX ||
                       op->kind == K_CONVTRANSPOSE;
        if (!weighted && (op->w1 || op->b1)) return fail(err, el, "op %zu has weights it does not use", i);
        if (op->fused != A_NONE && !(op->kind == K_CONV || op->kind == K_DWCONV || op->kind == K_ADD ||
                                     op->kind == K_CONVTRANSPOSE))
            return fail(err, el, "op %zu has an invalid folded activation", i);
        if (op->w1 && op->w0 + op->w1 > p->nweights) return fail(err, el, "op %zu weights past the end", i);
        if (op->b1 && op->b0 + op->b1 > p->nweights) return fail(err, el, "op %zu bias past the end", i);
    }
    return 0;
}

orc_plan *orc_load(const uint8_t *bytes, size_t len, char *err, size_t el) {
    if (len < 8 || memcmp(bytes, "PPOCRPL1", 8)) { fail(err, el, "not a ppocr-native plan"); return NULL; }
    size_t at = 8;
#define NEXT(v)                                                              \
    do {                                                                     \
        if (at + 4 > len) { fail(err, el, "the description is truncated"); goto bad; } \
        uint32_t w_; memcpy(&w_, bytes + at, 4); at += 4; (v) = w_;          \
    } while (0)
    orc_plan *p = calloc(1, sizeof *p);
    if (!p) return NULL;
    size_t nops;
    NEXT(p->slot); NEXT(p->h); NEXT(p->w); NEXT(p->c); NEXT(p->nbuf); NEXT(p->nout); NEXT(nops);
    if (p->nout > len / 4 || nops > len / 80) { fail(err, el, "the description is truncated"); goto bad; }
    p->outputs = calloc(p->nout + 1, sizeof(size_t));
    p->out_n = calloc(p->nout + 1, sizeof(size_t));
    p->ops = calloc(nops + 1, sizeof(orc_op));
    if (!p->outputs || !p->out_n || !p->ops) goto bad;
    for (size_t k = 0; k < p->nout; k++) NEXT(p->outputs[k]);
    for (size_t i = 0; i < nops; i++) {
        size_t f[OP_FIELDS];
        for (int j = 0; j < OP_FIELDS; j++) NEXT(f[j]);
        if (f[0] >= K_COUNT) { fail(err, el, "operation kind %zu is unknown", f[0]); goto bad; }
        if (f[1] >= A_COUNT) { fail(err, el, "activation %zu is unknown", f[1]); goto bad; }
        orc_op *op = &p->ops[i];
        op->kind = (int)f[0]; op->fused = (int)f[1];
        op->x = f[2]; op->x2 = f[3]; op->y = f[4]; op->ic = f[5]; op->oc = f[6];
        op->kh = f[7]; op->kw = f[8]; op->sh = f[9]; op->sw = f[10];
        op->pt = (long)f[11]; op->pb = (long)f[12]; op->pl = (long)f[13]; op->pr = (long)f[14];
        op->n2 = f[15]; op->w0 = f[16]; op->w1 = f[17]; op->b0 = f[18]; op->b1 = f[19];
    }
#undef NEXT
    p->nops = nops;
    if (p->nbuf == 0 || p->nbuf > nops + 1) { fail(err, el, "%zu buffers for %zu operations", p->nbuf, nops); goto bad; }
    size_t start = (at + 63) / 64 * 64;
    if (start > len) { fail(err, el, "the plan ends before its weights"); goto bad; }
    size_t raw = len - start;
    if (raw % 4) { fail(err, el, "the weights are not a whole number of floats"); goto bad; }
    p->nweights = raw / 4;
    p->weights = malloc((p->nweights + 1) * sizeof(float));
    p->pool = calloc(p->nbuf, sizeof(size_t));
    if (!p->weights || !p->pool) goto bad;
    for (size_t i = 0; i < p->nweights; i++) {
        float v;
        memcpy(&v, bytes + start + 4 * i, 4);
        if (isnan(v) || isinf(v)) { fail(err, el, "the weights hold a non-finite value at float %zu", i); goto bad; }
        if (fpclassify(v) == FP_SUBNORMAL) v = copysignf(0.0f, v); /* plan.rs:819-842 */
        p->weights[i] = v;
    }
    if (derive_shapes(p, p->h, p->w, err, el) || check(p, err, el)) goto bad;
    for (size_t i = 0; i < p->nops; i++)
        if (p->ops[i].kind == K_LAYERNORM && p->weights[p->ops[i].w0 + 2 * p->ops[i].oc] <= 0.0f) {
            fail(err, el, "layer normalization epsilon is not positive");
            goto bad;
        }
    return p;
bad:
    orc_free(p);
    return NULL;
}

void orc_free(orc_plan *p) {
    if (!p) return;
    if (p->kept)
        for (size_t b = 0; b < p->nbuf; b++) free(p->kept[b]);
    free(p->kept); free(p->kept_n);
    free(p->outputs); free(p->out_n); free(p->pool); free(p->ops); free(p->weights);
    free(p);
}

int orc_set_size(orc_plan *p, size_t h, size_t w, char *err, size_t el) {
    size_t oh = p->h, ow = p->w;
    if (derive_shapes(p, h, w, err, el) == 0 && check(p, err, el) == 0) return 0;
    char scratch[8];
    derive_shapes(p, oh, ow, scratch, sizeof scratch);
    return -1;
}

size_t orc_input_len(const orc_plan *p) { return p->h * p->w * p->c; }
size_t orc_output_count(const orc_plan *p) { return p->nout; }
size_t orc_output_len(const orc_plan *p, size_t k) { return k < p->nout ? p->out_n[k] : 0; }

/* ------------------------------------------------------------------ layers */

static const float *W(const orc_plan *p, size_t at) { return p->weights + at; }

/* Where the reference's tier-3 kernels add a convolution's bias: first for
 * RGB stems (conv.rs:171-177), for pointwise layers whose output width is a
 * multiple of 16 (pointwise.rs:77-102) and for windowed ones of such width
 * except the last `ow % 4` pixels of each row (dense.rs:60-66); last
 * otherwise (pointwise.rs:33-35, dense.rs:127-130). */
static int bias_first(const orc_op *op, size_t ox) {
    if (!is_pointwise(op) && op->ic == 3 && op->n2 == 0) return 1;
    if (op->oc % 16) return 0;
    if (is_pointwise(op)) return 1;
    return ox < op->ow - op->ow % 4;
}

/* The timed CPU path (bench.py's reference arm): register-tiled AVX2+FMA
 * loops with the reference tier-3 engine's tile shape (6 pixels x 16 output
 * columns in 12 ymm accumulators, kernels/pointwise.rs:429 pw_p6o16_avx2) for
 * the dense convolutions and the CTC head's logits. Every output keeps its
 * own chain of fused multiply-adds in the same order as the loops below
 * (bias first or last per bias_first, taps in row-major order, channels in
 * order), so the results are the same bits; tests/test_oracle.py checks it.
 * Off by default: the parity tests use the plain loops. */
static int g_fast = 0;
void orc_set_fast(int on) { g_fast = on; }

/* Whether the 6 output pixels from ox on all read every horizontal tap
 * inside the image (their ix run is monotonic in ox). */
/* Whether output pixels ox .. ox + n - 1 of a row read only columns inside
 * the input (no padded taps). */
static int row_interior(const orc_op *op, size_t ox, size_t n) {
    long first = (long)(ox * op->sw) - op->pl, last = (long)((ox + n - 1) * op->sw + op->kw - 1) - op->pl;
    return ox + n <= op->ow && first >= 0 && last < (long)op->iw;
}

/* The timed path's register tile: P interior pixels of one output row by
 * output columns o0 .. o0 + 8 * NV, the accumulators in registers. Each
 * output keeps conv_pixel's chain: the bias first or last per bias_first,
 * taps in kernel row-major order, each tap's x channels then x2's, one fused
 * multiply-add each. */
static inline __attribute__((always_inline)) void conv_tile(const orc_op *op, const float *w, const float *b,
                                                            const float *x, const float *x2, float *y, long oy,
                                                            size_t ox, size_t o0, const int P, const int NV) {
    const size_t co = op->oc, ch = op->ic + op->n2;
    __m256 acc[4][3];
    int first[4];
#pragma GCC unroll 6
    for (int r = 0; r < P; r++) {
        first[r] = bias_first(op, ox + r);
#pragma GCC unroll 3
        for (int v = 0; v < NV; v++)
            acc[r][v] = (b && first[r]) ? _mm256_loadu_ps(b + o0 + 8 * v) : _mm256_setzero_ps();
    }
    for (size_t ky = 0; ky < op->kh; ky++) {
        long iy = oy * (long)op->sh + (long)ky - op->pt;
        if (iy < 0 || iy >= (long)op->ih) continue;
        for (size_t kx = 0; kx < op->kw; kx++) {
            const float *tap = w + (ky * op->kw + kx) * ch * co + o0;
            const float *px[4];
#pragma GCC unroll 6
            for (int r = 0; r < P; r++)
                px[r] = x + ((size_t)iy * op->iw + (ox + r) * op->sw + kx - op->pl) * op->ic;
            for (size_t i = 0; i < op->ic; i++) {
                const float *row = tap + i * co;
                __m256 wv[3];
#pragma GCC unroll 3
                for (int v = 0; v < NV; v++) wv[v] = _mm256_loadu_ps(row + 8 * v);
#pragma GCC unroll 6
                for (int r = 0; r < P; r++) {
                    __m256 xv = _mm256_broadcast_ss(px[r] + i);
#pragma GCC unroll 3
                    for (int v = 0; v < NV; v++) acc[r][v] = _mm256_fmadd_ps(wv[v], xv, acc[r][v]);
                }
            }
            if (op->n2) {
#pragma GCC unroll 6
                for (int r = 0; r < P; r++)
                    px[r] = x2 + ((size_t)iy * op->iw + (ox + r) * op->sw + kx - op->pl) * op->n2;
                for (size_t i = 0; i < op->n2; i++) {
                    const float *row = tap + (op->ic + i) * co;
                    __m256 wv[3];
#pragma GCC unroll 3
                    for (int v = 0; v < NV; v++) wv[v] = _mm256_loadu_ps(row + 8 * v);
#pragma GCC unroll 6
                    for (int r = 0; r < P; r++) {
                        __m256 xv = _mm256_broadcast_ss(px[r] + i);
#pragma GCC unroll 3
                        for (int v = 0; v < NV; v++) acc[r][v] = _mm256_fmadd_ps(wv[v], xv, acc[r][v]);
                    }
                }
            }
        }
    }
#pragma GCC unroll 6
    for (int r = 0; r < P; r++) {
        float *out = y + ((size_t)oy * op->ow + ox + r) * co + o0;
#pragma GCC unroll 3
        for (int v = 0; v < NV; v++) {
            __m256 a = acc[r][v];
            if (b && !first[r]) a = _mm256_add_ps(a, _mm256_loadu_ps(b + o0 + 8 * v));
            _mm256_storeu_ps(out + 8 * v, a);
        }
    }
}


static void conv_tile_p4v3(const orc_op *op, const float *w, const float *b, const float *x, const float *x2,
                           float *y, long oy, size_t ox, size_t o0) { conv_tile(op, w, b, x, x2, y, oy, ox, o0, 4, 3); }
static void conv_tile_p4v2(const orc_op *op, const float *w, const float *b, const float *x, const float *x2,
                           float *y, long oy, size_t ox, size_t o0) { conv_tile(op, w, b, x, x2, y, oy, ox, o0, 4, 2); }
static void conv_tile_p4v1(const orc_op *op, const float *w, const float *b, const float *x, const float *x2,
                           float *y, long oy, size_t ox, size_t o0) { conv_tile(op, w, b, x, x2, y, oy, ox, o0, 4, 1); }

static void conv_pixel(const orc_plan *p, const orc_op *op, const float *x, const float *x2, float *y, long oy,
                       size_t ox);

/* One output row of the timed path's dense convolution: 4-pixel register
 * tiles where the window lies inside the input, conv_pixel elsewhere. */
static void conv_fast_row(const orc_plan *p, const orc_op *op, const float *w, const float *b, const float *x,
                          const float *x2, float *y, long oy) {
    const size_t co = op->oc, P = 4;
    size_t ox = 0;
    while (ox < op->ow) {
        if (row_interior(op, ox, P)) {
            size_t o0 = 0;
            for (; o0 + 24 <= co; o0 += 24) conv_tile_p4v3(op, w, b, x, x2, y, oy, ox, o0);
            for (; o0 + 16 <= co; o0 += 16) conv_tile_p4v2(op, w, b, x, x2, y, oy, ox, o0);
            for (; o0 + 8 <= co; o0 += 8) conv_tile_p4v1(op, w, b, x, x2, y, oy, ox, o0);
            tail(y + ((size_t)oy * op->ow + ox) * co, P * co, op->fused);
            ox += P;
        } else {
            conv_pixel(p, op, x, x2, y, oy, ox);
            ox++;
        }
    }
}

/* The timed path's dense convolution, rows over the threads. With `mean`
 * (the convolution feeds a channel mean), each finished row is added to
 * the mean's f64 sums in row order while it is still in the cache of the
 * thread that wrote it, the reference's fused mean (layers.rs:408-431):
 * mean()'s sums, in mean()'s order. */
static void conv_fast(const orc_plan *p, const orc_op *op, const float *x, const float *x2, float *y, float *mean) {
    const float *w = W(p, op->w0), *b = op->b1 ? W(p, op->b0) : NULL;
    const size_t co = op->oc;
    long rows = (long)op->oh;
    if (!mean) {
#pragma omp parallel for schedule(static)
        for (long oy = 0; oy < rows; oy++) conv_fast_row(p, op, w, b, x, x2, y, oy);
        return;
    }
    double *sums = calloc(co, sizeof(double));
#pragma omp parallel for schedule(static, 1) ordered
    for (long oy = 0; oy < rows; oy++) {
        conv_fast_row(p, op, w, b, x, x2, y, oy);
#pragma omp ordered
        {
            const float *r = y + (size_t)oy * op->ow * co;
            for (size_t px = 0; px < op->ow; px++)
                for (size_t k = 0; k < co; k++) sums[k] += (double)r[px * co + k];
        }
    }
    const size_t pixels = op->oh * op->ow;
    for (size_t k = 0; k < co; k++) mean[k] = (float)(sums[k] / (double)pixels);
    free(sums);
}

/* Dense convolution of any window over the channel concatenation of x (ic
 * channels) and x2 (n2 channels): kernels/dense.rs:20-141 and the stem path
 * conv.rs:146-236. Weights [kh][kw][ic+n2][oc]; padded taps are skipped (the
 * reference multiplies them by zeros, which leaves every sum unchanged). */
static void conv_pixel(const orc_plan *p, const orc_op *op, const float *x, const float *x2, float *y, long oy,
                       size_t ox) {
    const float *w = W(p, op->w0), *b = op->b1 ? W(p, op->b0) : NULL;
    size_t co = op->oc, ch = op->ic + op->n2;
    {
        {
            float *acc = y + ((size_t)oy * op->ow + ox) * co;
            int first = bias_first(op, ox);
            for (size_t o = 0; o < co; o++) acc[o] = (b && first) ? b[o] : 0.0f;
            for (size_t ky = 0; ky < op->kh; ky++) {
                long iy = oy * (long)op->sh + (long)ky - op->pt;
                if (iy < 0 || iy >= (long)op->ih) continue;
                for (size_t kx = 0; kx < op->kw; kx++) {
                    long ix = (long)(ox * op->sw + kx) - op->pl;
                    if (ix < 0 || ix >= (long)op->iw) continue;
                    const float *tap = w + (ky * op->kw + kx) * ch * co;
                    const float *px = x + ((size_t)iy * op->iw + (size_t)ix) * op->ic;
                    for (size_t i = 0; i < op->ic; i++) {
                        float v = px[i];
                        const float *row = tap + i * co;
                        for (size_t o = 0; o < co; o++) acc[o] = fmaf(row[o], v, acc[o]);
                    }
                    if (op->n2) {
                        const float *px2 = x2 + ((size_t)iy * op->iw + (size_t)ix) * op->n2;
                        for (size_t i = 0; i < op->n2; i++) {
                            float v = px2[i];
                            const float *row = tap + (op->ic + i) * co;
                            for (size_t o = 0; o < co; o++) acc[o] = fmaf(row[o], v, acc[o]);
                        }
                    }
                }
            }
            if (b && !first)
                for (size_t o = 0; o < co; o++) acc[o] += b[o];
            tail(acc, co, op->fused);
        }
    }
}

static void conv(const orc_plan *p, const orc_op *op, const float *x, const float *x2, float *y) {
    if (g_fast && op->oc % 8 == 0) {
        conv_fast(p, op, x, x2, y, NULL);
        return;
    }
    long rows = (long)op->oh;
#pragma omp parallel for schedule(static)
    for (long oy = 0; oy < rows; oy++)
        for (size_t ox = 0; ox < op->ow; ox++) conv_pixel(p, op, x, x2, y, oy, ox);
}

/* Depthwise convolution: conv.rs:244-339, kernels/depthwise.rs:12-45 —
 * bias first, taps in row-major order, one fused multiply-add per tap. */
/* The timed path's depthwise tile: six interior pixels of a row, eight
 * channels, the accumulators in registers, the same chain per output. */
static inline void dw_tile6(const orc_op *op, const float *w, const float *b, const float *x, float *y, long oy,
                            size_t ox, size_t c0) {
    const size_t c = op->oc;
    __m256 acc[6];
    for (int r = 0; r < 6; r++) acc[r] = b ? _mm256_loadu_ps(b + c0) : _mm256_setzero_ps();
    for (size_t ky = 0; ky < op->kh; ky++) {
        long iy = oy * (long)op->sh + (long)ky - op->pt;
        if (iy < 0 || iy >= (long)op->ih) continue;
        const float *xrow = x + (size_t)iy * op->iw * c + c0;
        for (size_t kx = 0; kx < op->kw; kx++) {
            __m256 wv = _mm256_loadu_ps(w + (ky * op->kw + kx) * c + c0);
            for (int r = 0; r < 6; r++) {
                size_t ix = (ox + r) * op->sw + kx - op->pl;
                acc[r] = _mm256_fmadd_ps(wv, _mm256_loadu_ps(xrow + ix * c), acc[r]);
            }
        }
    }
    for (int r = 0; r < 6; r++) _mm256_storeu_ps(y + ((size_t)oy * op->ow + ox + r) * c + c0, acc[r]);
}

static void dwconv(const orc_plan *p, const orc_op *op, const float *x, float *y) {
    const float *w = W(p, op->w0), *b = op->b1 ? W(p, op->b0) : NULL;
    size_t c = op->oc;
    long rows = (long)op->oh;
    if (g_fast && c % 8 == 0) {
#pragma omp parallel for schedule(static)
        for (long oy = 0; oy < rows; oy++) {
            size_t ox = 0;
            while (ox < op->ow) {
                if (row_interior(op, ox, 6)) {
                    for (size_t c0 = 0; c0 < c; c0 += 8) dw_tile6(op, w, b, x, y, oy, ox, c0);
                    tail(y + ((size_t)oy * op->ow + ox) * c, 6 * c, op->fused);
                    ox += 6;
                    continue;
                }
                float *acc = y + ((size_t)oy * op->ow + ox) * c;
                for (size_t k = 0; k < c; k++) acc[k] = b ? b[k] : 0.0f;
                for (size_t ky = 0; ky < op->kh; ky++) {
                    long iy = oy * (long)op->sh + (long)ky - op->pt;
                    if (iy < 0 || iy >= (long)op->ih) continue;
                    for (size_t kx = 0; kx < op->kw; kx++) {
                        long ix = (long)(ox * op->sw + kx) - op->pl;
                        if (ix < 0 || ix >= (long)op->iw) continue;
                        const float *tap = w + (ky * op->kw + kx) * c;
                        const float *px = x + ((size_t)iy * op->iw + (size_t)ix) * c;
                        for (size_t k = 0; k < c; k++) acc[k] = fmaf(tap[k], px[k], acc[k]);
                    }
                }
                tail(acc, c, op->fused);
                ox++;
            }
        }
        return;
    }
#pragma omp parallel for schedule(static)
    for (long oy = 0; oy < rows; oy++) {
        for (size_t ox = 0; ox < op->ow; ox++) {
            float *acc = y + ((size_t)oy * op->ow + ox) * c;
            for (size_t k = 0; k < c; k++) acc[k] = b ? b[k] : 0.0f;
            for (size_t ky = 0; ky < op->kh; ky++) {
                long iy = oy * (long)op->sh + (long)ky - op->pt;
                if (iy < 0 || iy >= (long)op->ih) continue;
                for (size_t kx = 0; kx < op->kw; kx++) {
                    long ix = (long)(ox * op->sw + kx) - op->pl;
                    if (ix < 0 || ix >= (long)op->iw) continue;
                    const float *tap = w + (ky * op->kw + kx) * c;
                    const float *px = x + ((size_t)iy * op->iw + (size_t)ix) * c;
                    for (size_t k = 0; k < c; k++) acc[k] = fmaf(tap[k], px[k], acc[k]);
                }
            }
            tail(acc, c, op->fused);
        }
    }
}

/* conv.rs:404-440: windows cut short at the bottom and right edges; the
 * first tap is copied, later ones kept only when greater
 * (kernels/elementwise.rs:101-115). */
static void maxpool(const orc_op *op, const float *x, float *y) {
    size_t c = op->oc;
    for (size_t oy = 0; oy < op->oh; oy++)
        for (size_t ox = 0; ox < op->ow; ox++) {
            float *out = y + (oy * op->ow + ox) * c;
            int seeded = 0;
            for (size_t ky = 0; ky < op->kh; ky++) {
                size_t iy = oy * op->sh + ky;
                if (iy >= op->ih) continue;
                for (size_t kx = 0; kx < op->kw; kx++) {
                    size_t ix = ox * op->sw + kx;
                    if (ix >= op->iw) continue;
                    const float *src = x + (iy * op->iw + ix) * c;
                    if (!seeded) { memcpy(out, src, c * sizeof(float)); seeded = 1; }
                    else for (size_t k = 0; k < c; k++) if (src[k] > out[k]) out[k] = src[k];
                }
            }
        }
}

/* layers.rs:443-463: taps summed in row-major order, then divided. */
static void avgpool(const orc_op *op, const float *x, float *y) {
    float divisor = (float)(op->kh * op->kw);
    for (size_t oy = 0; oy < op->oh; oy++)
        for (size_t ox = 0; ox < op->ow; ox++) {
            float *out = y + (oy * op->ow + ox) * op->oc;
            for (size_t k = 0; k < op->oc; k++) out[k] = 0.0f;
            for (size_t ky = 0; ky < op->kh; ky++)
                for (size_t kx = 0; kx < op->kw; kx++) {
                    const float *src = x + ((oy * op->sh + ky) * op->iw + ox * op->sw + kx) * op->ic;
                    for (size_t k = 0; k < op->ic; k++) out[k] += src[k];
                }
            for (size_t k = 0; k < op->oc; k++) out[k] /= divisor;
        }
}

/* layers.rs:391-406: pixels summed in order in f64, then divided. */
static void mean(const orc_op *op, const float *x, float *y) {
    size_t c = op->ic, pixels = op->ih * op->iw;
    double *sums = calloc(c, sizeof(double));
    for (size_t px = 0; px < pixels; px++)
        for (size_t k = 0; k < c; k++) sums[k] += (double)x[px * c + k];
    for (size_t k = 0; k < c; k++) y[k] = (float)(sums[k] / (double)pixels);
    free(sums);
}

/* layers.rs:467-479 */
static void layernorm(const orc_plan *p, const orc_op *op, const float *x, float *y) {
    size_t c = op->oc;
    const float *gamma = W(p, op->w0), *beta = gamma + c;
    float eps = gamma[2 * c];
    for (size_t px = 0; px < op->oh * op->ow; px++) {
        const float *v = x + px * c;
        float s = 0.0f;
        for (size_t k = 0; k < c; k++) s += v[k];
        float m = s / (float)c;
        float q = 0.0f;
        for (size_t k = 0; k < c; k++) { float d = v[k] - m; q += d * d; }
        float var = q / (float)c;
        float r = sqrtf(var + eps);
        for (size_t k = 0; k < c; k++) y[px * c + k] = (v[k] - m) / r * gamma[k] + beta[k];
    }
}

/* layers.rs:254-294 (softmax_scalar, tier 3): maximum and sum in 8 lanes over
 * the whole groups of eight, the lanes then folded in order, the rest added
 * one value at a time; then multiplied by the reciprocal of the sum. */
static void softmax_row(float *v, size_t n) {
    size_t body = n / 8 * 8;
    float lanes[8];
    for (int l = 0; l < 8; l++) lanes[l] = -INFINITY;
    for (size_t j = 0; j < body; j++) { float a = lanes[j % 8]; lanes[j % 8] = a > v[j] ? a : v[j]; }
    float mx = -INFINITY;
    for (int l = 0; l < 8; l++) mx = fmaxf(mx, lanes[l]);
    for (size_t j = body; j < n; j++) mx = fmaxf(mx, v[j]);
    float sums[8] = {0};
    for (size_t j = 0; j < body; j++) { v[j] = orc_exp_neg(v[j] - mx); sums[j % 8] += v[j]; }
    float sum = 0.0f;
    for (int l = 0; l < 8; l++) sum += sums[l];
    for (size_t j = body; j < n; j++) { v[j] = orc_exp_neg(v[j] - mx); sum += v[j]; }
    float r = 1.0f / sum;
    for (size_t j = 0; j < n; j++) v[j] *= r;
}

/* softmax_row's operations, the eight lanes as one vector: the same lane
 * maxima and lane sums, the same final reductions in lane order. */
static void softmax_row_fast(float *v, size_t n) {
    size_t body = n / 8 * 8;
    __m256 lanes = _mm256_set1_ps(-INFINITY);
    for (size_t j = 0; j < body; j += 8) {
        __m256 a = _mm256_loadu_ps(v + j);
        lanes = _mm256_blendv_ps(a, lanes, _mm256_cmp_ps(lanes, a, _CMP_GT_OQ));
    }
    float ln[8];
    _mm256_storeu_ps(ln, lanes);
    float mx = -INFINITY;
    for (int l = 0; l < 8; l++) mx = fmaxf(mx, ln[l]);
    for (size_t j = body; j < n; j++) mx = fmaxf(mx, v[j]);
    __m256 sums = _mm256_setzero_ps(), m8 = _mm256_set1_ps(mx);
    for (size_t j = 0; j < body; j += 8) {
        __m256 e = exp_neg8(_mm256_sub_ps(_mm256_loadu_ps(v + j), m8));
        _mm256_storeu_ps(v + j, e);
        sums = _mm256_add_ps(sums, e);
    }
    _mm256_storeu_ps(ln, sums);
    float sum = 0.0f;
    for (int l = 0; l < 8; l++) sum += ln[l];
    for (size_t j = body; j < n; j++) { v[j] = orc_exp_neg(v[j] - mx); sum += v[j]; }
    float r = 1.0f / sum;
    for (size_t j = 0; j < n; j++) v[j] *= r;
}

/* The timed path's attention for a head size of 9 to 16: attention's
 * products with the accumulators in registers. Scores run eight keys a
 * vector over a transposed copy of the head's keys, four queries at a time;
 * S V runs the head's 16 (masked) value columns as two vectors, four query
 * rows at a time. Every score and output keeps attention's chain (the head
 * dimension in order, then the keys in order). */
static void attention_fast(const float *x, float *y, size_t t, size_t c, size_t heads, float scale) {
    const size_t hd = c / heads, tp = (t + 7) / 8 * 8;
    const __m256i tailmask = _mm256_cmpgt_epi32(_mm256_set1_epi32((int)hd - 8), _mm256_setr_epi32(0, 1, 2, 3, 4, 5, 6, 7));
#pragma omp parallel for schedule(static)
    for (long hh = 0; hh < (long)heads; hh++) {
        size_t h = (size_t)hh;
        float *q = malloc(t * hd * sizeof(float)), *kt = calloc(hd * tp, sizeof(float));
        float *scores = malloc(t * tp * sizeof(float));
        for (size_t s = 0; s < t; s++)
            for (size_t d = 0; d < hd; d++) q[s * hd + d] = x[s * 3 * c + h * hd + d] * scale;
        for (size_t j = 0; j < t; j++)
            for (size_t d = 0; d < hd; d++) kt[d * tp + j] = x[j * 3 * c + c + h * hd + d];
        size_t s = 0;
        for (; s < t; s += 4) {
            const size_t rows = t - s < 4 ? t - s : 4;
            for (size_t j = 0; j < tp; j += 8) {
                __m256 acc[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps()};
                for (size_t d = 0; d < hd; d++) {
                    __m256 kv = _mm256_loadu_ps(kt + d * tp + j);
                    for (size_t r = 0; r < 4; r++)
                        if (r < rows) acc[r] = _mm256_fmadd_ps(kv, _mm256_broadcast_ss(q + (s + r) * hd + d), acc[r]);
                }
                for (size_t r = 0; r < rows; r++) _mm256_storeu_ps(scores + (s + r) * tp + j, acc[r]);
            }
        }
        for (size_t i = 0; i < t; i++) softmax_row_fast(scores + i * tp, t);
        const float *v = x + 2 * c + h * hd;
        for (size_t i = 0; i < t; i += 4) {
            const size_t rows = t - i < 4 ? t - i : 4;
            __m256 a0[4], a1[4];
            for (int r = 0; r < 4; r++) { a0[r] = _mm256_setzero_ps(); a1[r] = _mm256_setzero_ps(); }
            for (size_t j = 0; j < t; j++) {
                __m256 v0 = _mm256_loadu_ps(v + j * 3 * c), v1 = _mm256_maskload_ps(v + j * 3 * c + 8, tailmask);
                for (size_t r = 0; r < 4; r++)
                    if (r < rows) {
                        __m256 pr = _mm256_broadcast_ss(scores + (i + r) * tp + j);
                        a0[r] = _mm256_fmadd_ps(v0, pr, a0[r]);
                        a1[r] = _mm256_fmadd_ps(v1, pr, a1[r]);
                    }
            }
            for (size_t r = 0; r < rows; r++) {
                float *out = y + (i + r) * c + h * hd;
                _mm256_storeu_ps(out, a0[r]);
                _mm256_maskstore_ps(out + 8, tailmask, a1[r]);
            }
        }
        free(q); free(kt); free(scores);
    }
}

/* layers.rs:494-522: per head, scores (Q * scale) K^T with sums over the
 * head dimension in order, a softmax per row, then S V with sums over the
 * keys in order (both products through pointwise_with, no bias). */
static void attention(const orc_plan *p, const orc_op *op, const float *x, float *y) {
    size_t t = op->iw, c = op->oc, heads = op->n2, hd = c / heads;
    float scale = *W(p, op->w0);
    if (g_fast && hd > 8 && hd <= 16) {
        attention_fast(x, y, t, c, heads, scale);
        return;
    }
    float *q = malloc(t * hd * sizeof(float)), *scores = malloc(t * t * sizeof(float));
    for (size_t h = 0; h < heads; h++) {
        for (size_t s = 0; s < t; s++)
            for (size_t d = 0; d < hd; d++) q[s * hd + d] = x[s * 3 * c + h * hd + d] * scale;
        for (size_t s = 0; s < t; s++) {
            float *row = scores + s * t;
            for (size_t j = 0; j < t; j++) {
                float acc = 0.0f;
                for (size_t d = 0; d < hd; d++) acc = fmaf(x[j * 3 * c + c + h * hd + d], q[s * hd + d], acc);
                row[j] = acc;
            }
            softmax_row(row, t);
        }
        for (size_t i = 0; i < t; i++)
            for (size_t d = 0; d < hd; d++) {
                float acc = 0.0f;
                for (size_t j = 0; j < t; j++) acc = fmaf(x[j * 3 * c + 2 * c + h * hd + d], scores[i * t + j], acc);
                y[i * c + h * hd + d] = acc;
            }
    }
    free(q); free(scores);
}

/* One panel's logits for ROWS time steps (bias first, inputs in order) and
 * each step's online-softmax update, the eight lanes at once: state holds
 * per step the lane maxima, sums and best columns (3 x 8 floats). */
static inline __attribute__((always_inline)) void head_panel(const float *panel, const float *bias, const float *xv,
                                                             size_t ci, float *state, float *y, size_t j,
                                                             size_t vocab, int probs, size_t step0, int rows) {
    __m256 acc[6][2];
    for (int r = 0; r < rows; r++) {
        acc[r][0] = _mm256_loadu_ps(bias);
        acc[r][1] = _mm256_loadu_ps(bias + 8);
    }
    for (size_t i = 0; i < ci; i++) {
        __m256 w0 = _mm256_loadu_ps(panel + i * 16), w1 = _mm256_loadu_ps(panel + i * 16 + 8);
        for (int r = 0; r < rows; r++) {
            __m256 xb = _mm256_broadcast_ss(xv + (size_t)r * ci + i);
            acc[r][0] = _mm256_fmadd_ps(w0, xb, acc[r][0]);
            acc[r][1] = _mm256_fmadd_ps(w1, xb, acc[r][1]);
        }
    }
    const __m256 col = _mm256_add_ps(_mm256_set1_ps((float)(j * 16)), _mm256_setr_ps(0, 1, 2, 3, 4, 5, 6, 7));
    for (int r = 0; r < rows; r++) {
        float *st = state + (size_t)r * 24;
        __m256 a0 = acc[r][0], a1 = acc[r][1];
        __m256 mm = _mm256_loadu_ps(st), sum = _mm256_loadu_ps(st + 8), best = _mm256_loadu_ps(st + 16);
        __m256 second = _mm256_cmp_ps(a1, a0, _CMP_GT_OQ);
        __m256 top = _mm256_blendv_ps(a1, a0, _mm256_cmp_ps(a0, a1, _CMP_GT_OQ));
        __m256 grown = _mm256_blendv_ps(top, mm, _mm256_cmp_ps(mm, top, _CMP_GT_OQ));
        /* where no lane's maximum moved (and each is finite) the rescale is
         * exp_neg(+-0) = 1 exactly, so the sum is kept as it is */
        const __m256 kept = _mm256_and_ps(_mm256_cmp_ps(grown, mm, _CMP_EQ_OQ),
                                          _mm256_cmp_ps(_mm256_andnot_ps(_mm256_set1_ps(-0.0f), mm),
                                                        _mm256_set1_ps(INFINITY), _CMP_LT_OQ));
        __m256 sn = _mm256_movemask_ps(kept) == 0xff ? sum : _mm256_mul_ps(sum, exp_neg8(_mm256_sub_ps(mm, grown)));
        sn = _mm256_add_ps(sn, exp_neg8(_mm256_sub_ps(a0, grown)));
        sn = _mm256_add_ps(sn, exp_neg8(_mm256_sub_ps(a1, grown)));
        __m256 c = _mm256_add_ps(col, _mm256_and_ps(second, _mm256_set1_ps(8.0f)));
        best = _mm256_blendv_ps(best, c, _mm256_cmp_ps(top, mm, _CMP_GT_OQ));
        _mm256_storeu_ps(st, grown);
        _mm256_storeu_ps(st + 8, sn);
        _mm256_storeu_ps(st + 16, best);
        if (probs) {
            float logits[16];
            _mm256_storeu_ps(logits, a0);
            _mm256_storeu_ps(logits + 8, a1);
            size_t n = vocab - j * 16 < 16 ? vocab - j * 16 : 16;
            memcpy(y + (step0 + (size_t)r) * vocab + j * 16, logits, n * sizeof(float));
        }
    }
}

/* The timed path's CTC head, as the reference's tier-3 head runs it: each
 * 16-column panel stays in cache while every time step of the thread's
 * block passes through it (six steps a register tile), so the weights are
 * read once per block instead of once per step. Every step's logits and
 * lane updates are the ones ctc_head's per-step loop makes, in the same
 * order (panels in order), so the results are the same bits. */
static void head_fast(const float *w, const float *b, const float *x, float *y, size_t t, size_t ci, size_t vocab,
                      int probs) {
    size_t npanels = (vocab + 15) / 16;
    float *state = malloc(t * 24 * sizeof(float));
    for (size_t pp = 0; pp < t; pp++)
        for (int l = 0; l < 8; l++) {
            state[pp * 24 + l] = -INFINITY;
            state[pp * 24 + 8 + l] = 0.0f;
            state[pp * 24 + 16 + l] = 0.0f;
        }
    long nthreads = omp_get_max_threads();
    long per = ((long)t + nthreads - 1) / nthreads;
    per = (per + 5) / 6 * 6;
    long blocks = per ? ((long)t + per - 1) / per : 0;
#pragma omp parallel for schedule(static)
    for (long blk = 0; blk < blocks; blk++) {
        size_t s0 = (size_t)(blk * per), s1 = s0 + (size_t)per < t ? s0 + (size_t)per : t;
        for (size_t j = 0; j < npanels; j++) {
            const float *panel = w + j * ci * 16, *bias = b + j * 16;
            size_t pp = s0;
            for (; pp + 6 <= s1; pp += 6)
                head_panel(panel, bias, x + pp * ci, ci, state + pp * 24, y, j, vocab, probs, pp, 6);
            for (; pp < s1; pp++)
                head_panel(panel, bias, x + pp * ci, ci, state + pp * 24, y, j, vocab, probs, pp, 1);
        }
    }
#pragma omp parallel for schedule(static)
    for (long q = 0; q < (long)t; q++) {
        size_t pp = (size_t)q;
        const float *m = state + pp * 24, *sum = m + 8, *best = m + 16;
        float mx = -INFINITY;
        for (int l = 0; l < 8; l++) mx = fmaxf(mx, m[l]);
        float total = 0.0f;
        for (int l = 0; l < 8; l++) total += sum[l] * orc_exp_neg(m[l] - mx);
        float rr = 1.0f / total;
        if (probs) {
            for (size_t k = 0; k < vocab; k++) y[pp * vocab + k] = orc_exp_neg(y[pp * vocab + k] - mx) * rr;
        } else {
            float bc = INFINITY;
            for (int l = 0; l < 8; l++) if (m[l] == mx && best[l] < bc) bc = best[l];
            y[2 * pp] = bc;
            y[2 * pp + 1] = rr;
        }
    }
    free(state);
}

/* layers.rs:692-832 (head_scalar, tier 3): logits from the bias, inputs
 * added in order; an online softmax in 8 lanes, lane l holding columns
 * 16j+l and 16j+8+l of panel j; the best column the first to reach the
 * maximum. probs: y = [t][vocab] probabilities; else [t][2] = (class, 1/sum). */
static void ctc_head(const orc_plan *p, const orc_op *op, const float *x, float *y, int probs) {
    size_t t = op->iw, ci = op->ic, vocab = probs ? op->oc : op->n2;
    size_t npanels = (vocab + 15) / 16;
    const float *w = W(p, op->w0), *b = W(p, op->b0);
    long tl = (long)t;
    if (g_fast) {
        head_fast(w, b, x, y, t, ci, vocab, probs);
        return;
    }
#pragma omp parallel for schedule(static)
    for (long pp = 0; pp < tl; pp++) {
        float m[8], sum[8], best[8], logits[16];
        for (int l = 0; l < 8; l++) { m[l] = -INFINITY; sum[l] = 0.0f; best[l] = 0.0f; }
        const float *xv = x + (size_t)pp * ci;
        for (size_t j = 0; j < npanels; j++) {
            const float *panel = w + j * ci * 16;
            for (int col = 0; col < 16; col++) {
                float acc = b[j * 16 + col];
                for (size_t i = 0; i < ci; i++) acc = fmaf(panel[i * 16 + col], xv[i], acc);
                logits[col] = acc;
            }
            for (int l = 0; l < 8; l++) {
                float a0 = logits[l], a1 = logits[8 + l], mm = m[l];
                float top = a0 > a1 ? a0 : a1;
                float grown = mm > top ? mm : top;
                float s = sum[l] * orc_exp_neg(mm - grown);
                s += orc_exp_neg(a0 - grown);
                s += orc_exp_neg(a1 - grown);
                m[l] = grown; sum[l] = s;
                if (top > mm) best[l] = (float)(j * 16 + l + (a1 > a0 ? 8 : 0));
            }
            if (probs) {
                size_t n = vocab - j * 16 < 16 ? vocab - j * 16 : 16;
                memcpy(y + (size_t)pp * vocab + j * 16, logits, n * sizeof(float));
            }
        }
        float mx = -INFINITY;
        for (int l = 0; l < 8; l++) mx = fmaxf(mx, m[l]);
        float total = 0.0f;
        for (int l = 0; l < 8; l++) total += sum[l] * orc_exp_neg(m[l] - mx);
        float r = 1.0f / total;
        if (probs) {
            for (size_t k = 0; k < vocab; k++) y[(size_t)pp * vocab + k] = orc_exp_neg(y[(size_t)pp * vocab + k] - mx) * r;
        } else {
            float bc = INFINITY;
            for (int l = 0; l < 8; l++) if (m[l] == mx && best[l] < bc) bc = best[l];
            y[2 * pp] = bc;
            y[2 * pp + 1] = r;
        }
    }
}

/* layers.rs:595-680: each input pixel's channels times w [ic][kh][kw][oc]
 * give its kh x kw block of outputs (bias per tap, placed as a pointwise
 * layer of kh*kw*oc columns places it), then the tail. */
/* Columns c0 .. c0 + 8 * NV of one input pixel's block of a transposed
 * convolution, in registers, stored where they land in the output rows of
 * `out` (a column group never crosses a kernel row: kw * oc is a multiple
 * of eight). */
static inline __attribute__((always_inline)) void ct_cols(const orc_op *op, const float *px, const float *w,
                                                          const float *b, int first, float *out, size_t ix,
                                                          size_t c0, const int NV) {
    const size_t cols = op->kh * op->kw * op->oc, span = op->kw * op->oc;
    __m256 acc[8];
#pragma GCC unroll 8
    for (int v = 0; v < NV; v++) acc[v] = (b && first) ? _mm256_loadu_ps(b + c0 + 8 * v) : _mm256_setzero_ps();
    for (size_t i = 0; i < op->ic; i++) {
        __m256 xv = _mm256_broadcast_ss(px + i);
        const float *row = w + i * cols + c0;
#pragma GCC unroll 8
        for (int v = 0; v < NV; v++) acc[v] = _mm256_fmadd_ps(_mm256_loadu_ps(row + 8 * v), xv, acc[v]);
    }
#pragma GCC unroll 8
    for (int v = 0; v < NV; v++) {
        size_t c = c0 + 8 * (size_t)v, ky = c / span, k = c % span;
        __m256 a = acc[v];
        if (b && !first) a = _mm256_add_ps(a, _mm256_loadu_ps(b + c));
        _mm256_storeu_ps(out + (ky * op->ow + ix * op->kw) * op->oc + k, a);
    }
}

/* The timed path's transposed convolution: each input pixel's block of
 * kh*kw*oc outputs in registers (eight columns a lane group; four-column
 * blocks two pixels at a time, one per half), stored in place (the kw*oc
 * outputs of one kernel row lie side by side), the activation once per
 * output row pair. Every output keeps convtranspose's chain: the bias first
 * or last as there, then the input channels in order. */
static void convtranspose_fast(const orc_op *op, const float *w, const float *b, const float *x, float *y) {
    const size_t cols = op->kh * op->kw * op->oc, span = op->kw * op->oc, ic = op->ic;
    const int first = cols % 16 == 0;
    long rows = (long)op->ih;
#pragma omp parallel for schedule(static)
    for (long iy = 0; iy < rows; iy++) {
        float *out = y + (size_t)iy * op->kh * op->ow * op->oc;
        if (cols == 4) {
            const __m256 bias = b ? _mm256_setr_ps(b[0], b[1], b[2], b[3], b[0], b[1], b[2], b[3])
                                  : _mm256_setzero_ps();
            size_t ix = 0;
            for (; ix + 2 <= op->iw; ix += 2) {
                const float *p0 = x + ((size_t)iy * op->iw + ix) * ic, *p1 = p0 + ic;
                __m256 acc = (b && first) ? bias : _mm256_setzero_ps();
                for (size_t i = 0; i < ic; i++) {
                    __m128 wr = _mm_loadu_ps(w + i * 4);
                    __m256 wv = _mm256_set_m128(wr, wr);
                    __m256 xv = _mm256_set_m128(_mm_broadcast_ss(p1 + i), _mm_broadcast_ss(p0 + i));
                    acc = _mm256_fmadd_ps(wv, xv, acc);
                }
                if (b && !first) acc = _mm256_add_ps(acc, bias);
                float v[8];
                _mm256_storeu_ps(v, acc);
                for (size_t ky = 0; ky < op->kh; ky++) {
                    float *o = out + (ky * op->ow + ix * op->kw) * op->oc;
                    memcpy(o, v + ky * span, span * sizeof(float));
                    memcpy(o + span, v + 4 + ky * span, span * sizeof(float));
                }
            }
            for (; ix < op->iw; ix++) {
                const float *px = x + ((size_t)iy * op->iw + ix) * ic;
                float v[4];
                for (size_t o = 0; o < 4; o++) v[o] = (b && first) ? b[o] : 0.0f;
                for (size_t i = 0; i < ic; i++)
                    for (size_t o = 0; o < 4; o++) v[o] = fmaf(w[i * 4 + o], px[i], v[o]);
                if (b && !first)
                    for (size_t o = 0; o < 4; o++) v[o] += b[o];
                for (size_t ky = 0; ky < op->kh; ky++)
                    memcpy(out + (ky * op->ow + ix * op->kw) * op->oc, v + ky * span, span * sizeof(float));
            }
        } else {
            for (size_t ix = 0; ix < op->iw; ix++) {
                const float *px = x + ((size_t)iy * op->iw + ix) * ic;
                size_t c0 = 0;
                for (; c0 + 64 <= cols; c0 += 64) ct_cols(op, px, w, b, first, out, ix, c0, 8);
                for (; c0 + 32 <= cols; c0 += 32) ct_cols(op, px, w, b, first, out, ix, c0, 4);
                for (; c0 + 16 <= cols; c0 += 16) ct_cols(op, px, w, b, first, out, ix, c0, 2);
                for (; c0 + 8 <= cols; c0 += 8) ct_cols(op, px, w, b, first, out, ix, c0, 1);
            }
        }
        tail(out, op->kh * op->ow * op->oc, op->fused);
    }
}

static void convtranspose(const orc_plan *p, const orc_op *op, const float *x, float *y) {
    const float *w = W(p, op->w0), *b = op->b1 ? W(p, op->b0) : NULL;
    size_t cols = op->kh * op->kw * op->oc;
    long rows = (long)op->ih;
    if (g_fast && (cols == 4 || (cols % 8 == 0 && (op->kw * op->oc) % 8 == 0))) {
        convtranspose_fast(op, w, b, x, y);
        return;
    }
#pragma omp parallel for schedule(static)
    for (long iy = 0; iy < rows; iy++) {
        float *block = malloc(cols * sizeof(float));
        for (size_t ix = 0; ix < op->iw; ix++) {
            const float *px = x + ((size_t)iy * op->iw + ix) * op->ic;
            int first = cols % 16 == 0;
            for (size_t o = 0; o < cols; o++) block[o] = (b && first) ? b[o] : 0.0f;
            for (size_t i = 0; i < op->ic; i++)
                for (size_t o = 0; o < cols; o++) block[o] = fmaf(w[i * cols + o], px[i], block[o]);
            if (b && !first)
                for (size_t o = 0; o < cols; o++) block[o] += b[o];
            tail(block, cols, op->fused);
            for (size_t ky = 0; ky < op->kh; ky++)
                for (size_t kx = 0; kx < op->kw; kx++) {
                    size_t oy = (size_t)iy * op->kh + ky, ox = ix * op->kw + kx;
                    memcpy(y + (oy * op->ow + ox) * op->oc, block + (ky * op->kw + kx) * op->oc,
                           op->oc * sizeof(float));
                }
        }
        free(block);
    }
}

/* ----------------------------------------------------------------- execute */

int orc_run(orc_plan *p, const float *input, float *const *outputs, int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
    if (!p->kept) {
        p->kept = calloc(p->nbuf, sizeof(float *));
        p->kept_n = calloc(p->nbuf, sizeof(size_t));
        if (!p->kept || !p->kept_n) return -1;
    }
    float **buf = p->kept;
    int rc = 0;
    for (size_t b = 0; b < p->nbuf; b++) {
        const size_t need = p->pool[b] ? p->pool[b] : 1;
        if (p->kept_n[b] < need) {
            free(buf[b]);
            buf[b] = malloc(need * sizeof(float));
            p->kept_n[b] = buf[b] ? need : 0;
        }
        if (!buf[b]) { rc = -1; goto done; }
    }
    memcpy(buf[p->slot], input, orc_input_len(p) * sizeof(float));
    for (size_t i = 0; i < p->nops; i++) {
        const orc_op *op = &p->ops[i];
        const float *x = buf[op->x], *x2 = has_second(op) ? buf[op->x2] : NULL;
        float *y = buf[op->y];
        size_t n = op->oh * op->ow * op->oc;
        switch (op->kind) {
        case K_CONV:
            if (g_fast && op->oc % 8 == 0 && i + 1 < p->nops && p->ops[i + 1].kind == K_MEAN &&
                p->ops[i + 1].x == op->y && p->ops[i + 1].y != op->y && p->ops[i + 1].ic == op->oc &&
                p->ops[i + 1].ih == op->oh && p->ops[i + 1].iw == op->ow) {
                conv_fast(p, op, x, x2, y, buf[p->ops[i + 1].y]); /* and the mean after it */
                i++;
                break;
            }
            conv(p, op, x, x2, y);
            break;
        case K_DWCONV: dwconv(p, op, x, y); break;
        case K_ADD: /* conv.rs:74-79 */
#pragma omp parallel for schedule(static)
            for (size_t k = 0; k < n; k++) y[k] = x[k] + x2[k];
            tail(y, n, op->fused);
            break;
        case K_MAXPOOL: maxpool(op, x, y); break;
        case K_AVGPOOL: avgpool(op, x, y); break;
        case K_CHANNELMUL: /* kernels/elementwise.rs:178-200 */
#pragma omp parallel for schedule(static)
            for (size_t px = 0; px < op->oh * op->ow; px++)
                for (size_t k = 0; k < op->oc; k++) y[px * op->oc + k] = x[px * op->oc + k] * x2[k];
            break;
        case K_CONCATC: /* layers.rs:375-381 */
#pragma omp parallel for schedule(static)
            for (size_t px = 0; px < op->oh * op->ow; px++) {
                memcpy(y + px * op->oc, x + px * op->ic, op->ic * sizeof(float));
                memcpy(y + px * op->oc + op->ic, x2 + px * op->n2, op->n2 * sizeof(float));
            }
            break;
        case K_LAYERNORM: layernorm(p, op, x, y); break;
        case K_ATTENTION: attention(p, op, x, y); break;
        case K_MEAN: mean(op, x, y); break;
        case K_CTCHEAD: ctc_head(p, op, x, y, 1); break;
        case K_CTCARGMAX: ctc_head(p, op, x, y, 0); break;
        case K_UPSAMPLE: case K_UPSAMPLEADD: /* layers.rs:526-565 */
#pragma omp parallel for schedule(static)
            for (size_t oy = 0; oy < op->oh; oy++)
                for (size_t ox = 0; ox < op->ow; ox++) {
                    const float *src = x + ((oy / op->sh) * op->iw + ox / op->sw) * op->oc;
                    float *dst = y + (oy * op->ow + ox) * op->oc;
                    if (op->kind == K_UPSAMPLE) memcpy(dst, src, op->oc * sizeof(float));
                    else {
                        const float *add = x2 + (oy * op->ow + ox) * op->oc;
                        for (size_t k = 0; k < op->oc; k++) dst[k] = add[k] + src[k];
                    }
                }
            break;
        case K_CONVTRANSPOSE: convtranspose(p, op, x, y); break;
        default: rc = -1; goto done;
        }
    }
    for (size_t k = 0; k < p->nout; k++) memcpy(outputs[k], buf[p->outputs[k]], p->out_n[k] * sizeof(float));
done:
    return rc;
}

/* ------------------------------------------------------------ det input */

/* One output coordinate of the bilinear resize (image.rs:34-63): output d
 * sits at source (d + 0.5) * src / dst - 0.5, computed in f64 and rounded to
 * f32; its two source indices are clamped to the edge, and each weight is
 * rounded to 1/2048 on its own (ties to even). */
typedef struct {
    size_t near, far;
    int near_w, far_w;
} orc_tap;

static orc_tap orc_resize_tap(size_t src, size_t dst, size_t d) {
    const double scale = 1.0 / ((double)dst / (double)src);
    const float f = (float)(((double)d + 0.5) * scale - 0.5);
    const float fl = floorf(f);
    const float a = f - fl;
    const long s = (long)fl, last = (long)src - 1;
    orc_tap t;
    t.near = (size_t)(s < 0 ? 0 : s > last ? last : s);
    t.far = (size_t)(s + 1 < 0 ? 0 : s + 1 > last ? last : s + 1);
    t.near_w = (int)rintf((1.0f - a) * 2048.0f);
    t.far_w = (int)rintf(a * 2048.0f);
    return t;
}

/* reference det.rs:230-292, image.rs:91-142: the horizontal pass keeps the
 * 1/2048 products, the vertical pass drops four bits of each row before
 * weighting and sixteen after, then rounds the sum of the two; the byte then
 * goes through ((f64)(byte * (f32)(1/255)) - mean) / std, rounded to f32. */
int orc_det_input_hwc(const unsigned char *image, size_t iw, size_t ih, size_t ow, size_t oh, const double *mean,
                      const double *std, float *out) {
    if (!iw || !ih || !ow || !oh) return 1;
    const float scale = (float)(1.0 / 255.0);
    /* the reference's per-channel table of the 256 byte values (det.rs:239-241)
     * and the column taps, computed once; bands of rows over the threads */
    float table[3][256];
    for (int c = 0; c < 3; c++)
        for (int v = 0; v < 256; v++) table[c][v] = (float)(((double)((float)v * scale) - mean[c]) / std[c]);
    orc_tap *tx = malloc(ow * sizeof(orc_tap));
    if (!tx) return 1;
    for (size_t ox = 0; ox < ow; ox++) tx[ox] = orc_resize_tap(iw, ow, ox);
#pragma omp parallel for schedule(static)
    for (long y = 0; y < (long)oh; y++) {
        const size_t oy = (size_t)y;
        const orc_tap ty = orc_resize_tap(ih, oh, oy);
        const unsigned char *r0 = image + ty.near * iw * 3, *r1 = image + ty.far * iw * 3;
        float *o = out + oy * ow * 3;
        for (size_t ox = 0; ox < ow; ox++) {
            const orc_tap t = tx[ox];
            for (int c = 0; c < 3; c++) {
                const int a = (int)r0[t.near * 3 + c] * t.near_w + (int)r0[t.far * 3 + c] * t.far_w;
                const int b = (int)r1[t.near * 3 + c] * t.near_w + (int)r1[t.far * 3 + c] * t.far_w;
                const int v = (((a >> 4) * ty.near_w) >> 16) + (((b >> 4) * ty.far_w) >> 16);
                int byte = (v + 2) >> 2;
                byte = byte < 0 ? 0 : byte > 255 ? 255 : byte;
                o[ox * 3 + c] = table[c][byte];
            }
        }
    }
    free(tx);
    return 0;
}

/* reference rec.rs:19-43: width = trunc(48 * max(320 / 48, w / h)); the
 * resized width ceil(48 * w / h), cut to the width; (v / 255 - 0.5) / 0.5 in
 * f32; zeros on the right. */
size_t orc_rec_input_hwc(const unsigned char *crop, size_t cw, size_t ch, float *out) {
    if (!cw || !ch) return 0;
    const double h = (double)ch, w = (double)cw, height = 48.0;
    const double ratio = 320.0 / height > w / h ? 320.0 / height : w / h;
    const size_t width = (size_t)(height * ratio);
    const double fitted = ceil(height * (w / h));
    const size_t rw = fitted > (double)width ? width : (size_t)fitted;
    if (!out) return width;
    float table[256];
    for (int v = 0; v < 256; v++) table[v] = ((float)v / 255.0f - 0.5f) / 0.5f;
    orc_tap *tx = malloc((rw ? rw : 1) * sizeof(orc_tap));
    if (!tx) return 0;
    for (size_t ox = 0; ox < rw; ox++) tx[ox] = orc_resize_tap(cw, rw, ox);
    for (size_t oy = 0; oy < 48; oy++) {
        const orc_tap ty = orc_resize_tap(ch, 48, oy);
        const unsigned char *r0 = crop + ty.near * cw * 3, *r1 = crop + ty.far * cw * 3;
        float *o = out + oy * width * 3;
        for (size_t ox = 0; ox < rw; ox++) {
            const orc_tap t = tx[ox];
            for (int c = 0; c < 3; c++) {
                const int a = (int)r0[t.near * 3 + c] * t.near_w + (int)r0[t.far * 3 + c] * t.far_w;
                const int b = (int)r1[t.near * 3 + c] * t.near_w + (int)r1[t.far * 3 + c] * t.far_w;
                const int v = (((a >> 4) * ty.near_w) >> 16) + (((b >> 4) * ty.far_w) >> 16);
                int byte = (v + 2) >> 2;
                byte = byte < 0 ? 0 : byte > 255 ? 255 : byte;
                o[ox * 3 + c] = table[byte];
            }
        }
        for (size_t k = rw * 3; k < width * 3; k++) o[k] = 0.0f;
    }
    free(tx);
    return width;
}
