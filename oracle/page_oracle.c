/* TEST INFRASTRUCTURE ONLY: the CPU oracle of ppocr-native's host page
 * steps, for parity tests and bench.py's reference arm. The product library
 * never links, loads or calls it.
 *
 * A plain C restatement, function by function, of the reference's page
 * steps around the two networks: OpenCV's bilinear resize and the quarter
 * turn (src/image.rs), page preparation and the DB postprocess (src/det.rs),
 * border following and the contour mean (src/contour.rs), minimum-area
 * rectangles and the unclip offset (src/geometry.rs), the perspective crop
 * (src/crop.rs), the CTC decode's score (src/rec.rs) and the page-line
 * mapping (src/lib.rs). Every float operation is written in the reference's
 * order and precision (compiled with -ffp-contract=off), because the
 * reference matches OpenCV / pyclipper / numpy bit for bit and its fixtures
 * (tests/fixtures, asserted by tests/parity.rs) pin exactly those bits.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "ppocr_oracle.h"

/* ---------------------------------------------------------------- resize */

typedef struct {
    size_t near, far;
    int near_w, far_w;
} pg_tap;

/* image.rs:46-63 taps: output d at source (d + 0.5) * scale - 0.5 rounded
 * to f32, edge-clamped indices, each weight rounded to 1/2048 on its own. */
static pg_tap pg_tap_of(size_t src, size_t dst, size_t d) {
    const double scale = 1.0 / ((double)dst / (double)src);
    const float f = (float)(((double)d + 0.5) * scale - 0.5);
    const float fl = floorf(f);
    const float a = f - fl;
    const long s = (long)fl, last = (long)src - 1;
    pg_tap t;
    t.near = (size_t)(s < 0 ? 0 : s > last ? last : s);
    t.far = (size_t)(s + 1 < 0 ? 0 : s + 1 > last ? last : s + 1);
    t.near_w = (int)rintf((1.0f - a) * 2048.0f);
    t.far_w = (int)rintf(a * 2048.0f);
    return t;
}

/* image.rs:91-142 resize_linear_rows over every row: the horizontal pass
 * keeps the 1/2048 products, the vertical one drops 4 bits before and 16
 * after weighting, then rounds the sum. */
int orc_resize_linear(const uint8_t *image, size_t iw, size_t ih, size_t ow, size_t oh, uint8_t *out) {
    if (!iw || !ih || !ow || !oh) return 1;
    pg_tap *xs = malloc(ow * sizeof(pg_tap));
    if (!xs) return 1;
    for (size_t x = 0; x < ow; x++) xs[x] = pg_tap_of(iw, ow, x);
    for (size_t y = 0; y < oh; y++) {
        const pg_tap ty = pg_tap_of(ih, oh, y);
        const uint8_t *r0 = image + ty.near * iw * 3, *r1 = image + ty.far * iw * 3;
        for (size_t x = 0; x < ow; x++) {
            const pg_tap tx = xs[x];
            for (int c = 0; c < 3; c++) {
                const int a = (int)r0[tx.near * 3 + c] * tx.near_w + (int)r0[tx.far * 3 + c] * tx.far_w;
                const int b = (int)r1[tx.near * 3 + c] * tx.near_w + (int)r1[tx.far * 3 + c] * tx.far_w;
                const int v = (((a >> 4) * ty.near_w) >> 16) + (((b >> 4) * ty.far_w) >> 16);
                const int byte = (v + 2) >> 2;
                out[(y * ow + x) * 3 + c] = (uint8_t)(byte < 0 ? 0 : byte > 255 ? 255 : byte);
            }
        }
    }
    free(xs);
    return 0;
}

/* image.rs:145-155 rotate_ccw (np.rot90): out is h wide, w tall. */
void orc_rotate_ccw(const uint8_t *image, size_t w, size_t h, uint8_t *out) {
    size_t k = 0;
    for (size_t col = w; col-- > 0;)
        for (size_t row = 0; row < h; row++) {
            memcpy(out + k, image + (row * w + col) * 3, 3);
            k += 3;
        }
}

/* ------------------------------------------------------- page preparation */

/* det.rs:12-14: Python's int(round(x / 32) * 32), halves to even. */
static size_t pg_snap32(size_t x) { return (size_t)nearbyint((double)x / 32.0) * 32; }

/* det.rs:19-26 scaled_size; 0 when a side vanishes. */
static int pg_scaled_size(size_t w, size_t h, double ratio, size_t *ow, size_t *oh) {
    if (!w || !h) return 0;
    *ow = pg_snap32((size_t)((double)w * ratio));
    *oh = pg_snap32((size_t)((double)h * ratio));
    return *ow > 0 && *oh > 0;
}

/* det.rs:166-193 det_size with Limit::Max (limit_min = 0) or Limit::Min. */
int orc_det_size(size_t w, size_t h, size_t limit_min, size_t *ow, size_t *oh) {
    double ratio;
    if (!limit_min) {
        const size_t lng = w > h ? w : h;
        const size_t side = lng < 960 ? 960 : lng < 1500 ? 1500 : 2000;
        ratio = lng > side ? (double)side / (double)lng : 1.0;
    } else {
        const size_t shrt = w < h ? w : h;
        ratio = shrt < limit_min ? (double)limit_min / (double)shrt : 1.0;
    }
    return pg_scaled_size(w, h, ratio, ow, oh);
}

/* det.rs:95-104 band_height. */
static size_t pg_band(size_t w, size_t h, double whr, size_t min_height) {
    const int too_wide = whr != -1.0 && (double)w / (double)h > whr;
    if (h > min_height && !too_wide) return 0;
    /* Rust's `as usize`: negative and NaN give 0, too large saturates */
    const double t = (double)w / whr;
    size_t target = t > 0.0 ? (t >= 1.8e19 ? SIZE_MAX : (size_t)t) : 0;
    if (target < min_height) target = min_height;
    target = target > SIZE_MAX / 2 ? SIZE_MAX : target * 2;
    const size_t diff = target > h ? target - h : h - target;
    return diff / 2;
}

/* det.rs:44-70 fit_page + det.rs:110-131 prepare_page, sizes only: the
 * fitted size, the ratios and the band. Returns 0 when there is no page. */
int orc_prepare_page(size_t w, size_t h, size_t min_side, size_t max_side, double whr, size_t min_height,
                     size_t *fw, size_t *fh, double *ratio_h, double *ratio_w, size_t *pad_top) {
    size_t cw = w, ch = h;
    int resized = 0;
    if ((w > h ? w : h) > max_side) {
        const double ratio = (double)max_side / (double)(h > w ? h : w);
        if (!pg_scaled_size(w, h, ratio, &cw, &ch)) return 0;
        resized = 1;
    }
    double rh = 1.0, rw = 1.0;
    if ((cw < ch ? cw : ch) < min_side) {
        const double ratio = (double)min_side / (double)(ch < cw ? ch : cw);
        size_t rw2, rh2;
        if (!pg_scaled_size(cw, ch, ratio, &rw2, &rh2)) return 0;
        rh = (double)ch / (double)rh2;
        rw = (double)cw / (double)rw2;
        cw = rw2;
        ch = rh2;
    } else if (resized) {
        rh = (double)h / (double)ch;
        rw = (double)w / (double)cw;
    }
    const size_t pad = pg_band(cw, ch, whr, min_height);
    const size_t padded = pad > (SIZE_MAX - ch) / 2 ? SIZE_MAX : 2 * pad + ch;
    const size_t area = max_side > 0 && max_side > SIZE_MAX / max_side ? SIZE_MAX : max_side * max_side;
    if (padded && cw > area / padded) return 0;
    *fw = cw;
    *fh = ch + 2 * pad;
    *ratio_h = rh;
    *ratio_w = rw;
    *pad_top = pad;
    return 1;
}

/* ------------------------------------------------------------- contours */

enum { PG_BACKGROUND = 0, PG_UNSEEN = 1, PG_MARKED = 2, PG_MARKED_EAST = 3 };

struct orc_contours {
    size_t n, np;
    size_t *start; /* n + 1 offsets into pts (points) */
    int32_t *pts;  /* [np][2] */
};

static int pg_push(orc_contours *c, size_t *cap_n, size_t *cap_p, const int32_t *pts, size_t k) {
    if (c->n + 2 > *cap_n) {
        size_t nc = *cap_n * 2 + 16;
        size_t *s = realloc(c->start, nc * sizeof(size_t));
        if (!s) return 1;
        c->start = s;
        *cap_n = nc;
    }
    if (c->np + k > *cap_p) {
        size_t nc = (*cap_p + k) * 2 + 64;
        int32_t *p = realloc(c->pts, nc * 2 * sizeof(int32_t));
        if (!p) return 1;
        c->pts = p;
        *cap_p = nc;
    }
    memcpy(c->pts + 2 * c->np, pts, k * 2 * sizeof(int32_t));
    c->np += k;
    c->n++;
    c->start[c->n] = c->np;
    return 0;
}

/* contour.rs:44-130 find_contours: Suzuki-Abe border following on a frame
 * of background, cv2.RETR_LIST + CHAIN_APPROX_SIMPLE, the borders found last
 * listed first. */
orc_contours *orc_find_contours(const uint8_t *mask, size_t width, size_t height) {
    static const int STEPS[8][2] = {{1, 0}, {1, -1}, {0, -1}, {-1, -1}, {-1, 0}, {-1, 1}, {0, 1}, {1, 1}};
    const size_t stride = width + 2;
    uint8_t *state = calloc(stride * (height + 2), 1);
    orc_contours *c = calloc(1, sizeof(orc_contours));
    size_t cap_n = 0, cap_p = 0, cap_chain = 0;
    size_t *chain_at = NULL;
    int *chain_dir = NULL;
    int32_t *corners = NULL;
    if (!state || !c) goto fail;
    c->start = calloc(1, sizeof(size_t));
    if (!c->start) goto fail;
    cap_n = 1;
    for (size_t y = 0; y < height; y++)
        for (size_t x = 0; x < width; x++)
            state[(y + 1) * stride + x + 1] = mask[y * width + x] ? PG_UNSEEN : PG_BACKGROUND;
    long off[8];
    for (int d = 0; d < 8; d++) off[d] = STEPS[d][0] + STEPS[d][1] * (long)stride;
    for (size_t y = 1; y <= height; y++) {
        for (size_t x = 1; x <= width; x++) {
            const size_t start = y * stride + x;
            const uint8_t here = state[start];
            int from;
            if (here == PG_UNSEEN && state[start - 1] == PG_BACKGROUND)
                from = 4; /* west */
            else if ((here == PG_UNSEEN || here == PG_MARKED) && state[start + 1] == PG_BACKGROUND)
                from = 0; /* east */
            else
                continue;
            int last_dir = -1;
            for (int k = 0; k < 8; k++) {
                const int d = (from + 8 - k) % 8;
                if (state[start + off[d]] != PG_BACKGROUND) {
                    last_dir = d;
                    break;
                }
            }
            if (last_dir < 0) {
                state[start] = PG_MARKED_EAST;
                int32_t p[2] = {(int32_t)(start % stride) - 1, (int32_t)(start / stride) - 1};
                if (pg_push(c, &cap_n, &cap_p, p, 1)) goto fail;
                continue;
            }
            const size_t last = start + off[last_dir];
            size_t n = 0, cur = start;
            int back = last_dir;
            for (;;) {
                int east_bg = 0, next_dir = back;
                for (int k = 1; k <= 8; k++) {
                    const int d = (back + k) % 8;
                    if (state[cur + off[d]] != PG_BACKGROUND) {
                        next_dir = d;
                        break;
                    }
                    if (d == 0) east_bg = 1;
                }
                if (east_bg)
                    state[cur] = PG_MARKED_EAST;
                else if (state[cur] == PG_UNSEEN)
                    state[cur] = PG_MARKED;
                if (n == cap_chain) {
                    cap_chain = cap_chain * 2 + 64;
                    size_t *a = realloc(chain_at, cap_chain * sizeof(size_t));
                    int *b = realloc(chain_dir, cap_chain * sizeof(int));
                    if (a) chain_at = a;
                    if (b) chain_dir = b;
                    if (!a || !b) goto fail;
                }
                chain_at[n] = cur;
                chain_dir[n] = next_dir;
                n++;
                const size_t next = cur + off[next_dir];
                if (next == start && cur == last) break;
                back = (next_dir + 4) % 8;
                cur = next;
            }
            /* the pixels where the step direction changes, from the first such */
            size_t first = 0, k = 0;
            for (size_t i = 0; i < n; i++)
                if (chain_dir[i] != chain_dir[(i + n - 1) % n]) {
                    first = i;
                    break;
                }
            int32_t *cs = realloc(corners, (n + 1) * 2 * sizeof(int32_t));
            if (!cs) goto fail;
            corners = cs;
            for (size_t j = 0; j < n; j++) {
                const size_t i = (first + j) % n;
                if (chain_dir[i] != chain_dir[(i + n - 1) % n]) {
                    corners[2 * k] = (int32_t)(chain_at[i] % stride) - 1;
                    corners[2 * k + 1] = (int32_t)(chain_at[i] / stride) - 1;
                    k++;
                }
            }
            if (pg_push(c, &cap_n, &cap_p, corners, k)) goto fail;
        }
    }
    free(state);
    free(chain_at);
    free(chain_dir);
    free(corners);
    /* reverse the list (contours.reverse()) */
    {
        int32_t *pts = malloc((c->np ? c->np : 1) * 2 * sizeof(int32_t));
        size_t *st = malloc((c->n + 1) * sizeof(size_t));
        if (!pts || !st) {
            free(pts);
            free(st);
            orc_contours_free(c);
            return NULL;
        }
        size_t at = 0;
        st[0] = 0;
        for (size_t i = 0; i < c->n; i++) {
            const size_t src = c->n - 1 - i, len = c->start[src + 1] - c->start[src];
            memcpy(pts + 2 * at, c->pts + 2 * c->start[src], len * 2 * sizeof(int32_t));
            at += len;
            st[i + 1] = at;
        }
        free(c->pts);
        free(c->start);
        c->pts = pts;
        c->start = st;
    }
    return c;
fail:
    free(state);
    free(chain_at);
    free(chain_dir);
    free(corners);
    orc_contours_free(c);
    return NULL;
}

size_t orc_contours_count(const orc_contours *c) { return c ? c->n : 0; }

const int32_t *orc_contour(const orc_contours *c, size_t i, size_t *len) {
    *len = c->start[i + 1] - c->start[i];
    return c->pts + 2 * c->start[i];
}

void orc_contours_free(orc_contours *c) {
    if (!c) return;
    free(c->start);
    free(c->pts);
    free(c);
}

static int pg_cmp_int(const void *a, const void *b) {
    const int x = *(const int *)a, y = *(const int *)b;
    return (x > y) - (x < y);
}

/* contour.rs:142-199 contour_mean: the map's f64 mean over the pixels on
 * the contour's edges or inside it by the even-odd rule along each row. */
double orc_contour_mean(const float *map, size_t width, size_t height, const int32_t *pts, size_t n) {
    const int W = (int)width, H = (int)height;
#define PG_CLAMP(v, hi) ((v) < 0 ? 0 : (v) > (hi) ? (hi) : (v))
    int mnx = 0, mxx = 0, mny = 0, mxy = 0;
    for (size_t i = 0; i < n; i++) {
        const int x = pts[2 * i], y = pts[2 * i + 1];
        if (i == 0 || x < mnx) mnx = x;
        if (i == 0 || x > mxx) mxx = x;
        if (i == 0 || y < mny) mny = y;
        if (i == 0 || y > mxy) mxy = y;
    }
    const int x0 = PG_CLAMP(mnx, W - 1), x1 = PG_CLAMP(mxx, W - 1);
    const int y0 = PG_CLAMP(mny, H - 1), y1 = PG_CLAMP(mxy, H - 1);
#undef PG_CLAMP
    const size_t w = (size_t)(x1 - x0 + 1), h = (size_t)(y1 - y0 + 1);
    uint8_t *inside = calloc(w * h, 1);
    int *cross = malloc((n + 1) * sizeof(int));
    if (!inside || !cross) {
        free(inside);
        free(cross);
        return NAN;
    }
#define PG_MARK(X, Y)                                                   \
    do {                                                                \
        const int mx_ = (X), my_ = (Y);                                 \
        if (mx_ >= x0 && mx_ <= x1 && my_ >= y0 && my_ <= y1)           \
            inside[(size_t)(my_ - y0) * w + (size_t)(mx_ - x0)] = 1;    \
    } while (0)
    for (size_t e = 0; e < n; e++) {
        const int32_t *a = pts + 2 * e, *b = pts + 2 * ((e + 1) % n);
        const int dx = b[0] - a[0], dy = b[1] - a[1];
        const int adx = dx < 0 ? -dx : dx, ady = dy < 0 ? -dy : dy;
        const int m = adx > ady ? adx : ady;
        const int sx = (dx > 0) - (dx < 0), sy = (dy > 0) - (dy < 0);
        for (int i = 0; i <= m; i++) PG_MARK(a[0] + sx * i, a[1] + sy * i);
    }
    for (int y = y0; y <= y1; y++) {
        size_t k = 0;
        for (size_t e = 0; e < n; e++) {
            const int32_t *a = pts + 2 * e, *b = pts + 2 * ((e + 1) % n);
            const int32_t *lo = a[1] < b[1] ? a : b, *hi = a[1] < b[1] ? b : a;
            if (lo[1] <= y && y < hi[1]) cross[k++] = lo[0] + (y - lo[1]) * (hi[0] - lo[0]) / (hi[1] - lo[1]);
        }
        qsort(cross, k, sizeof(int), pg_cmp_int);
        for (size_t j = 0; j + 1 < k; j += 2)
            for (int x = cross[j]; x <= cross[j + 1]; x++) PG_MARK(x, y);
    }
#undef PG_MARK
    double sum = 0.0;
    size_t count = 0;
    for (size_t r = 0; r < h; r++) {
        const float *line = map + ((size_t)y0 + r) * width + (size_t)x0;
        for (size_t i = 0; i < w; i++)
            if (inside[r * w + i]) {
                sum += (double)line[i];
                count++;
            }
    }
    free(inside);
    free(cross);
    return count ? sum / (double)count : 0.0;
}

/* ------------------------------------------------------------- geometry */

static int64_t pg_cross(const int32_t *o, const int32_t *a, const int32_t *b) {
    const int64_t ux = (int64_t)a[0] - o[0], uy = (int64_t)a[1] - o[1];
    const int64_t vx = (int64_t)b[0] - o[0], vy = (int64_t)b[1] - o[1];
    return ux * vy - uy * vx;
}

static const int32_t *pg_sort_pts;
static int pg_cmp_idx(const void *a, const void *b) {
    const size_t i = *(const size_t *)a, j = *(const size_t *)b;
    const int32_t *p = pg_sort_pts + 2 * i, *q = pg_sort_pts + 2 * j;
    if (p[0] != q[0]) return p[0] < q[0] ? -1 : 1;
    if (p[1] != q[1]) return p[1] < q[1] ? -1 : 1;
    return (i > j) - (i < j); /* stable */
}

/* One side of Andrew's monotone chain without its last point
 * (geometry.rs:273-285). Returns its length. */
static size_t pg_chain(const int32_t *pts, const size_t *seq, size_t n, int rev, size_t *h) {
    size_t k = 0;
    for (size_t t = 0; t < n; t++) {
        const size_t i = rev ? seq[n - 1 - t] : seq[t];
        while (k >= 2 && pg_cross(pts + 2 * h[k - 2], pts + 2 * h[k - 1], pts + 2 * i) <= 0) k--;
        h[k++] = i;
    }
    return k ? k - 1 : 0;
}

/* geometry.rs:263-320 hull_order: cv2.convexHull's indices in its order.
 * Returns the count written to out (capacity 2 n + 2). */
static size_t pg_hull_order(const int32_t *pts, size_t n, size_t *out) {
    size_t *order = malloc((n ? n : 1) * sizeof(size_t));
    size_t *tmp = malloc((2 * n + 2) * sizeof(size_t));
    size_t m = 0, len = 0;
    for (size_t i = 0; i < n; i++) order[i] = i;
    pg_sort_pts = pts;
    qsort(order, n, sizeof(size_t), pg_cmp_idx);
    for (size_t i = 0; i < n; i++) /* dedup, keeping the first of each run */
        if (m == 0 || pts[2 * order[m - 1]] != pts[2 * order[i]] || pts[2 * order[m - 1] + 1] != pts[2 * order[i] + 1])
            order[m++] = order[i];
    if (m < 3) {
        for (size_t i = 0; i < m; i++) out[i] = order[m - 1 - i];
        free(order);
        free(tmp);
        return m;
    }
    const size_t lo = pg_chain(pts, order, m, 0, tmp);
    size_t *lower = malloc((lo + 1) * sizeof(size_t));
    memcpy(lower, tmp, lo * sizeof(size_t));
    const size_t up = pg_chain(pts, order, m, 1, tmp);
    for (size_t i = 0; i < up; i++) out[len++] = tmp[i];
    for (size_t i = 0; i < lo; i++) out[len++] = lower[i];
    free(lower);
    free(order);
    free(tmp);
    const size_t hn = len;
    if (hn < 3) return hn;
    size_t lowest = 0, highest = 0, ascents = 0;
    for (size_t i = 1; i < hn; i++) {
        ascents += out[i - 1] < out[i];
        if (ascents > 1 && ascents + 1 < i) break;
        if (out[i] < out[lowest]) lowest = i;
        if (out[i] > out[highest]) highest = i;
    }
    const size_t gap = lowest > highest ? lowest - highest : highest - lowest;
    if ((gap == 1 || gap == hn - 1) && (ascents <= 1 || ascents + 2 >= hn)) {
        const int ascending = (highest + 1) % hn == lowest;
        const size_t first = ascending ? lowest : highest;
        size_t *rot = malloc(hn * sizeof(size_t));
        for (size_t k = 0; k < hn; k++) rot[k] = out[(first + k) % hn];
        int mono = 1;
        for (size_t k = 0; k + 1 < hn; k++)
            if ((rot[k] < rot[k + 1]) != ascending) mono = 0;
        if (first > 0 && mono) memcpy(out, rot, hn * sizeof(size_t));
        free(rot);
    }
    return hn;
}

/* geometry.rs:324-394 calipers: OpenCV's rotating calipers in f32. */
static void pg_calipers(const float (*p)[2], size_t n, float corner[2], float u[2], float v[2]) {
    float (*edge)[2] = malloc(n * sizeof(*edge));
    float *inv_len = malloc(n * sizeof(float));
    size_t left = 0, bottom = 0, right = 0, top = 0;
    for (size_t i = 0; i < n; i++) {
        const float *q = p[i], *r = p[(i + 1) % n];
        if (q[0] < p[left][0]) left = i;
        if (q[0] > p[right][0]) right = i;
        if (q[1] > p[top][1]) top = i;
        if (q[1] < p[bottom][1]) bottom = i;
        const double dx = (double)(r[0] - q[0]), dy = (double)(r[1] - q[1]);
        edge[i][0] = (float)dx;
        edge[i][1] = (float)dy;
        inv_len[i] = (float)(1.0 / sqrt(dx * dx + dy * dy));
    }
    size_t seq[4] = {bottom, right, top, left};
    float min_area = 3.40282347e+38f;
    size_t b_l = 0, b_bt = 0;
    float b_a = 0, b_w = 0, b_b = 0, b_h = 0;
    for (size_t it = 0; it < n; it++) {
        float e[4][2], t[4][2];
        for (int i = 0; i < 4; i++) {
            e[i][0] = edge[seq[i]][0];
            e[i][1] = edge[seq[i]][1];
        }
        t[0][0] = e[0][0]; t[0][1] = e[0][1];
        t[1][0] = e[1][1]; t[1][1] = -e[1][0];
        t[2][0] = -e[2][0]; t[2][1] = -e[2][1];
        t[3][0] = -e[3][1]; t[3][1] = e[3][0];
        int main_ = 0;
        for (int i = 1; i < 4; i++) {
            const float *vv = t[i], *ww = t[main_];
            const float s1 = vv[1] * ww[0];
            const float s2 = -vv[0] * ww[1];
            if (s1 + s2 < 0.0f) main_ = i;
        }
        const size_t k = seq[main_];
        const float lx = edge[k][0] * inv_len[k], ly = edge[k][1] * inv_len[k];
        float a, b;
        switch (main_) {
        case 0: a = lx; b = ly; break;
        case 1: a = ly; b = -lx; break;
        case 2: a = -lx; b = -ly; break;
        default: a = -ly; b = lx; break;
        }
        seq[main_] = (seq[main_] + 1) % n;
        const float w1 = (p[seq[1]][0] - p[seq[3]][0]) * a;
        const float w2 = (p[seq[1]][1] - p[seq[3]][1]) * b;
        const float width = w1 + w2;
        const float h1 = -(p[seq[2]][0] - p[seq[0]][0]) * b;
        const float h2 = (p[seq[2]][1] - p[seq[0]][1]) * a;
        const float height = h1 + h2;
        const float area = width * height;
        if (area <= min_area) {
            min_area = area;
            b_l = seq[3]; b_a = a; b_w = width; b_b = b; b_h = height; b_bt = seq[0];
        }
    }
    const float a1 = b_a, b1 = b_b, a2 = -b1, b2 = a1;
    const float c1 = a1 * p[b_l][0] + p[b_l][1] * b1;
    const float c2 = a2 * p[b_bt][0] + p[b_bt][1] * b2;
    const float inv_det = 1.0f / (a1 * b2 - a2 * b1);
    corner[0] = (c1 * b2 - c2 * b1) * inv_det;
    corner[1] = (a1 * c2 - a2 * c1) * inv_det;
    u[0] = a1 * b_w; u[1] = b1 * b_w;
    v[0] = a2 * b_h; v[1] = b2 * b_h;
    free(edge);
    free(inv_len);
}

/* geometry.rs:406-457 min_area_rect: rect = {cx, cy, width, height, angle}. */
void orc_min_area_rect(const int32_t *pts, size_t n, float rect[5]) {
    size_t *idx = malloc((2 * n + 2) * sizeof(size_t));
    const size_t hn = pg_hull_order(pts, n, idx);
    float (*hull)[2] = malloc((hn ? hn : 1) * sizeof(*hull));
    for (size_t i = 0; i < hn; i++) {
        hull[i][0] = (float)pts[2 * idx[i]];
        hull[i][1] = (float)pts[2 * idx[i] + 1];
    }
    double angle = -M_PI / 2;
    float cx = 0, cy = 0, w = 0, h = 0;
    if (hn == 1) {
        cx = hull[0][0];
        cy = hull[0][1];
    } else if (hn == 2) {
        const float *p = hull[0], *q = hull[1];
        cx = (p[0] + q[0]) * 0.5f;
        cy = (p[1] + q[1]) * 0.5f;
        const double dx = (double)(p[0] - q[0]), dy = (double)(p[1] - q[1]);
        const float size = (float)sqrt(dx * dx + dy * dy);
        if (dx == 0.0) {
            w = size;
        } else if (dy < 0.0) {
            angle = atan2(dy, dx);
            w = size;
        } else {
            if (dy > 0.0) angle = -atan2(dx, dy);
            h = size;
        }
    } else if (hn >= 3) {
        float corner[2], u[2], v[2];
        pg_calipers((const float (*)[2])hull, hn, corner, u, v);
        cx = corner[0] + (u[0] + v[0]) * 0.5f;
        cy = corner[1] + (u[1] + v[1]) * 0.5f;
        const float ul = (float)sqrt((double)u[0] * u[0] + (double)u[1] * u[1]);
        const float vl = (float)sqrt((double)v[0] * v[0] + (double)v[1] * v[1]);
        if (u[0] == 0.0f && u[1] > 0.0f) {
            w = ul;
            h = vl;
        } else {
            angle = -atan2((double)u[0], (double)u[1]);
            w = vl;
            h = ul;
        }
    }
    rect[0] = cx;
    rect[1] = cy;
    rect[2] = w;
    rect[3] = h;
    rect[4] = (float)(angle * 180.0 / M_PI);
    free(idx);
    free(hull);
}

/* geometry.rs:228-240 RotatedRect::points (cv2.boxPoints). */
void orc_box_points(const float rect[5], float quad[8]) {
    const double rad = (double)rect[4] * M_PI / 180.0;
    const float a = (float)sin(rad) * 0.5f, b = (float)cos(rad) * 0.5f;
    const float cx = rect[0], cy = rect[1], w = rect[2], h = rect[3];
    quad[0] = cx - a * h - b * w; quad[1] = cy + b * h - a * w;
    quad[2] = cx + a * h - b * w; quad[3] = cy - b * h - a * w;
    quad[4] = cx + a * h + b * w; quad[5] = cy - b * h + a * w;
    quad[6] = cx - a * h + b * w; quad[7] = cy + b * h + a * w;
}

/* f32 total order as Rust's total_cmp: -0 before +0. */
static int pg_total_lt(float a, float b) {
    int32_t x, y;
    memcpy(&x, &a, 4);
    memcpy(&y, &b, 4);
    x ^= (int32_t)(((uint32_t)(x >> 31)) >> 1);
    y ^= (int32_t)(((uint32_t)(y >> 31)) >> 1);
    return x < y;
}

/* geometry.rs:462-477 mini_box: corners tl, tr, br, bl; returns the shorter side. */
float orc_mini_box(const int32_t *pts, size_t n, float quad[8]) {
    float rect[5], p[4][2];
    orc_min_area_rect(pts, n, rect);
    float flat[8];
    orc_box_points(rect, flat);
    memcpy(p, flat, sizeof(flat));
    for (int i = 1; i < 4; i++) /* stable insertion sort by x */
        for (int j = i; j > 0 && pg_total_lt(p[j][0], p[j - 1][0]); j--) {
            float t0 = p[j][0], t1 = p[j][1];
            p[j][0] = p[j - 1][0]; p[j][1] = p[j - 1][1];
            p[j - 1][0] = t0; p[j - 1][1] = t1;
        }
    const float *tl, *bl, *tr, *br;
    if (p[1][1] > p[0][1]) { tl = p[0]; bl = p[1]; } else { tl = p[1]; bl = p[0]; }
    if (p[3][1] > p[2][1]) { tr = p[2]; br = p[3]; } else { tr = p[3]; br = p[2]; }
    quad[0] = tl[0]; quad[1] = tl[1]; quad[2] = tr[0]; quad[3] = tr[1];
    quad[4] = br[0]; quad[5] = br[1]; quad[6] = bl[0]; quad[7] = bl[1];
    return rect[2] < rect[3] ? rect[2] : rect[3];
}

/* geometry.rs:502-508 Clipper's rounding, half away from zero. */
static int32_t pg_clipper_round(double v) { return v < 0.0 ? (int32_t)(v - 0.5) : (int32_t)(v + 0.5); }

/* geometry.rs:611-634 clipper_cleanup, in place; returns the new length. */
static size_t pg_cleanup(int32_t *ring, size_t n) {
    while (n >= 3) {
        size_t found = n;
        for (size_t i = 0; i < n; i++) {
            const int32_t *prev = ring + 2 * ((i + n - 1) % n), *here = ring + 2 * i, *next = ring + 2 * ((i + 1) % n);
            if ((here[0] == next[0] && here[1] == next[1]) || pg_cross(prev, here, next) == 0) {
                found = i;
                break;
            }
        }
        if (found == n) break;
        memmove(ring + 2 * found, ring + 2 * (found + 1), (n - found - 1) * 2 * sizeof(int32_t));
        n--;
    }
    if (!n) return 0;
    int32_t top = ring[1];
    for (size_t i = 1; i < n; i++)
        if (ring[2 * i + 1] < top) top = ring[2 * i + 1];
    size_t last = n - 1;
    for (size_t i = 0; i < n; i++)
        if (ring[2 * i + 1] == top && ring[2 * ((i + 1) % n) + 1] != top) {
            last = i;
            break;
        }
    const size_t r = (last + 1) % n;
    if (r) {
        int32_t *tmp = malloc(n * 2 * sizeof(int32_t));
        for (size_t i = 0; i < n; i++) {
            tmp[2 * i] = ring[2 * ((i + r) % n)];
            tmp[2 * i + 1] = ring[2 * ((i + r) % n) + 1];
        }
        memcpy(ring, tmp, n * 2 * sizeof(int32_t));
        free(tmp);
    }
    return n;
}

/* geometry.rs:519-606 unclip: the quad grown by area * ratio / perimeter with
 * round joins (pyclipper JT_ROUND, arc tolerance 0.25). Writes at most cap
 * points; returns the count (0 for a degenerate quad), or -1 if cap is short. */
long orc_unclip(const float quad[8], double ratio, int32_t *out, size_t cap) {
    double p[4][2];
    for (int i = 0; i < 4; i++) {
        p[i][0] = (double)quad[2 * i];
        p[i][1] = (double)quad[2 * i + 1];
    }
    double sum = 0.0;
    for (int i = 1; i < 4; i++) sum += (p[i][0] - p[0][0]) * (p[i - 1][1] - p[(i + 1) % 4][1]);
    double perimeter = 0.0;
    for (int i = 0; i < 4; i++) {
        const double dx = p[(i + 1) % 4][0] - p[i][0], dy = p[(i + 1) % 4][1] - p[i][1];
        perimeter += sqrt(dx * dx + dy * dy);
    }
    const double area = fabs(sum / 2.0);
    const double delta = area * ratio / perimeter;
    double ring[4][2];
    size_t n = 0;
    for (int i = 0; i < 4; i++) {
        const double x = (double)truncf(quad[2 * i]), y = (double)truncf(quad[2 * i + 1]);
        if (n == 0 || ring[n - 1][0] != x || ring[n - 1][1] != y) {
            ring[n][0] = x;
            ring[n][1] = y;
            n++;
        }
    }
    while (n > 1 && ring[0][0] == ring[n - 1][0] && ring[0][1] == ring[n - 1][1]) n--;
    if (n < 3) return 0;
    if (fabs(delta) < 1e-20) {
        if (cap < n) return -1;
        for (size_t i = 0; i < n; i++) {
            out[2 * i] = (int32_t)ring[i][0];
            out[2 * i + 1] = (int32_t)ring[i][1];
        }
        return (long)pg_cleanup(out, n);
    }
    double signed_area = 0.0;
    for (size_t i = 0; i < n; i++)
        signed_area += ring[i][0] * ring[(i + 1) % n][1] - ring[(i + 1) % n][0] * ring[i][1];
    if (signed_area < 0.0)
        for (size_t i = 0; i < n / 2; i++) {
            double t0 = ring[i][0], t1 = ring[i][1];
            ring[i][0] = ring[n - 1 - i][0]; ring[i][1] = ring[n - 1 - i][1];
            ring[n - 1 - i][0] = t0; ring[n - 1 - i][1] = t1;
        }
    const double ad = fabs(delta);
    const double tolerance = 0.25 < ad * 0.25 ? 0.25 : ad * 0.25;
    double steps = M_PI / acos(1.0 - tolerance / ad);
    if (ad * M_PI < steps) steps = ad * M_PI;
    const double step_sin = sin(2 * M_PI / steps), step_cos = cos(2 * M_PI / steps);
    const double steps_per_rad = steps / (2 * M_PI);
    double normals[4][2];
    for (size_t i = 0; i < n; i++) {
        const double dx = ring[(i + 1) % n][0] - ring[i][0], dy = ring[(i + 1) % n][1] - ring[i][1];
        const double inv = 1.0 / sqrt(dx * dx + dy * dy);
        normals[i][0] = dy * inv;
        normals[i][1] = -dx * inv;
    }
    size_t k = n - 1, m = 0;
#define PG_OUT(X, Y)                    \
    do {                                \
        if (m >= cap) return -1;        \
        out[2 * m] = (X);               \
        out[2 * m + 1] = (Y);           \
        m++;                            \
    } while (0)
#define PG_AT(P, N) PG_OUT(pg_clipper_round((P)[0] + (N)[0] * delta), pg_clipper_round((P)[1] + (N)[1] * delta))
    for (size_t j = 0; j < n; j++) {
        const double *pp = ring[j], *nk = normals[k], *nj = normals[j];
        double sin_a = nk[0] * nj[1] - nj[0] * nk[1];
        const double cos_a = nk[0] * nj[0] + nk[1] * nj[1];
        if (fabs(sin_a * delta) < 1.0) {
            if (cos_a > 0.0) {
                PG_AT(pp, nk);
                continue;
            }
        } else {
            sin_a = sin_a < -1.0 ? -1.0 : sin_a > 1.0 ? 1.0 : sin_a;
        }
        if (sin_a * delta < 0.0) {
            PG_AT(pp, nk);
            PG_OUT((int32_t)pp[0], (int32_t)pp[1]);
            PG_AT(pp, nj);
        } else {
            int32_t turns = pg_clipper_round(steps_per_rad * fabs(atan2(sin_a, cos_a)));
            if (turns < 1) turns = 1;
            double v[2] = {nk[0], nk[1]};
            for (int32_t t = 0; t < turns; t++) {
                PG_AT(pp, v);
                const double v0 = v[0] * step_cos - step_sin * v[1];
                const double v1 = v[0] * step_sin + v[1] * step_cos;
                v[0] = v0;
                v[1] = v1;
            }
            PG_AT(pp, nj);
        }
        k = j;
    }
#undef PG_AT
#undef PG_OUT
    return (long)pg_cleanup(out, m);
}

/* --------------------------------------------------------- DB postprocess */

/* det.rs:399-402 distance: f32 norm of the difference. */
static float pg_distance(const float *p, const float *q) {
    const float dx = p[0] - q[0], dy = p[1] - q[1];
    return sqrtf(dx * dx + dy * dy);
}

/* det.rs:342-372 contour_candidate. Returns 0 Small, 1 LowScore,
 * 2 SmallAfterUnclip, 3 Kept (corners in page pixels); *score set from 1 on. */
int orc_contour_candidate(const float *prob, size_t mw, size_t mh, const int32_t *contour, size_t n, size_t dw,
                          size_t dh, double box_thresh, double unclip_ratio, double *score, int32_t corners[8]) {
    float quad[8];
    const float side = orc_mini_box(contour, n, quad);
    if (side < 3.0f) return 0;
    *score = orc_contour_mean(prob, mw, mh, contour, n);
    if (box_thresh > *score) return 1;
    int32_t ring[1024];
    long m = orc_unclip(quad, unclip_ratio, ring, 512);
    if (m < 0) return 2; /* not reached for quads of this size */
    float grown[8];
    const float side2 = orc_mini_box(ring, (size_t)m, grown);
    if (side2 < 3.0f + 2.0f) return 2;
    for (int i = 0; i < 4; i++) {
        const float fdw = (float)dw, fdh = (float)dh;
        float x = rintf(grown[2 * i] / (float)mw * fdw);
        float y = rintf(grown[2 * i + 1] / (float)mh * fdh);
        x = x < 0.0f ? 0.0f : x > fdw ? fdw : x;
        y = y < 0.0f ? 0.0f : y > fdh ? fdh : y;
        corners[2 * i] = (int32_t)x;
        corners[2 * i + 1] = (int32_t)y;
    }
    return 3;
}

/* det.rs:377-396 order_and_clip; 1 when the box is kept. */
int orc_order_and_clip(const int32_t corners[8], size_t width, size_t height, float quad[8]) {
    int32_t p[4][2];
    memcpy(p, corners, sizeof(p));
    for (int i = 1; i < 4; i++) /* stable sort by x */
        for (int j = i; j > 0 && p[j][0] < p[j - 1][0]; j--) {
            int32_t t0 = p[j][0], t1 = p[j][1];
            p[j][0] = p[j - 1][0]; p[j][1] = p[j - 1][1];
            p[j - 1][0] = t0; p[j - 1][1] = t1;
        }
    int32_t *a = p[0], *b = p[1], *c = p[2], *d = p[3];
    if (b[1] < a[1]) { int32_t *t = a; a = b; b = t; }
    if (d[1] < c[1]) { int32_t *t = c; c = d; d = t; }
    const int32_t *order[4] = {a, c, d, b};
    const int32_t mx = (int32_t)width - 1, my = (int32_t)height - 1;
    for (int i = 0; i < 4; i++) {
        int32_t x = order[i][0] > 0 ? order[i][0] : 0, y = order[i][1] > 0 ? order[i][1] : 0;
        x = x < mx ? x : mx;
        y = y < my ? y : my;
        quad[2 * i] = (float)x;
        quad[2 * i + 1] = (float)y;
    }
    return (int32_t)pg_distance(quad, quad + 2) > 3 && (int32_t)pg_distance(quad, quad + 6) > 3;
}

/* det.rs:407-421 sort_boxes: stable by top-left y, then lines (a jump of 10
 * or more starts one) left to right, stable. */
void orc_sort_boxes(float *quads, size_t n) {
    float *tmp = malloc((n ? n : 1) * 8 * sizeof(float));
    uint32_t *line = malloc((n ? n : 1) * sizeof(uint32_t));
    for (size_t i = 1; i < n; i++) /* stable insertion sort by quad[0][1] */
        for (size_t j = i; j > 0 && pg_total_lt(quads[8 * j + 1], quads[8 * (j - 1) + 1]); j--) {
            float t[8];
            memcpy(t, quads + 8 * j, sizeof(t));
            memcpy(quads + 8 * j, quads + 8 * (j - 1), sizeof(t));
            memcpy(quads + 8 * (j - 1), t, sizeof(t));
        }
    uint32_t l = 0;
    for (size_t i = 0; i < n; i++) {
        if (i > 0 && quads[8 * i + 1] - quads[8 * (i - 1) + 1] >= 10.0f) l++;
        line[i] = l;
    }
    memcpy(tmp, quads, n * 8 * sizeof(float));
    size_t *idx = malloc((n ? n : 1) * sizeof(size_t));
    for (size_t i = 0; i < n; i++) idx[i] = i;
    for (size_t i = 1; i < n; i++)
        for (size_t j = i; j > 0; j--) {
            const size_t a = idx[j], b = idx[j - 1];
            const int lt = line[a] < line[b] || (line[a] == line[b] && pg_total_lt(tmp[8 * a], tmp[8 * b]));
            if (!lt) break;
            idx[j] = b;
            idx[j - 1] = a;
        }
    for (size_t i = 0; i < n; i++) memcpy(quads + 8 * i, tmp + 8 * idx[i], 8 * sizeof(float));
    free(tmp);
    free(line);
    free(idx);
}

/* det.rs:430-452 boxes_from_prob: quads (8 floats each) in reading order.
 * Writes at most cap quads; returns the number of boxes (which may exceed cap). */
size_t orc_boxes_from_prob(const float *prob, size_t mw, size_t mh, size_t dw, size_t dh, float thresh,
                           double box_thresh, double unclip_ratio, size_t max_candidates, float *quads, size_t cap) {
    uint8_t *mask = malloc(mw * mh > 0 ? mw * mh : 1);
    for (size_t i = 0; i < mw * mh; i++) mask[i] = prob[i] > thresh;
    orc_contours *c = orc_find_contours(mask, mw, mh);
    free(mask);
    if (!c) return 0;
    const size_t take = c->n < max_candidates ? c->n : max_candidates;
    float *all = malloc((take ? take : 1) * 8 * sizeof(float));
    size_t kept = 0;
    for (size_t i = 0; i < take; i++) {
        size_t len;
        const int32_t *pts = orc_contour(c, i, &len);
        double score;
        int32_t corners[8];
        if (orc_contour_candidate(prob, mw, mh, pts, len, dw, dh, box_thresh, unclip_ratio, &score, corners) != 3)
            continue;
        if (orc_order_and_clip(corners, dw, dh, all + 8 * kept)) kept++;
    }
    orc_contours_free(c);
    orc_sort_boxes(all, kept);
    memcpy(quads, all, (kept < cap ? kept : cap) * 8 * sizeof(float));
    free(all);
    return kept;
}

/* ------------------------------------------------------------------ crop */

/* crop.rs:10-50 rectangle_to_quad: Gaussian elimination with partial
 * pivoting (of equal magnitudes the last row wins, as Rust's max_by). */
static void pg_rect_to_quad(double width, double height, const float *quad, double out[9]) {
    const double from[4][2] = {{0, 0}, {width, 0}, {width, height}, {0, height}};
    double m[8][9];
    for (int i = 0; i < 4; i++) {
        const double x = from[i][0], y = from[i][1], u = (double)quad[2 * i], v = (double)quad[2 * i + 1];
        const double r0[9] = {x, y, 1, 0, 0, 0, -x * u, -y * u, u};
        const double r1[9] = {0, 0, 0, x, y, 1, -x * v, -y * v, v};
        memcpy(m[i], r0, sizeof(r0));
        memcpy(m[i + 4], r1, sizeof(r1));
    }
    for (int col = 0; col < 8; col++) {
        int pivot = col;
        for (int r = col + 1; r < 8; r++)
            if (!(fabs(m[r][col]) < fabs(m[pivot][col]))) pivot = r; /* >=: the last of equals */
        if (pivot != col) {
            double t[9];
            memcpy(t, m[col], sizeof(t));
            memcpy(m[col], m[pivot], sizeof(t));
            memcpy(m[pivot], t, sizeof(t));
        }
        const double p = m[col][col];
        if (p == 0.0) continue;
        double prow[9];
        memcpy(prow, m[col], sizeof(prow));
        for (int r = 0; r < 8; r++) {
            const double f = m[r][col] / p;
            if (r != col && f != 0.0)
                for (int k = col; k < 9; k++) m[r][k] -= f * prow[k];
        }
    }
    for (int i = 0; i < 8; i++) out[i] = m[i][i] == 0.0 ? 0.0 : m[i][8] / m[i][i];
    out[8] = 1.0;
}

/* crop.rs:56-62 cubic_weights, OpenCV's factoring of Keys' a = -0.75. */
static void pg_cubic(float t, float w[4]) {
    const float A = -0.75f;
    const float t1 = t + 1.0f, s = 1.0f - t;
    w[0] = ((A * t1 - 5.0f * A) * t1 + 8.0f * A) * t1 - 4.0f * A;
    w[1] = ((A + 2.0f) * t - (A + 3.0f)) * t * t + 1.0f;
    w[2] = ((A + 2.0f) * s - (A + 3.0f)) * s * s + 1.0f;
    w[3] = 1.0f - w[0] - w[1] - w[2];
}

/* The crop's size before its possible quarter turn (crop.rs:85-86), and
 * whether it turns (crop.rs:122). */
void orc_crop_size(const float quad[8], size_t *width, size_t *height, int *turns) {
    const float a = pg_distance(quad, quad + 2), b = pg_distance(quad + 4, quad + 6);
    const float c = pg_distance(quad, quad + 6), d = pg_distance(quad + 2, quad + 4);
    *width = (size_t)(a > b ? a : b);
    *height = (size_t)(c > d ? c : d);
    *turns = (double)*height / (double)*width >= 1.5;
}

/* crop.rs:84-127 crop_text: out receives the crop, turned when tall
 * (out_w x out_h RGB bytes, out_w = height and out_h = width then). */
int orc_crop_text(const uint8_t *image, size_t iw, size_t ih, const float quad[8], uint8_t *out) {
    size_t width, height;
    int turns;
    orc_crop_size(quad, &width, &height, &turns);
    if (!iw || !ih) return 1;
    double m[9];
    pg_rect_to_quad((double)width, (double)height, quad, m);
    const long last_x = (long)iw - 1, last_y = (long)ih - 1;
    const size_t stride = iw * 3;
    uint8_t *crop = turns ? malloc(width * height * 3 + 1) : out;
    for (size_t y = 0; y < height; y++)
        for (size_t x = 0; x < width; x++) {
            const double xf = (double)x, yf = (double)y;
            double w = m[6] * xf + m[7] * yf + m[8];
            w = w == 0.0 ? 0.0 : 1.0 / w;
            const float sx = (float)((m[0] * xf + m[1] * yf + m[2]) * w);
            const float sy = (float)((m[3] * xf + m[4] * yf + m[5]) * w);
            const float fx = floorf(sx), fy = floorf(sy);
            float wx[4], wy[4];
            pg_cubic(sx - fx, wx);
            pg_cubic(sy - fy, wy);
            const long ix = (long)fx - 1, iy = (long)fy - 1;
            size_t cols[4];
            for (int i = 0; i < 4; i++) {
                long v = ix + i;
                v = v < 0 ? 0 : v > last_x ? last_x : v;
                cols[i] = (size_t)v * 3;
            }
            float acc[3] = {0, 0, 0};
            for (int j = 0; j < 4; j++) {
                long rv = iy + j;
                rv = rv < 0 ? 0 : rv > last_y ? last_y : rv;
                const uint8_t *row = image + (size_t)rv * stride;
                float line[3] = {0, 0, 0};
                for (int i = 0; i < 4; i++) {
                    const uint8_t *px = row + cols[i];
                    line[0] += (float)px[0] * wx[i];
                    line[1] += (float)px[1] * wx[i];
                    line[2] += (float)px[2] * wx[i];
                }
                for (int c = 0; c < 3; c++) acc[c] += line[c] * wy[j];
            }
            for (int c = 0; c < 3; c++) {
                float v = rintf(acc[c]);
                v = v < 0.0f ? 0.0f : v > 255.0f ? 255.0f : v;
                crop[(y * width + x) * 3 + c] = (uint8_t)v;
            }
        }
    if (turns) {
        orc_rotate_ccw(crop, width, height, out);
        free(crop);
    }
    return 0;
}

/* ------------------------------------------------------------ CTC decode */

/* rec.rs:112-134 pairwise_sum: numpy's float64 add.reduce. */
static double pg_pairwise(const double *v, size_t n) {
    if (n < 8) {
        double s = 0.0;
        for (size_t i = 0; i < n; i++) s += v[i];
        return s;
    }
    if (n <= 128) {
        double r[8];
        memcpy(r, v, sizeof(r));
        const size_t full = n - n % 8;
        for (size_t i = 8; i < full; i += 8)
            for (int k = 0; k < 8; k++) r[k] += v[i + k];
        double s = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
        for (size_t i = full; i < n; i++) s += v[i];
        return s;
    }
    const size_t half = n / 2 - (n / 2) % 8;
    return pg_pairwise(v, half) + pg_pairwise(v + half, n - half);
}

/* rec.rs:144-161 ctc_decode, classes only: kept[] receives the classes of
 * the text (repeats collapsed, blanks dropped); returns the score. */
double orc_ctc_decode(const uint32_t *best, const float *prob, size_t n, uint32_t *kept, size_t *kept_n) {
    double *probs = malloc((n ? n : 1) * sizeof(double));
    size_t k = 0;
    for (size_t t = 0; t < n; t++) {
        if (best[t] == 0 || (t > 0 && best[t] == best[t - 1])) continue;
        kept[k] = best[t];
        probs[k++] = nearbyint((double)prob[t] * 1e5) / 1e5;
    }
    *kept_n = k;
    double score = 0.0;
    if (k) score = nearbyint(pg_pairwise(probs, k) / (double)k * 1e5) / 1e5;
    free(probs);
    return score;
}

/* lib.rs:121-129 to_page: a quad on the prepared page mapped back, in f32. */
void orc_to_page(const float quad[8], double ratio_w, double ratio_h, size_t pad_top, size_t width, size_t height,
                 float out[8]) {
    const float rw = (float)ratio_w, rh = (float)ratio_h, mx = (float)width, my = (float)height;
    for (int i = 0; i < 4; i++) {
        float x = quad[2 * i] * rw, y = (quad[2 * i + 1] - (float)pad_top) * rh;
        x = fmaxf(x, 0.0f);
        x = fminf(x, mx);
        y = fmaxf(y, 0.0f);
        y = fminf(y, my);
        out[2 * i] = x;
        out[2 * i + 1] = y;
    }
}
