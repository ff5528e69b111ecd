// Host page steps (page.hpp): border following, box geometry, page sizes,
// crop maps, CTC decoding. The reference restates OpenCV 5, pyclipper 1.4
// and numpy 2 and its fixtures pin their bits, so each function here keeps
// the reference's arithmetic: f32 where it computes in f32, f64 where it
// promotes, the same association of every sum and product (this file is
// compiled with -ffp-contract=off), glibc's sqrt / sin / cos / atan2 / acos
// as Rust's std calls them.
#include "page.hpp"

#include <emmintrin.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>

namespace ppocr {
namespace page {

namespace {

constexpr uint8_t BACKGROUND = 0, UNSEEN = 1, MARKED = 2, MARKED_EAST = 3;
// Neighbour steps counter-clockwise on screen (y down), from east.
constexpr int STEP_DX[8] = {1, 1, 0, -1, -1, -1, 0, 1};
constexpr int STEP_DY[8] = {0, -1, -1, -1, 0, 1, 1, 1};

int64_t cross(const Point &o, const Point &a, const Point &b) {
    const int64_t ux = int64_t(a.x) - o.x, uy = int64_t(a.y) - o.y;
    const int64_t vx = int64_t(b.x) - o.x, vy = int64_t(b.y) - o.y;
    return ux * vy - uy * vx;
}

// Rust's f32::total_cmp as a less-than: -0 before +0, NaNs at the ends.
bool total_less(float a, float b) {
    int32_t x, y;
    std::memcpy(&x, &a, 4);
    std::memcpy(&y, &b, 4);
    x ^= int32_t(uint32_t(x >> 31) >> 1);
    y ^= int32_t(uint32_t(y >> 31) >> 1);
    return x < y;
}

// Per byte of a word of scan states (0..3): 0x80 where the byte is nonzero
// (no byte reaches 0x81 when 0x7f is added, so nothing carries).
inline uint64_t nonzero_bytes(uint64_t w) { return (w + 0x7f7f7f7f7f7f7f7full) & 0x8080808080808080ull; }

// The next pixel at or after `from` in [from, end) of a frame row that can
// start a border: foreground with background to its west or east (the only
// starts of an outer or a hole border; background never changes during the
// scan). Eight pixels at a time; `row` has a background byte before `from`
// and after `end`.
size_t next_start(const uint8_t *row, size_t from, size_t end) {
    size_t i = from;
    // sixteen at a time (SSE2, every x86-64): a byte's nonzero bit from a
    // compare with zero, the same test as below
    const __m128i zero = _mm_setzero_si128();
    while (i + 16 <= end) {
        const __m128i w = _mm_loadu_si128(reinterpret_cast<const __m128i *>(row + i));
        const __m128i wl = _mm_loadu_si128(reinterpret_cast<const __m128i *>(row + i - 1));
        const __m128i wr = _mm_loadu_si128(reinterpret_cast<const __m128i *>(row + i + 1));
        const unsigned nz = ~unsigned(_mm_movemask_epi8(_mm_cmpeq_epi8(w, zero))) & 0xffffu;
        const unsigned nzl = ~unsigned(_mm_movemask_epi8(_mm_cmpeq_epi8(wl, zero))) & 0xffffu;
        const unsigned nzr = ~unsigned(_mm_movemask_epi8(_mm_cmpeq_epi8(wr, zero))) & 0xffffu;
        const unsigned cand = nz & ~(nzl & nzr);
        if (cand) return i + size_t(__builtin_ctz(cand));
        i += 16;
    }
    while (i + 9 <= end + 1) {
        uint64_t w, wl, wr;
        std::memcpy(&w, row + i, 8);
        std::memcpy(&wl, row + i - 1, 8);
        std::memcpy(&wr, row + i + 1, 8);
        const uint64_t cand = nonzero_bytes(w) & ~(nonzero_bytes(wl) & nonzero_bytes(wr));
        if (cand) return i + size_t(__builtin_ctzll(cand) >> 3);
        i += 8;
    }
    for (; i < end; i++)
        if (row[i] && (!row[i - 1] || !row[i + 1])) return i;
    return end;
}

}  // namespace

// contour.rs:44-130: Suzuki-Abe border following on a frame of background
// (cv2.findContours RETR_LIST + CHAIN_APPROX_SIMPLE), the borders found last
// listed first. A border starts at an unseen pixel with background to its
// west (an outer border) or at an unseen or marked pixel with background to
// its east (a hole border).
void find_contours(const uint8_t *mask, size_t width, size_t height, Contours &out, ContourScratch &s) {
    out.start.assign(1, 0);
    out.pts.clear();
    const size_t stride = width + 2;
    if (s.state.size() < stride * (height + 2)) s.state.resize(stride * (height + 2));
    uint8_t *state = s.state.data();
    // the frame of background, then each row (one pass over the buffer)
    std::memset(state, BACKGROUND, stride);
    std::memset(state + (height + 1) * stride, BACKGROUND, stride);
    for (size_t y = 0; y < height; y++) {
        uint8_t *dst = state + (y + 1) * stride;
        const uint8_t *src = mask + y * width;
        dst[0] = dst[width + 1] = BACKGROUND;
        for (size_t x = 0; x < width; x++) dst[x + 1] = src[x] ? UNSEEN : BACKGROUND;
    }
    long off[8];
    for (int d = 0; d < 8; d++) off[d] = STEP_DX[d] + STEP_DY[d] * long(stride);
    const auto point = [stride](size_t at) { return Point{int32_t(at % stride) - 1, int32_t(at / stride) - 1}; };
    // Contours are collected in scan order and reversed at the end.
    std::vector<std::pair<size_t, size_t>> found;  // (first point, count) in `corners`
    std::vector<Point> corners;
    for (size_t y = 1; y <= height; y++) {
        const uint8_t *row = state + y * stride;
        size_t x = next_start(row, 1, width + 1);
        while (x <= width) {
            const size_t start = y * stride + x;
            const uint8_t here = state[start];
            int from = -1;
            if (here == UNSEEN && state[start - 1] == BACKGROUND)
                from = 4;  // west
            else if ((here == UNSEEN || here == MARKED) && state[start + 1] == BACKGROUND)
                from = 0;  // east
            if (from >= 0) {
                int last_dir = -1;
                for (int k = 0; k < 8; k++) {
                    const int d = (from + 8 - k) & 7;
                    if (state[start + off[d]] != BACKGROUND) {
                        last_dir = d;
                        break;
                    }
                }
                if (last_dir < 0) {
                    state[start] = MARKED_EAST;
                    found.emplace_back(corners.size(), 1);
                    corners.push_back(point(start));
                } else {
                    const size_t last = start + off[last_dir];
                    // CHAIN_APPROX_SIMPLE on the fly: a point is kept where
                    // the step leaving it turns from the step before; the
                    // first point's turn (against the last step) is known at
                    // the end, and it then leads the list
                    const size_t at = corners.size();
                    size_t cur = start, first_at = start;
                    int back = last_dir, first_dir = -1, prev_dir = -1;
                    for (;;) {
                        bool east_bg = false;
                        int next_dir = back;
                        for (int k = 1; k <= 8; k++) {
                            const int d = (back + k) & 7;
                            if (state[cur + off[d]] != BACKGROUND) {
                                next_dir = d;
                                break;
                            }
                            if (d == 0) east_bg = true;
                        }
                        if (east_bg)
                            state[cur] = MARKED_EAST;
                        else if (state[cur] == UNSEEN)
                            state[cur] = MARKED;
                        if (first_dir < 0) {
                            first_dir = next_dir;
                            first_at = cur;
                        } else if (next_dir != prev_dir) {
                            corners.push_back(point(cur));
                        }
                        prev_dir = next_dir;
                        const size_t next = cur + off[next_dir];
                        if (next == start && cur == last) break;
                        back = (next_dir + 4) & 7;
                        cur = next;
                    }
                    if (first_dir != prev_dir) corners.insert(corners.begin() + long(at), point(first_at));
                    found.emplace_back(at, corners.size() - at);
                }
            }
            x = next_start(row, x + 1, width + 1);
        }
    }
    out.pts.reserve(corners.size());
    out.start.reserve(found.size() + 1);
    for (size_t i = found.size(); i-- > 0;) {
        out.pts.insert(out.pts.end(), corners.begin() + long(found[i].first),
                       corners.begin() + long(found[i].first + found[i].second));
        out.start.push_back(out.pts.size());
    }
}

Box contour_box(const Point *c, size_t n, size_t width, size_t height) {
    int mnx = 0, mxx = 0, mny = 0, mxy = 0;
    for (size_t i = 0; i < n; i++) {
        mnx = i ? std::min(mnx, c[i].x) : c[i].x;
        mxx = i ? std::max(mxx, c[i].x) : c[i].x;
        mny = i ? std::min(mny, c[i].y) : c[i].y;
        mxy = i ? std::max(mxy, c[i].y) : c[i].y;
    }
    const auto cl = [](int v, int hi) { return v < 0 ? 0 : v > hi ? hi : v; };
    return Box{cl(mnx, int(width) - 1), cl(mny, int(height) - 1), cl(mxx, int(width) - 1), cl(mxy, int(height) - 1)};
}

// contour.rs:142-199: the f64 mean of the map over the pixels on the
// contour's edges or inside it by the even-odd rule along each row, summed
// in row order.
double contour_mean(const float *map, size_t width, size_t height, const Point *c, size_t n) {
    const Box b = contour_box(c, n, width, height);
    const size_t w = size_t(b.x1 - b.x0 + 1), h = size_t(b.y1 - b.y0 + 1);
    std::vector<uint8_t> inside(w * h, 0);
    const auto mark = [&](int x, int y) {
        if (x >= b.x0 && x <= b.x1 && y >= b.y0 && y <= b.y1) inside[size_t(y - b.y0) * w + size_t(x - b.x0)] = 1;
    };
    for (size_t e = 0; e < n; e++) {
        const Point &a = c[e], &q = c[(e + 1) % n];
        const int dx = q.x - a.x, dy = q.y - a.y;
        const int m = std::max(std::abs(dx), std::abs(dy));
        const int sx = (dx > 0) - (dx < 0), sy = (dy > 0) - (dy < 0);
        for (int i = 0; i <= m; i++) mark(a.x + sx * i, a.y + sy * i);
    }
    std::vector<int> crossings;
    for (int y = b.y0; y <= b.y1; y++) {
        crossings.clear();
        for (size_t e = 0; e < n; e++) {
            const Point &a = c[e], &q = c[(e + 1) % n];
            const Point &lo = a.y < q.y ? a : q, &hi = a.y < q.y ? q : a;
            if (lo.y <= y && y < hi.y) crossings.push_back(lo.x + (y - lo.y) * (hi.x - lo.x) / (hi.y - lo.y));
        }
        std::sort(crossings.begin(), crossings.end());
        for (size_t j = 0; j + 1 < crossings.size(); j += 2)
            for (int x = crossings[j]; x <= crossings[j + 1]; x++) mark(x, y);
    }
    double sum = 0.0;
    size_t count = 0;
    for (size_t r = 0; r < h; r++) {
        const float *line = map + (size_t(b.y0) + r) * width + size_t(b.x0);
        for (size_t i = 0; i < w; i++)
            if (inside[r * w + i]) {
                sum += double(line[i]);
                count++;
            }
    }
    return count ? sum / double(count) : 0.0;
}

namespace {

// geometry.rs:263-320 hull_order: cv2.convexHull's indices in its order
// (Andrew's monotone chain, then OpenCV's rotation to one monotonic run).
std::vector<size_t> hull_order(const Point *pts, size_t n) {
    std::vector<size_t> order(n);
    for (size_t i = 0; i < n; i++) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [pts](size_t i, size_t j) {
        return pts[i].x != pts[j].x ? pts[i].x < pts[j].x : pts[i].y < pts[j].y;
    });
    order.erase(std::unique(order.begin(), order.end(), [pts](size_t i, size_t j) { return pts[i] == pts[j]; }),
                order.end());
    if (order.size() < 3) {
        std::reverse(order.begin(), order.end());
        return order;
    }
    const auto chain = [pts](auto first, auto last) {
        std::vector<size_t> h;
        for (auto it = first; it != last; ++it) {
            while (h.size() >= 2 && cross(pts[h[h.size() - 2]], pts[h.back()], pts[*it]) <= 0) h.pop_back();
            h.push_back(*it);
        }
        h.pop_back();
        return h;
    };
    const std::vector<size_t> lower = chain(order.begin(), order.end());
    std::vector<size_t> hull = chain(order.rbegin(), order.rend());
    hull.insert(hull.end(), lower.begin(), lower.end());
    const size_t m = hull.size();
    if (m < 3) return hull;
    size_t lowest = 0, highest = 0, ascents = 0;
    for (size_t i = 1; i < m; i++) {
        ascents += hull[i - 1] < hull[i];
        if (ascents > 1 && ascents + 1 < i) break;
        if (hull[i] < hull[lowest]) lowest = i;
        if (hull[i] > hull[highest]) highest = i;
    }
    const size_t gap = lowest > highest ? lowest - highest : highest - lowest;
    if ((gap == 1 || gap == m - 1) && (ascents <= 1 || ascents + 2 >= m)) {
        const bool ascending = (highest + 1) % m == lowest;
        const size_t first = ascending ? lowest : highest;
        std::vector<size_t> rotated(m);
        for (size_t k = 0; k < m; k++) rotated[k] = hull[(first + k) % m];
        bool mono = true;
        for (size_t k = 0; k + 1 < m; k++)
            if ((rotated[k] < rotated[k + 1]) != ascending) mono = false;
        if (first > 0 && mono) return rotated;
    }
    return hull;
}

// geometry.rs:324-394 calipers: OpenCV's rotating calipers, in f32.
void calipers(const std::vector<PointF> &p, PointF &corner, PointF &u, PointF &v) {
    const size_t n = p.size();
    std::vector<PointF> edge(n);
    std::vector<float> inv_len(n);
    size_t left = 0, bottom = 0, right = 0, top = 0;
    for (size_t i = 0; i < n; i++) {
        const PointF &q = p[i], &r = p[(i + 1) % n];
        if (q.x < p[left].x) left = i;
        if (q.x > p[right].x) right = i;
        if (q.y > p[top].y) top = i;
        if (q.y < p[bottom].y) bottom = i;
        const double dx = double(r.x - q.x), dy = double(r.y - q.y);
        edge[i] = PointF{float(dx), float(dy)};
        inv_len[i] = float(1.0 / std::sqrt(dx * dx + dy * dy));
    }
    size_t seq[4] = {bottom, right, top, left};
    float min_area = std::numeric_limits<float>::max();
    size_t best_l = 0, best_bt = 0;
    float best_a = 0, best_w = 0, best_b = 0, best_h = 0;
    for (size_t it = 0; it < n; it++) {
        // Each caliper's next edge turned into the bottom caliper's frame.
        const PointF e0 = edge[seq[0]], e1 = edge[seq[1]], e2 = edge[seq[2]], e3 = edge[seq[3]];
        const PointF t[4] = {e0, {e1.y, -e1.x}, {-e2.x, -e2.y}, {-e3.y, e3.x}};
        int main = 0;
        for (int i = 1; i < 4; i++) {
            const float lhs = t[i].y * t[main].x;
            const float rhs = -t[i].x * t[main].y;
            if (lhs + rhs < 0.0f) main = i;
        }
        const size_t k = seq[main];
        const float lx = edge[k].x * inv_len[k], ly = edge[k].y * inv_len[k];
        float a, b;
        switch (main) {
        case 0: a = lx; b = ly; break;
        case 1: a = ly; b = -lx; break;
        case 2: a = -lx; b = -ly; break;
        default: a = -ly; b = lx; break;
        }
        seq[main] = (seq[main] + 1) % n;
        const float wa = (p[seq[1]].x - p[seq[3]].x) * a, wb = (p[seq[1]].y - p[seq[3]].y) * b;
        const float width = wa + wb;
        const float ha = -(p[seq[2]].x - p[seq[0]].x) * b, hb = (p[seq[2]].y - p[seq[0]].y) * a;
        const float height = ha + hb;
        const float area = width * height;
        if (area <= min_area) {
            min_area = area;
            best_l = seq[3];
            best_a = a;
            best_w = width;
            best_b = b;
            best_h = height;
            best_bt = seq[0];
        }
    }
    const float a1 = best_a, b1 = best_b, a2 = -b1, b2 = a1;
    const float c1 = a1 * p[best_l].x + p[best_l].y * b1;
    const float c2 = a2 * p[best_bt].x + p[best_bt].y * b2;
    const float inv_det = 1.0f / (a1 * b2 - a2 * b1);
    corner = PointF{(c1 * b2 - c2 * b1) * inv_det, (a1 * c2 - a2 * c1) * inv_det};
    u = PointF{a1 * best_w, b1 * best_w};
    v = PointF{a2 * best_h, b2 * best_h};
}

}  // namespace

// geometry.rs:406-457: cv2.minAreaRect as OpenCV 5 computes it.
RotatedRect min_area_rect(const Point *pts, size_t n) {
    const std::vector<size_t> idx = hull_order(pts, n);
    std::vector<PointF> hull(idx.size());
    for (size_t i = 0; i < idx.size(); i++) hull[i] = PointF{float(pts[idx[i]].x), float(pts[idx[i]].y)};
    const auto length = [](double dx, double dy) { return float(std::sqrt(dx * dx + dy * dy)); };
    double angle = -M_PI / 2;
    RotatedRect r{0, 0, 0, 0, 0};
    if (hull.size() == 1) {
        r.cx = hull[0].x;
        r.cy = hull[0].y;
    } else if (hull.size() == 2) {
        const PointF p = hull[0], q = hull[1];
        r.cx = (p.x + q.x) * 0.5f;
        r.cy = (p.y + q.y) * 0.5f;
        const double dx = double(p.x - q.x), dy = double(p.y - q.y);
        const float size = length(dx, dy);
        if (dx == 0.0) {
            r.width = size;
        } else if (dy < 0.0) {
            angle = std::atan2(dy, dx);
            r.width = size;
        } else {
            if (dy > 0.0) angle = -std::atan2(dx, dy);
            r.height = size;
        }
    } else if (hull.size() >= 3) {
        PointF corner, u, v;
        calipers(hull, corner, u, v);
        r.cx = corner.x + (u.x + v.x) * 0.5f;
        r.cy = corner.y + (u.y + v.y) * 0.5f;
        const float ul = length(double(u.x), double(u.y)), vl = length(double(v.x), double(v.y));
        if (u.x == 0.0f && u.y > 0.0f) {
            r.width = ul;
            r.height = vl;
        } else {
            angle = -std::atan2(double(u.x), double(u.y));
            r.width = vl;
            r.height = ul;
        }
    }
    r.angle = float(angle * 180.0 / M_PI);
    return r;
}

// geometry.rs:228-240: cv2.boxPoints, f32 but for the sine and cosine.
Quad box_points(const RotatedRect &r) {
    const double rad = double(r.angle) * M_PI / 180.0;
    const float a = float(std::sin(rad)) * 0.5f, b = float(std::cos(rad)) * 0.5f;
    const float cx = r.cx, cy = r.cy, w = r.width, h = r.height;
    return Quad{PointF{cx - a * h - b * w, cy + b * h - a * w}, PointF{cx + a * h - b * w, cy - b * h - a * w},
                PointF{cx + a * h + b * w, cy - b * h + a * w}, PointF{cx - a * h + b * w, cy + b * h + a * w}};
}

// geometry.rs:462-477 (RapidOCR's get_mini_boxes).
float mini_box(const Point *pts, size_t n, Quad &quad) {
    const RotatedRect r = min_area_rect(pts, n);
    Quad p = box_points(r);
    std::stable_sort(p.begin(), p.end(), [](const PointF &a, const PointF &b) { return total_less(a.x, b.x); });
    const PointF tl = p[1].y > p[0].y ? p[0] : p[1], bl = p[1].y > p[0].y ? p[1] : p[0];
    const PointF tr = p[3].y > p[2].y ? p[2] : p[3], br = p[3].y > p[2].y ? p[3] : p[2];
    quad = Quad{tl, tr, br, bl};
    return std::min(r.width, r.height);
}

namespace {

int32_t clipper_round(double v) { return v < 0.0 ? int32_t(v - 0.5) : int32_t(v + 0.5); }

// geometry.rs:611-634: the ring as Clipper's union hands it back.
void clipper_cleanup(std::vector<Point> &ring) {
    while (ring.size() >= 3) {
        const size_t n = ring.size();
        size_t found = n;
        for (size_t i = 0; i < n; i++) {
            const Point &prev = ring[(i + n - 1) % n], &here = ring[i], &next = ring[(i + 1) % n];
            if (here == next || cross(prev, here, next) == 0) {
                found = i;
                break;
            }
        }
        if (found == n) break;
        ring.erase(ring.begin() + long(found));
    }
    const size_t n = ring.size();
    if (!n) return;
    int32_t top = ring[0].y;
    for (const Point &p : ring) top = std::min(top, p.y);
    size_t last = n - 1;
    for (size_t i = 0; i < n; i++)
        if (ring[i].y == top && ring[(i + 1) % n].y != top) {
            last = i;
            break;
        }
    std::rotate(ring.begin(), ring.begin() + long((last + 1) % n), ring.end());
}

}  // namespace

// geometry.rs:519-606: RapidOCR's unclip (pyclipper JT_ROUND,
// ET_CLOSEDPOLYGON, arc tolerance 0.25) on the truncated corners.
std::vector<Point> unclip(const Quad &quad, double ratio) {
    double p[4][2];
    for (int i = 0; i < 4; i++) {
        p[i][0] = double(quad[size_t(i)].x);
        p[i][1] = double(quad[size_t(i)].y);
    }
    double sum = 0.0;  // shapely's shoelace relative to the first x
    for (int i = 1; i < 4; i++) sum += (p[i][0] - p[0][0]) * (p[i - 1][1] - p[(i + 1) % 4][1]);
    double perimeter = 0.0;
    for (int i = 0; i < 4; i++) {
        const double dx = p[(i + 1) % 4][0] - p[i][0], dy = p[(i + 1) % 4][1] - p[i][1];
        perimeter += std::sqrt(dx * dx + dy * dy);
    }
    const double delta = std::fabs(sum / 2.0) * ratio / perimeter;
    std::vector<std::array<double, 2>> ring;
    for (const PointF &q : quad) {
        const std::array<double, 2> t{double(std::trunc(q.x)), double(std::trunc(q.y))};
        if (ring.empty() || ring.back() != t) ring.push_back(t);
    }
    while (ring.size() > 1 && ring.front() == ring.back()) ring.pop_back();
    std::vector<Point> out;
    if (ring.size() < 3) return out;
    if (std::fabs(delta) < 1e-20) {
        for (const auto &q : ring) out.push_back(Point{int32_t(q[0]), int32_t(q[1])});
        clipper_cleanup(out);
        return out;
    }
    const size_t n = ring.size();
    double signed_area = 0.0;
    for (size_t i = 0; i < n; i++)
        signed_area += ring[i][0] * ring[(i + 1) % n][1] - ring[(i + 1) % n][0] * ring[i][1];
    if (signed_area < 0.0) std::reverse(ring.begin(), ring.end());
    const double ad = std::fabs(delta);
    const double tolerance = std::min(0.25, ad * 0.25);
    const double steps = std::fmin(M_PI / std::acos(1.0 - tolerance / ad), ad * M_PI);
    const double step_sin = std::sin(2 * M_PI / steps), step_cos = std::cos(2 * M_PI / steps);
    const double steps_per_rad = steps / (2 * M_PI);
    std::vector<std::array<double, 2>> normals(n);
    for (size_t i = 0; i < n; i++) {
        const double dx = ring[(i + 1) % n][0] - ring[i][0], dy = ring[(i + 1) % n][1] - ring[i][1];
        const double inv = 1.0 / std::sqrt(dx * dx + dy * dy);
        normals[i] = {dy * inv, -dx * inv};
    }
    const auto at = [delta](const std::array<double, 2> &q, const std::array<double, 2> &nv) {
        return Point{clipper_round(q[0] + nv[0] * delta), clipper_round(q[1] + nv[1] * delta)};
    };
    size_t k = n - 1;
    for (size_t j = 0; j < n; j++) {
        const auto &q = ring[j], &nk = normals[k], &nj = normals[j];
        double sin_a = nk[0] * nj[1] - nj[0] * nk[1];
        const double cos_a = nk[0] * nj[0] + nk[1] * nj[1];
        if (std::fabs(sin_a * delta) < 1.0) {
            if (cos_a > 0.0) {  // nearly straight: one point, k stays
                out.push_back(at(q, nk));
                continue;
            }
        } else {
            sin_a = std::clamp(sin_a, -1.0, 1.0);
        }
        if (sin_a * delta < 0.0) {
            out.push_back(at(q, nk));
            out.push_back(Point{int32_t(q[0]), int32_t(q[1])});
            out.push_back(at(q, nj));
        } else {
            const int32_t turns = std::max<int32_t>(clipper_round(steps_per_rad * std::fabs(std::atan2(sin_a, cos_a))), 1);
            std::array<double, 2> v = nk;
            for (int32_t t = 0; t < turns; t++) {
                out.push_back(at(q, v));
                v = {v[0] * step_cos - step_sin * v[1], v[0] * step_sin + v[1] * step_cos};
            }
            out.push_back(at(q, nj));
        }
        k = j;
    }
    clipper_cleanup(out);
    return out;
}

float distance(const PointF &p, const PointF &q) {
    const float dx = p.x - q.x, dy = p.y - q.y;
    return std::sqrt(dx * dx + dy * dy);
}

// det.rs:358-371: the box grown by the unclip distance, thinner than 5
// pixels refused, scaled from the map to the page in f32.
bool grow_box(const Quad &quad, size_t mw, size_t mh, size_t dw, size_t dh, double unclip_ratio, Point corners[4]) {
    const std::vector<Point> ring = unclip(quad, unclip_ratio);
    Quad grown;
    const float side = mini_box(ring.data(), ring.size(), grown);
    if (side < 3.0f + 2.0f) return false;
    const float fdw = float(dw), fdh = float(dh);
    for (size_t i = 0; i < 4; i++) {
        const float x = std::clamp(std::nearbyint(grown[i].x / float(mw) * fdw), 0.0f, fdw);
        const float y = std::clamp(std::nearbyint(grown[i].y / float(mh) * fdh), 0.0f, fdh);
        corners[i] = Point{int32_t(x), int32_t(y)};
    }
    return true;
}

// det.rs:377-396 (RapidOCR's filter_det_res for one box).
bool order_and_clip(const Point corners[4], size_t width, size_t height, Quad &out) {
    std::array<Point, 4> p{corners[0], corners[1], corners[2], corners[3]};
    std::stable_sort(p.begin(), p.end(), [](const Point &a, const Point &b) { return a.x < b.x; });
    Point a = p[0], b = p[1], c = p[2], d = p[3];
    if (b.y < a.y) std::swap(a, b);
    if (d.y < c.y) std::swap(c, d);
    const auto clip = [width, height](const Point &q) {
        return PointF{float(std::min(std::max(q.x, 0), int32_t(width) - 1)),
                      float(std::min(std::max(q.y, 0), int32_t(height) - 1))};
    };
    out = Quad{clip(a), clip(c), clip(d), clip(b)};
    return int32_t(distance(out[0], out[1])) > 3 && int32_t(distance(out[0], out[3])) > 3;
}

// det.rs:407-421: RapidOCR's reading order.
void sort_boxes(std::vector<Quad> &boxes) {
    std::stable_sort(boxes.begin(), boxes.end(), [](const Quad &a, const Quad &b) { return total_less(a[0].y, b[0].y); });
    std::vector<uint32_t> line(boxes.size(), 0);
    uint32_t l = 0;
    for (size_t i = 0; i < boxes.size(); i++) {
        if (i > 0 && boxes[i][0].y - boxes[i - 1][0].y >= 10.0f) l++;
        line[i] = l;
    }
    std::vector<size_t> idx(boxes.size());
    for (size_t i = 0; i < idx.size(); i++) idx[i] = i;
    std::stable_sort(idx.begin(), idx.end(), [&](size_t i, size_t j) {
        return line[i] != line[j] ? line[i] < line[j] : total_less(boxes[i][0].x, boxes[j][0].x);
    });
    std::vector<Quad> sorted(boxes.size());
    for (size_t i = 0; i < idx.size(); i++) sorted[i] = boxes[idx[i]];
    boxes.swap(sorted);
}

std::vector<Quad> boxes_from_prob(const float *prob, size_t mw, size_t mh, size_t dw, size_t dh,
                                  const DbOptions &o) {
    std::vector<uint8_t> mask(mw * mh);
    for (size_t i = 0; i < mask.size(); i++) mask[i] = prob[i] > o.thresh;
    Contours cs;
    ContourScratch scratch;
    find_contours(mask.data(), mw, mh, cs, scratch);
    std::vector<Quad> boxes;
    for (size_t i = 0; i < cs.size() && i < o.max_candidates; i++) {
        Quad quad;
        if (mini_box(cs.at(i), cs.len(i), quad) < 3.0f) continue;
        if (o.box_thresh > contour_mean(prob, mw, mh, cs.at(i), cs.len(i))) continue;
        Point corners[4];
        Quad q;
        if (grow_box(quad, mw, mh, dw, dh, o.unclip_ratio, corners) && order_and_clip(corners, dw, dh, q))
            boxes.push_back(q);
    }
    sort_boxes(boxes);
    return boxes;
}

namespace {

size_t snap32(size_t x) { return size_t(std::nearbyint(double(x) / 32.0)) * 32; }

bool scaled_size(size_t w, size_t h, double ratio, size_t &ow, size_t &oh) {
    if (!w || !h) return false;
    ow = snap32(size_t(double(w) * ratio));
    oh = snap32(size_t(double(h) * ratio));
    return ow > 0 && oh > 0;
}

// Rust's float-to-usize `as`: NaN and negatives give 0, large values saturate.
size_t to_usize(double v) { return v > 0.0 ? (v >= 1.8e19 ? SIZE_MAX : size_t(v)) : 0; }

size_t band_height(size_t w, size_t h, double whr, size_t min_height) {
    const bool too_wide = whr != -1.0 && double(w) / double(h) > whr;
    if (h > min_height && !too_wide) return 0;
    size_t target = std::max(to_usize(double(w) / whr), min_height);
    target = target > SIZE_MAX / 2 ? SIZE_MAX : target * 2;
    return (target > h ? target - h : h - target) / 2;
}

}  // namespace

// det.rs:44-131: fit within max_side, then up to min_side, then the bands.
bool prepare_page(size_t w, size_t h, size_t min_side, size_t max_side, double whr, size_t min_height,
                  Prepared &out) {
    size_t cw = w, ch = h;
    bool resized = false;
    if (std::max(w, h) > max_side) {
        if (!scaled_size(w, h, double(max_side) / double(std::max(w, h)), cw, ch)) return false;
        resized = true;
    }
    double rh = 1.0, rw = 1.0;
    if (std::min(cw, ch) < min_side) {
        size_t uw, uh;
        if (!scaled_size(cw, ch, double(min_side) / double(std::min(cw, ch)), uw, uh)) return false;
        rh = double(ch) / double(uh);
        rw = double(cw) / double(uw);
        cw = uw;
        ch = uh;
    } else if (resized) {
        rh = double(h) / double(ch);
        rw = double(w) / double(cw);
    }
    const size_t pad = band_height(cw, ch, whr, min_height);
    const size_t padded = pad > (SIZE_MAX - ch) / 2 ? SIZE_MAX : 2 * pad + ch;
    const size_t area = max_side && max_side > SIZE_MAX / max_side ? SIZE_MAX : max_side * max_side;
    if (padded && cw > area / padded) return false;
    out = Prepared{cw, ch + 2 * pad, cw, ch, rh, rw, pad};
    return true;
}

bool det_size(size_t w, size_t h, size_t limit_min, size_t &ow, size_t &oh) {
    double ratio = 1.0;
    if (!limit_min) {
        const size_t lng = std::max(w, h);
        const size_t side = lng < 960 ? 960 : lng < 1500 ? 1500 : 2000;
        if (lng > side) ratio = double(side) / double(lng);
    } else {
        const size_t shrt = std::min(w, h);
        if (shrt < limit_min) ratio = double(limit_min) / double(shrt);
    }
    return scaled_size(w, h, ratio, ow, oh);
}

// crop.rs:10-50: the projective map of the upright rectangle onto the quad,
// eight equations solved by Gaussian elimination with partial pivoting (of
// equal magnitudes the last row is the pivot, as Rust's max_by picks).
CropPlan plan_crop(const Quad &quad) {
    CropPlan c;
    c.width = size_t(std::max(distance(quad[0], quad[1]), distance(quad[2], quad[3])));
    c.height = size_t(std::max(distance(quad[0], quad[3]), distance(quad[1], quad[2])));
    c.turns = double(c.height) / double(c.width) >= 1.5;
    const double W = double(c.width), H = double(c.height);
    const double from[4][2] = {{0, 0}, {W, 0}, {W, H}, {0, H}};
    double m[8][9];
    for (int i = 0; i < 4; i++) {
        const double x = from[i][0], y = from[i][1];
        const double u = double(quad[size_t(i)].x), v = double(quad[size_t(i)].y);
        const double r0[9] = {x, y, 1, 0, 0, 0, -x * u, -y * u, u};
        const double r1[9] = {0, 0, 0, x, y, 1, -x * v, -y * v, v};
        std::memcpy(m[i], r0, sizeof(r0));
        std::memcpy(m[i + 4], r1, sizeof(r1));
    }
    for (int col = 0; col < 8; col++) {
        int pivot = col;
        for (int r = col + 1; r < 8; r++)
            if (!(std::fabs(m[r][col]) < std::fabs(m[pivot][col]))) pivot = r;
        if (pivot != col) std::swap(m[col], m[pivot]);
        const double pv = m[col][col];
        if (pv == 0.0) continue;
        double prow[9];
        std::memcpy(prow, m[col], sizeof(prow));
        for (int r = 0; r < 8; r++) {
            const double f = m[r][col] / pv;
            if (r != col && f != 0.0)
                for (int k = col; k < 9; k++) m[r][k] -= f * prow[k];
        }
    }
    for (int i = 0; i < 8; i++) c.m[i] = m[i][i] == 0.0 ? 0.0 : m[i][8] / m[i][i];
    c.m[8] = 1.0;
    return c;
}

// rec.rs:19-31: the tensor width truncates, the resized width rounds up and
// is cut back to the tensor.
void rec_widths(size_t cw, size_t ch, size_t &width, size_t &resized) {
    const double h = double(ch), w = double(cw), rows = 48.0;
    const double ratio = std::max(320.0 / rows, w / h);
    width = size_t(rows * ratio);
    const double fitted = std::ceil(rows * (w / h));
    resized = fitted > double(width) ? width : size_t(fitted);
}

namespace {

// One code point of UTF-8 text at `i`, advancing i.
uint32_t next_code_point(const std::string &s, size_t &i) {
    const auto b = [&](size_t k) { return uint32_t(uint8_t(s[k])); };
    const uint32_t c = b(i);
    if (c < 0x80 || i + 1 >= s.size()) {
        i += 1;
        return c;
    }
    if ((c >> 5) == 6) {
        i += 2;
        return ((c & 0x1f) << 6) | (b(i - 1) & 0x3f);
    }
    if ((c >> 4) == 14 && i + 2 < s.size()) {
        i += 3;
        return ((c & 0x0f) << 12) | ((b(i - 2) & 0x3f) << 6) | (b(i - 1) & 0x3f);
    }
    if (i + 3 < s.size()) {
        i += 4;
        return ((c & 0x07) << 18) | ((b(i - 3) & 0x3f) << 12) | ((b(i - 2) & 0x3f) << 6) | (b(i - 1) & 0x3f);
    }
    i += 1;
    return c;
}

// The line breaks Python's str.splitlines knows (rec.rs:84-97), as UTF-8:
// the length of the break at text[i], 0 if none.
size_t line_break_at(const char *t, size_t len, size_t i) {
    const auto u = [&](size_t k) { return uint8_t(t[k]); };
    const uint8_t c = u(i);
    if (c == '\r') return i + 1 < len && t[i + 1] == '\n' ? 2 : 1;
    if (c == '\n' || c == 0x0b || c == 0x0c || c == 0x1c || c == 0x1d || c == 0x1e) return 1;
    if (c == 0xc2 && i + 1 < len && u(i + 1) == 0x85) return 2;                                   // U+0085
    if (c == 0xe2 && i + 2 < len && u(i + 1) == 0x80 && (u(i + 2) == 0xa8 || u(i + 2) == 0xa9)) return 3;  // U+2028/9
    return 0;
}

}  // namespace

// rec.rs:54-79: blank, the metadata's lines, a space.
Dictionary Dictionary::from_metadata(const char *text, size_t len) {
    Dictionary d;
    d.classes.emplace_back("blank");
    size_t begin = 0, i = 0;
    while (i < len) {
        const size_t br = line_break_at(text, len, i);
        if (br) {
            d.classes.emplace_back(text + begin, i - begin);
            i += br;
            begin = i;
        } else {
            i++;
        }
    }
    if (begin < len) d.classes.emplace_back(text + begin, len - begin);
    d.classes.emplace_back(" ");
    return d;
}

namespace {

// rec.rs:112-134: numpy's float64 add.reduce.
double pairwise_sum(const double *v, size_t n) {
    if (n < 8) {
        double s = 0.0;
        for (size_t i = 0; i < n; i++) s += v[i];
        return s;
    }
    if (n <= 128) {
        double r[8];
        std::memcpy(r, v, sizeof(r));
        const size_t full = n - n % 8;
        for (size_t i = 8; i < full; i += 8)
            for (int k = 0; k < 8; k++) r[k] += v[i + size_t(k)];
        double s = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
        for (size_t i = full; i < n; i++) s += v[i];
        return s;
    }
    const size_t half = n / 2 - (n / 2) % 8;
    return pairwise_sum(v, half) + pairwise_sum(v + half, n - half);
}

}  // namespace

// rec.rs:144-161 and ocr.rs:551-560: the recogniser's [steps][2] output
// (best class as a float, its probability) through the greedy decode. A
// class outside the dictionary makes the score NaN and adds no text (the
// reference panics there: the model and the dictionary do not belong
// together).
double ctc_decode(const float *output, size_t steps, const Dictionary &d, std::string &text) {
    text.clear();
    std::vector<double> kept;
    uint32_t prev = 0;
    bool bad = false;
    for (size_t t = 0; t < steps; t++) {
        const uint32_t cls = uint32_t(output[2 * t]);
        const float p = output[2 * t + 1];
        const bool repeat = t > 0 && cls == prev;
        prev = cls;
        if (cls == 0 || repeat) continue;
        if (cls >= d.classes.size()) {
            bad = true;
            continue;
        }
        text += d.classes[cls];
        kept.push_back(std::nearbyint(double(p) * 1e5) / 1e5);
    }
    if (bad) return std::numeric_limits<double>::quiet_NaN();
    if (kept.empty()) return 0.0;
    const double mean = pairwise_sum(kept.data(), kept.size()) / double(kept.size());
    return std::nearbyint(mean * 1e5) / 1e5;
}

// rec.rs:168-172: only Unicode white space and the separators 0x1c-0x1f.
bool is_blank(const std::string &text) {
    size_t i = 0;
    while (i < text.size()) {
        const uint32_t c = next_code_point(text, i);
        const bool space = (c >= 0x09 && c <= 0x0d) || c == 0x20 || c == 0x85 || c == 0xa0 || c == 0x1680 ||
                           (c >= 0x2000 && c <= 0x200a) || c == 0x2028 || c == 0x2029 || c == 0x202f ||
                           c == 0x205f || c == 0x3000 || (c >= 0x1c && c <= 0x1f);
        if (!space) return false;
    }
    return true;
}

Quad to_page(const Quad &q, double ratio_w, double ratio_h, size_t pad_top, size_t width, size_t height) {
    const float rw = float(ratio_w), rh = float(ratio_h), mx = float(width), my = float(height);
    Quad out;
    for (size_t i = 0; i < 4; i++) {
        out[i].x = std::fmin(std::fmax(q[i].x * rw, 0.0f), mx);
        out[i].y = std::fmin(std::fmax((q[i].y - float(pad_top)) * rh, 0.0f), my);
    }
    return out;
}

}  // namespace page
}  // namespace ppocr
