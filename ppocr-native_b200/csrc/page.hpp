// Host page steps around the two networks: what ppocr-native's library does
// between the detector and the recogniser (src/det.rs, contour.rs,
// geometry.rs, crop.rs, rec.rs, lib.rs), in C++ for the reader of this
// library. Every float operation follows the reference's order and
// precision: the reference matches OpenCV, pyclipper and numpy bit for bit,
// and so must the boxes and texts that come out of here.
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace ppocr {
namespace page {

struct Point {
    int32_t x, y;
    bool operator==(const Point &o) const { return x == o.x && y == o.y; }
};
struct PointF {
    float x, y;
};
using Quad = std::array<PointF, 4>;  // top-left, top-right, bottom-right, bottom-left

// Borders of a binary mask (contour.rs:44-130): contour i is
// pts[start[i] .. start[i + 1]).
struct Contours {
    std::vector<size_t> start{0};
    std::vector<Point> pts;
    size_t size() const { return start.size() - 1; }
    const Point *at(size_t i) const { return pts.data() + start[i]; }
    size_t len(size_t i) const { return start[i + 1] - start[i]; }
};

// Scan state reused between calls (the image inside a frame of background).
struct ContourScratch {
    std::vector<uint8_t> state;
};

void find_contours(const uint8_t *mask, size_t width, size_t height, Contours &out, ContourScratch &scratch);

// The mask's clamped bounding box of a contour, as contour_mean uses it.
struct Box {
    int x0, y0, x1, y1;
};
Box contour_box(const Point *c, size_t n, size_t width, size_t height);
double contour_mean(const float *map, size_t width, size_t height, const Point *c, size_t n);

struct RotatedRect {
    float cx, cy, width, height, angle;
};
RotatedRect min_area_rect(const Point *pts, size_t n);
Quad box_points(const RotatedRect &r);
float mini_box(const Point *pts, size_t n, Quad &quad);
std::vector<Point> unclip(const Quad &quad, double ratio);

struct DbOptions {
    float thresh = 0.3f;
    double box_thresh = 0.5;
    double unclip_ratio = 1.5;
    size_t max_candidates = 1000;
};

// contour_candidate past its score (det.rs:358-371): the grown box in page
// pixels, or false when it is thinner than 5 pixels once grown.
bool grow_box(const Quad &quad, size_t mw, size_t mh, size_t dw, size_t dh, double unclip_ratio, Point corners[4]);
bool order_and_clip(const Point corners[4], size_t width, size_t height, Quad &out);
void sort_boxes(std::vector<Quad> &boxes);
// The whole postprocess on the host (det.rs:430-452).
std::vector<Quad> boxes_from_prob(const float *prob, size_t mw, size_t mh, size_t dw, size_t dh,
                                  const DbOptions &o);

// Page preparation sizes (det.rs:44-131) and the detector size (:166-193).
struct Prepared {
    size_t width, height;  // after fitting and padding
    size_t fit_width, fit_height;
    double ratio_h, ratio_w;
    size_t pad_top;
};
bool prepare_page(size_t w, size_t h, size_t min_side, size_t max_side, double whr, size_t min_height,
                  Prepared &out);
bool det_size(size_t w, size_t h, size_t limit_min, size_t &ow, size_t &oh);

// The crop of a quad (crop.rs:84-127): its size before the turn, whether it
// turns, and the projective map from the upright rectangle onto the quad.
struct CropPlan {
    size_t width, height;
    bool turns;
    double m[9];
};
CropPlan plan_crop(const Quad &quad);
float distance(const PointF &p, const PointF &q);
// The recogniser tensor width of a crop and its resized width (rec.rs:19-31).
void rec_widths(size_t cw, size_t ch, size_t &width, size_t &resized);

// The recogniser's classes (rec.rs:54-79) and the greedy decode (:144-161).
struct Dictionary {
    std::vector<std::string> classes;
    static Dictionary from_metadata(const char *text, size_t len);
};
double ctc_decode(const float *output, size_t steps, const Dictionary &d, std::string &text);
bool is_blank(const std::string &text);

// page_lines' mapping of a quad back to the original page (lib.rs:121-129).
Quad to_page(const Quad &q, double ratio_w, double ratio_h, size_t pad_top, size_t width, size_t height);

}  // namespace page
}  // namespace ppocr
