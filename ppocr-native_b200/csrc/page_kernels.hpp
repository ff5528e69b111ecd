// Arguments of the page-step kernels (k_page.cu), shared with the reader.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace ppocr {

// At most this many edge crossings on one row of one contour go through the
// GPU box score; a contour with more is scored on the host.
constexpr int SCORE_CROSSINGS = 256;

// A contour's points (pts[first .. first + count)) and its clamped box.
struct ScoreBox {
    int x0, y0, x1, y1;
    int first, count;
};

struct ScoreOut {
    double sum, abs_sum;
    unsigned long long count;
    int overflow;
};

// One CTA's share of the box scores: rows [y0, y1] of contour `box`.
struct ScoreWork {
    int box, y0, y1;
};

// Rows of one contour a CTA scores: large contours are split over CTAs and
// their partial sums added on the host in order.
constexpr int SCORE_ROWS = 16;

struct ScoreArgs {
    const float *prob;
    int map_w;
    const int2 *pts;
    const ScoreBox *boxes;
    const ScoreWork *work;
    ScoreOut *out;  // per work item
    int words;      // bitmap words of the widest box
};

// One crop: the projective map from the upright width x height rectangle
// onto the quad (row-major, last entry 1), whether it turns, where its
// bytes go in the crop buffer.
struct CropLine {
    double m[9];
    int width, height, turns;
    long out;
};

struct CropArgs {
    const uint8_t *image;
    int iw, ih;
    const CropLine *line;  // null: the one line in `single`
    const long *first;     // per line: first pixel in the launch's pixel count
    int lines;
    long total;
    uint8_t *out;
    CropLine single;
};

// One recogniser lane: its crop (cw x ch bytes at `crop` in the crop
// buffer), resized width rw, tensor width, and the lane's input tensor.
struct RecLine {
    long crop;
    int cw, ch, rw, width;
    float *out;
    // the resize's f64 scales, 1 / (48 / ch) and 1 / (rw / cw), IEEE-rounded
    // on the host exactly as a device division rounds them
    double sy, sx;
};

struct RecLinesArgs {
    const uint8_t *crops;
    const RecLine *line;
    const long *first;
    int lines;
    long total;
};

struct FitArgs {
    const uint8_t *image;
    int iw, ih, fw, fh, pad;
    uint8_t *out;
};

size_t score_smem(int words);
void configure_page_kernels();
void launch_box_scores(const ScoreArgs &a, int work_items, cudaStream_t s);
void launch_crops(const CropArgs &a, cudaStream_t s);
void launch_rec_lines(const RecLinesArgs &a, cudaStream_t s);
void launch_fit_page(const FitArgs &a, cudaStream_t s);

}  // namespace ppocr
