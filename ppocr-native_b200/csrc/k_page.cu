// Page steps on the GPU, between and around the two networks:
//
// - box scores: the DB postprocess's mean probability inside each contour
//   (reference src/contour.rs:142-199 contour_mean), one CTA per contour;
// - crops: the perspective crop of every text box of a page
//   (src/crop.rs:84-127 crop_text), one launch per page;
// - recogniser inputs: every crop resized to height 48 and normalized into
//   its recogniser lane (src/rec.rs:19-43), one launch per page;
// - the page fit: the page resized and padded as prepare_page does it
//   (src/det.rs:44-131).
//
// The crops and inputs are the reference's bytes and bits: every float and
// double operation is a correctly rounded IEEE operation in the reference's
// order (no contraction). The box score's sum runs in parallel, so it can
// differ from the reference's row-order f64 sum in the last bits; the score
// only decides `box_thresh > score`, and the host recomputes in the
// reference's order every contour whose score lies within a bound on that
// difference of the threshold (reader.cpp), so the kept boxes are the same.
#include <cuda_runtime.h>

#include <cstdint>

#include "image.cuh"
#include "page_kernels.hpp"

namespace ppocr {

namespace {

constexpr int SCORE_WARPS = 8;

__device__ __forceinline__ void mark_run(uint32_t *bm, int l, int r, int width) {
    if (r < 0 || l >= width) return;
    l = l < 0 ? 0 : l;
    r = r >= width ? width - 1 : r;
    for (int w = l >> 5; w <= (r >> 5); w++) {
        const int lo = w == (l >> 5) ? (l & 31) : 0, hi = w == (r >> 5) ? (r & 31) : 31;
        const uint32_t m = (hi == 31 ? 0xffffffffu : ((1u << (hi + 1)) - 1u)) & ~((1u << lo) - 1u);
        atomicOr(bm + w, m);
    }
}

// One CTA per work item (a contour's rows y0..y1, at most SCORE_ROWS), a
// warp per row (rows y0 + warp, + 8, ...). A row's
// pixels inside or on the contour go into a bitmap in shared memory: the
// edge pixels on the row (contour.rs:159-166) and the spans between sorted
// pairs of edge crossings (:167-182); the warp then sums the map over the
// set bits, 32 consecutive pixels at a time.
__global__ void __launch_bounds__(SCORE_WARPS * 32) box_score_kernel(const ScoreArgs a) {
    extern __shared__ uint32_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x;
    const ScoreWork wk = a.work[c];
    const ScoreBox box = a.boxes[wk.box];
    const int width = box.x1 - box.x0 + 1;
    const int words = (width + 31) >> 5;
    uint32_t *bm = smem + warp * (a.words + 2 * SCORE_CROSSINGS + 1);
    int *cross = reinterpret_cast<int *>(bm + a.words);
    int *sorted = cross + SCORE_CROSSINGS;
    int *ncross = sorted + SCORE_CROSSINGS;
    const int2 *pts = a.pts + box.first;
    const int n = box.count;
    double sum = 0.0, asum = 0.0;
    unsigned count = 0;
    int overflow = 0;
    for (int y = wk.y0 + warp; y <= wk.y1; y += SCORE_WARPS) {
        for (int w = lane; w < words; w += 32) bm[w] = 0;
        if (lane == 0) *ncross = 0;
        __syncwarp();
        for (int e = lane; e < n; e += 32) {
            const int2 p = pts[e], q = pts[e + 1 == n ? 0 : e + 1];
            const int dx = q.x - p.x, dy = q.y - p.y;
            const int m = max(abs(dx), abs(dy));
            const int sx = (dx > 0) - (dx < 0), sy = (dy > 0) - (dy < 0);
            if (sy == 0) {
                if (p.y == y) mark_run(bm, min(p.x, p.x + sx * m) - box.x0, max(p.x, p.x + sx * m) - box.x0, width);
            } else {
                const int i = (y - p.y) * sy;
                if (i >= 0 && i <= m) mark_run(bm, p.x + sx * i - box.x0, p.x + sx * i - box.x0, width);
            }
            const int2 lo = p.y < q.y ? p : q, hi = p.y < q.y ? q : p;
            if (lo.y <= y && y < hi.y) {
                const int k = atomicAdd(ncross, 1);
                if (k < SCORE_CROSSINGS) cross[k] = lo.x + (y - lo.y) * (hi.x - lo.x) / (hi.y - lo.y);
            }
        }
        __syncwarp();
        const int k = *ncross;
        if (k > SCORE_CROSSINGS) {
            overflow = 1;
            __syncwarp();
            continue;
        }
        for (int i = lane; i < k; i += 32) {  // rank sort, ties by position
            const int v = cross[i];
            int r = 0;
            for (int j = 0; j < k; j++) r += cross[j] < v || (cross[j] == v && j < i);
            sorted[r] = v;
        }
        __syncwarp();
        for (int j = lane; 2 * j + 1 < k; j += 32)
            mark_run(bm, sorted[2 * j] - box.x0, sorted[2 * j + 1] - box.x0, width);
        __syncwarp();
        const float *row = a.prob + long(y) * a.map_w + box.x0;
        for (int w = 0; w < words; w++) {
            const uint32_t bits = bm[w];
            const int x = w * 32 + lane;
            if ((bits >> lane) & 1u) {
                const double v = double(__ldg(row + x));
                sum += v;
                asum += fabs(v);
                count++;
            }
        }
        __syncwarp();
    }
    // Fixed-order reductions: lanes by shuffles, then warps in order.
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        sum += __shfl_xor_sync(0xffffffffu, sum, o);
        asum += __shfl_xor_sync(0xffffffffu, asum, o);
        count += __shfl_xor_sync(0xffffffffu, count, o);
    }
    overflow = __any_sync(0xffffffffu, overflow);
    __shared__ double ws[SCORE_WARPS], wa[SCORE_WARPS];
    __shared__ unsigned wc[SCORE_WARPS];
    __shared__ int wo[SCORE_WARPS];
    if (lane == 0) {
        ws[warp] = sum;
        wa[warp] = asum;
        wc[warp] = count;
        wo[warp] = overflow;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0, t = 0.0;
        unsigned long long n_in = 0;
        int of = 0;
        for (int w = 0; w < SCORE_WARPS; w++) {
            s += ws[w];
            t += wa[w];
            n_in += wc[w];
            of |= wo[w];
        }
        a.out[c] = ScoreOut{s, t, n_in, of};
    }
}

// Keys' cubic weights, OpenCV's factoring (crop.rs:56-62), in f32.
__device__ __forceinline__ void cubic(float t, float w[4]) {
    const float A = -0.75f;
    const float t1 = __fadd_rn(t, 1.0f), s = __fsub_rn(1.0f, t);
    w[0] = __fsub_rn(__fmul_rn(__fadd_rn(__fmul_rn(__fsub_rn(__fmul_rn(A, t1), __fmul_rn(5.0f, A)), t1),
                                         __fmul_rn(8.0f, A)), t1), __fmul_rn(4.0f, A));
    w[1] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(__fmul_rn(__fadd_rn(A, 2.0f), t), __fadd_rn(A, 3.0f)), t), t), 1.0f);
    w[2] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(__fmul_rn(__fadd_rn(A, 2.0f), s), __fadd_rn(A, 3.0f)), s), s), 1.0f);
    w[3] = __fsub_rn(__fsub_rn(__fsub_rn(1.0f, w[0]), w[1]), w[2]);
}

__device__ __forceinline__ int find_line(const long *first, int n, long i) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (first[mid] <= i) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// A thread per crop pixel of every line: its source point through the
// line's projective map in f64, Keys' bicubic taps with the edge repeated,
// each row of four taps summed, then the rows (OpenCV's order), rounded to
// a byte. A tall crop is written turned a quarter counter-clockwise.
__global__ void __launch_bounds__(256) crop_kernel(const CropArgs a) {
    for (long i = long(blockIdx.x) * blockDim.x + threadIdx.x; i < a.total; i += long(gridDim.x) * blockDim.x) {
        const int l = a.line ? find_line(a.first, a.lines, i) : 0;
        const CropLine &L = a.line ? a.line[l] : a.single;
        const long r = a.line ? i - a.first[l] : i;
        const int y = int(r / L.width), x = int(r - long(y) * L.width);
        const double xf = double(x), yf = double(y);
        double w = __dadd_rn(__dadd_rn(__dmul_rn(L.m[6], xf), __dmul_rn(L.m[7], yf)), L.m[8]);
        w = w == 0.0 ? 0.0 : __ddiv_rn(1.0, w);
        const float sx = __double2float_rn(__dmul_rn(__dadd_rn(__dadd_rn(__dmul_rn(L.m[0], xf), __dmul_rn(L.m[1], yf)),
                                                               L.m[2]), w));
        const float sy = __double2float_rn(__dmul_rn(__dadd_rn(__dadd_rn(__dmul_rn(L.m[3], xf), __dmul_rn(L.m[4], yf)),
                                                               L.m[5]), w));
        const float fx = floorf(sx), fy = floorf(sy);
        float wx[4], wy[4];
        cubic(__fsub_rn(sx, fx), wx);
        cubic(__fsub_rn(sy, fy), wy);
        const long ix = long(fx) - 1, iy = long(fy) - 1;
        const long last_x = a.iw - 1, last_y = a.ih - 1;
        int cols[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const long v = ix + k;
            cols[k] = int(v < 0 ? 0 : v > last_x ? last_x : v) * 3;
        }
        float acc[3] = {0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            long rv = iy + j;
            rv = rv < 0 ? 0 : rv > last_y ? last_y : rv;
            const uint8_t *row = a.image + rv * long(a.iw) * 3;
            float line[3] = {0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint8_t *px = row + cols[k];
#pragma unroll
                for (int ch = 0; ch < 3; ch++) line[ch] = __fadd_rn(line[ch], __fmul_rn(float(px[ch]), wx[k]));
            }
#pragma unroll
            for (int ch = 0; ch < 3; ch++) acc[ch] = __fadd_rn(acc[ch], __fmul_rn(line[ch], wy[j]));
        }
        // turned (np.rot90): pixel (x, y) of a width x height crop lands at
        // column y, row width - 1 - x of the height x width result
        const long at = L.turns ? (long(L.width - 1 - x) * L.height + y) : r;
        uint8_t *o = a.out + L.out + at * 3;
#pragma unroll
        for (int ch = 0; ch < 3; ch++) {
            float v = rintf(acc[ch]);
            v = v < 0.0f ? 0.0f : v > 255.0f ? 255.0f : v;
            o[ch] = uint8_t(v);
        }
    }
}

// A thread per recogniser input pixel of every line: the crop resized to
// rw x 48 (INTER_LINEAR in the reference's staging), (v / 255 - 0.5) / 0.5
// in f32, zeros from rw to the tensor width.
__global__ void __launch_bounds__(256) rec_lines_kernel(const RecLinesArgs a) {
    // each value is a function of its byte alone: the 256 of them once per block
    __shared__ float norm[256];
    for (int e = threadIdx.x; e < 256; e += blockDim.x)
        norm[e] = __fdiv_rn(__fsub_rn(__fdiv_rn(float(e), 255.0f), 0.5f), 0.5f);
    __syncthreads();
    for (long i = long(blockIdx.x) * blockDim.x + threadIdx.x; i < a.total; i += long(gridDim.x) * blockDim.x) {
        const int l = find_line(a.first, a.lines, i);
        const RecLine &L = a.line[l];
        const long r = i - a.first[l];
        const int oy = int(r / L.width), ox = int(r - long(oy) * L.width);
        float *o = L.out + r * 3;
        if (ox >= L.rw) {
            o[0] = o[1] = o[2] = 0.0f;
            continue;
        }
        const Tap ty = resize_tap_scaled(L.ch, L.sy, oy), tx = resize_tap_scaled(L.cw, L.sx, ox);
        const uint8_t *crop = a.crops + L.crop;
        const uint8_t *r0 = crop + long(ty.near) * L.cw * 3, *r1 = crop + long(ty.far) * L.cw * 3;
#pragma unroll
        for (int c = 0; c < 3; c++) o[c] = norm[blend(r0, r1, tx, ty, c)];
    }
}

// The page fitted to its detector page: resized to fw x fh when the size
// changes, `pad` rows of zeros above and below (det.rs:81-92).
__global__ void __launch_bounds__(256) fit_page_kernel(const FitArgs a) {
    const double sy = resize_scale(a.ih, a.fh), sx = resize_scale(a.iw, a.fw);
    const long total = long(a.fw) * (a.fh + 2 * a.pad);
    for (long i = long(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += long(gridDim.x) * blockDim.x) {
        const int oy = int(i / a.fw), ox = int(i - long(oy) * a.fw);
        uint8_t *o = a.out + i * 3;
        const int y = oy - a.pad;
        if (y < 0 || y >= a.fh) {
            o[0] = o[1] = o[2] = 0;
            continue;
        }
        if (a.fw == a.iw && a.fh == a.ih) {
            const uint8_t *s = a.image + (long(y) * a.iw + ox) * 3;
            o[0] = s[0]; o[1] = s[1]; o[2] = s[2];
            continue;
        }
        const Tap ty = resize_tap_scaled(a.ih, sy, y), tx = resize_tap_scaled(a.iw, sx, ox);
        const uint8_t *r0 = a.image + long(ty.near) * a.iw * 3, *r1 = a.image + long(ty.far) * a.iw * 3;
#pragma unroll
        for (int c = 0; c < 3; c++) o[c] = uint8_t(blend(r0, r1, tx, ty, c));
    }
}

unsigned grid_of(long total) {
    long blocks = (total + 255) / 256;
    if (blocks > 148L * 16) blocks = 148L * 16;
    return unsigned(blocks < 1 ? 1 : blocks);
}

}  // namespace

size_t score_smem(int words) { return size_t(SCORE_WARPS) * (size_t(words) + 2 * SCORE_CROSSINGS + 1) * 4; }

void configure_page_kernels() {
    cudaFuncSetAttribute(box_score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
}

void launch_box_scores(const ScoreArgs &a, int work_items, cudaStream_t s) {
    if (work_items > 0) box_score_kernel<<<unsigned(work_items), SCORE_WARPS * 32, score_smem(a.words), s>>>(a);
}

void launch_crops(const CropArgs &a, cudaStream_t s) {
    if (a.total > 0) crop_kernel<<<grid_of(a.total), 256, 0, s>>>(a);
}

void launch_rec_lines(const RecLinesArgs &a, cudaStream_t s) {
    if (a.total > 0) rec_lines_kernel<<<grid_of(a.total), 256, 0, s>>>(a);
}

void launch_fit_page(const FitArgs &a, cudaStream_t s) {
    fit_page_kernel<<<grid_of(long(a.fw) * (a.fh + 2 * a.pad)), 256, 0, s>>>(a);
}

}  // namespace ppocr
