// The page reader: a page's bytes in, its text lines out, the way
// ppocr-native's worker reads a page on the GPU (src/bin/ppocr-native/
// ocr.rs:205-263 Reader::detect / read, :338-509 recognise_all /
// recognise_on_gpu, :513-530 read_on_gpu), with the page steps on the GPU
// where they are data-parallel and on the calling thread where they are
// sequential:
//
//   page bytes -> [fit / pad] -> detector input -> detector -> text mask
//     (GPU)                                                  | mask to host
//   border following, minimum-area boxes (host) -> box scores (GPU)
//   -> unclip, order, reading order (host)
//   -> crops -> recogniser inputs -> recogniser (GPU) -> CTC decode (host)
//   -> page lines (host)
//
// Every step gives the reference's bytes and bits (page.hpp, k_page.cu). A
// reader holds its own detector and recogniser models (sharing the weights
// of the models it was made from) on one stream, so several readers on
// several host threads keep one GPU busy, as the reference keeps its crop
// threads and GPU lanes busy. Calls on one reader are not thread-safe.
//
// Also here: the C ABI of the host page steps themselves (the reference's
// public find_contours, min_area_rect, unclip, boxes_from_prob, det_size,
// prepare_page, ctc_decode, Dictionary, and crop_text on the GPU).
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "../../include/ppocr_cuda.h"
#include "page.hpp"
#include "page_kernels.hpp"

namespace ppocr {
void set_last_error(const std::string &msg);
}

using namespace ppocr;
using page::Point;
using page::PointF;
using page::Quad;

namespace {

int fail(int code, const std::string &msg) {
    set_last_error(msg);
    return code;
}

bool cuda_ok(cudaError_t e, const char *what, int *code = nullptr) {
    if (e == cudaSuccess) return true;
    set_last_error(std::string(what) + ": " + cudaGetErrorString(e));
    if (code) *code = e == cudaErrorMemoryAllocation ? PPOCR_E_NOMEM : PPOCR_E_DEVICE;
    return false;
}

// Grow-only device and page-locked host buffers: a page of the same size as
// the last one allocates nothing.
struct Dev {
    void *p = nullptr;
    size_t bytes = 0;
    ~Dev() {
        if (p) cudaFree(p);
    }
    bool fit(size_t n, int &code) {
        if (n <= bytes && p) return true;
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
        const size_t grown = std::max<size_t>(n + n / 4, 256);
        if (!cuda_ok(cudaMalloc(&p, grown), "allocating reader memory", &code)) return false;
        bytes = grown;
        return true;
    }
    template <class T>
    T *as() const {
        return static_cast<T *>(p);
    }
};

struct Host {
    void *p = nullptr;
    size_t bytes = 0;
    ~Host() {
        if (p) cudaFreeHost(p);
    }
    bool fit(size_t n, int &code) {
        if (n <= bytes && p) return true;
        if (p) cudaFreeHost(p);
        p = nullptr;
        bytes = 0;
        const size_t grown = std::max<size_t>(n + n / 4, 256);
        if (!cuda_ok(cudaHostAlloc(&p, grown, cudaHostAllocDefault), "allocating page-locked reader memory", &code))
            return false;
        bytes = grown;
        return true;
    }
    template <class T>
    T *as() const {
        return static_cast<T *>(p);
    }
};

size_t align16(size_t n) { return (n + 15) & ~size_t(15); }

constexpr double U = 1.1102230246251565e-16;  // 2^-53, the f64 unit roundoff

}  // namespace

struct ppocr_reader {
    int device = 0;
    ppocr_model *det = nullptr, *rec = nullptr;
    cudaStream_t stream = nullptr;
    cudaEvent_t ev = nullptr;
    page::Dictionary dict;
    ppocr_reader_options opt{};

    Dev page_raw, page_fit, mask, pts, boxes, scores, desc, crops;
    Host page_host, mask_host, pts_host, boxes_host, scores_host, desc_host, rec_host, prob_host;

    // the page of the last detect
    bool have_page = false;
    size_t page_w = 0, page_h = 0;
    page::Prepared prep{};
    const uint8_t *prepared = nullptr;  // device: the detector's page (fitted and padded)
    size_t det_w = 0, det_h = 0;
    std::vector<Quad> found;
    std::vector<std::pair<std::string, double>> reads;
    struct Line {
        Quad quad;
        std::string text;
        double score;
    };
    std::vector<Line> lines;
    std::vector<std::pair<size_t, size_t>> rec_sizes;  // the recogniser's current lanes
    page::Contours contours;
    page::ContourScratch scratch;
    size_t rescored = 0, scored = 0;
    size_t launches = 0;  // kernels of the last detection and the recognitions after it

    ~ppocr_reader() {
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        if (rec) ppocr_model_free(rec);
        if (det) ppocr_model_free(det);
        if (ev) cudaEventDestroy(ev);
    }

    // Host time by step (nanoseconds, summed over calls): waiting for the
    // GPU, border following, box geometry, recogniser set-up, decoding.
    enum { T_WAIT, T_CONTOURS, T_BOXES, T_PREP, T_DECODE, T_COUNT };
    uint64_t t_ns[T_COUNT] = {0, 0, 0, 0, 0};
    struct Clock {
        uint64_t &acc;
        std::chrono::steady_clock::time_point t0 = std::chrono::steady_clock::now();
        explicit Clock(uint64_t &a) : acc(a) {}
        ~Clock() {
            acc += uint64_t(
                std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count());
        }
    };

    // Wait for everything queued on the stream, at most timeout_ms (0: no
    // limit). A few quick polls catch short waits; then the thread sleeps
    // between polls, so readers waiting on the GPU leave the host cores to
    // the readers doing page steps.
    int sync(uint32_t timeout_ms) {
        Clock c(t_ns[T_WAIT]);
        if (!cuda_ok(cudaEventRecord(ev, stream), "recording a reader event")) return PPOCR_E_DEVICE;
        const auto start = std::chrono::steady_clock::now();
        for (unsigned poll = 0;; poll++) {
            const cudaError_t e = cudaEventQuery(ev);
            if (e == cudaSuccess) return PPOCR_OK;
            if (e != cudaErrorNotReady) return cuda_ok(e, "reading a page") ? PPOCR_OK : PPOCR_E_DEVICE;
            if (timeout_ms && std::chrono::steady_clock::now() - start > std::chrono::milliseconds(timeout_ms))
                return fail(PPOCR_E_TIMEOUT, "the GPU did not finish the page within " + std::to_string(timeout_ms) +
                                                 " ms");
            if (poll >= 8) std::this_thread::sleep_for(std::chrono::microseconds(poll < 64 ? 20 : 100));
        }
    }

    int detect(const uint8_t *page, size_t w, size_t h, uint32_t timeout_ms, bool on_device = false);
    int recognise(const Quad *quads, size_t n, uint32_t timeout_ms);
    int score_boxes(const std::vector<std::pair<size_t, Quad>> &cand, uint32_t timeout_ms);
};

// ocr.rs:205-231 Reader::detect: the page prepared (det.rs:110-131), the
// detector at det_size (the page limit squared bounds Limit::Min, else
// Limit::Max), the DB postprocess (det.rs:430-452) on its map.
int ppocr_reader::detect(const uint8_t *page, size_t w, size_t h, uint32_t timeout_ms, bool on_device) {
    found.clear();
    reads.clear();
    lines.clear();
    have_page = false;
    if (!cuda_ok(cudaSetDevice(device), "selecting the device")) return PPOCR_E_DEVICE;
    page::Prepared p;
    if (!page::prepare_page(w, h, opt.min_side, opt.max_side, opt.width_height_ratio, opt.min_height, p))
        return PPOCR_OK;  // no page: no text (RapidOCR raises there)
    const size_t limit = size_t(opt.max_side) * opt.max_side;
    size_t dw = 0, dh = 0;
    bool sized = page::det_size(p.width, p.height, opt.limit_min, dw, dh) && dw * dh <= limit;
    if (!sized) sized = page::det_size(p.width, p.height, 0, dw, dh);
    if (!sized) return PPOCR_OK;
    int code = PPOCR_OK;
    launches = 0;
    // the page on the device (a device page is read where it lies and must
    // stay unchanged until the next detection or recognition returns)
    const size_t raw = w * h * 3;
    const uint8_t *src = page;
    if (!on_device) {
        if (!page_raw.fit(raw, code)) return code;
        if (!cuda_ok(cudaMemcpyAsync(page_raw.p, page, raw, cudaMemcpyHostToDevice, stream), "copying the page in"))
            return PPOCR_E_DEVICE;
        src = page_raw.as<uint8_t>();
    }
    if (p.fit_width != w || p.fit_height != h || p.pad_top) {
        if (!page_fit.fit(p.width * p.height * 3, code)) return code;
        FitArgs fa{src, int(w), int(h), int(p.fit_width), int(p.fit_height), int(p.pad_top), page_fit.as<uint8_t>()};
        launch_fit_page(fa, stream);
        launches++;
        src = page_fit.as<uint8_t>();
    }
    // the detector
    if (dw != det_w || dh != det_h) {
        int rc = ppocr_model_set_input_size(det, uint32_t(dh), uint32_t(dw));
        if (rc) return rc;
        det_w = dw;
        det_h = dh;
    }
    size_t in_len = 0, out_len = 0;
    float *din = ppocr_model_lane_device_input(det, 0, &in_len);
    if (!din) return PPOCR_E_ARG;
    int rc = ppocr_det_input_hwc(src, p.width, p.height, dw, dh, opt.mean, opt.std, din, in_len, stream);
    if (rc) return rc;
    if ((rc = ppocr_model_enqueue_device(det))) return rc;
    launches += 2 + ppocr_model_launches(det);  // input, network, and the mask below
    const float *prob = ppocr_model_lane_device_output(det, 0, 0, &out_len);
    if (!prob || out_len != dw * dh) return fail(PPOCR_E_UNSUPPORTED, "the detector's first output is not a map");
    if (!mask.fit(out_len, code) || !mask_host.fit(out_len, code)) return code;
    if ((rc = ppocr_db_mask(prob, out_len, opt.thresh, mask.as<uint8_t>(), stream))) return rc;
    if (!cuda_ok(cudaMemcpyAsync(mask_host.p, mask.p, out_len, cudaMemcpyDeviceToHost, stream), "copying the mask"))
        return PPOCR_E_DEVICE;
    if ((rc = sync(timeout_ms))) return rc;
    if ((rc = ppocr_model_wait(det, timeout_ms))) return rc;  // the detector's own error word
    prep = p;
    prepared = src;
    page_w = w;
    page_h = h;
    have_page = true;
    // border following and the first rejections on the host
    {
        Clock c(t_ns[T_CONTOURS]);
        page::find_contours(mask_host.as<uint8_t>(), dw, dh, contours, scratch);
    }
    std::vector<std::pair<size_t, Quad>> cand;
    {
        Clock c(t_ns[T_BOXES]);
        for (size_t i = 0; i < contours.size() && i < opt.max_candidates; i++) {
            Quad q;
            if (page::mini_box(contours.at(i), contours.len(i), q) >= 3.0f) cand.emplace_back(i, q);
        }
    }
    if (!cand.empty() && (rc = score_boxes(cand, timeout_ms))) return rc;
    page::sort_boxes(found);
    return PPOCR_OK;
}

// The candidates' mean probabilities on the GPU; the host recomputes in the
// reference's order any whose mean is within the parallel sum's error bound
// of box_thresh (or whose rows have more crossings than the kernel holds),
// then grows, scales and clips the kept boxes (det.rs:355-371, :377-396).
int ppocr_reader::score_boxes(const std::vector<std::pair<size_t, Quad>> &cand, uint32_t timeout_ms) {
    int code = PPOCR_OK;
    size_t npts = 0, items = 0;
    for (const auto &c : cand) npts += contours.len(c.first);
    if (npts > size_t(INT32_MAX) / 2) return fail(PPOCR_E_SIZE, "too many contour points");
    std::vector<page::Box> bx(cand.size());
    for (size_t k = 0; k < cand.size(); k++) {
        bx[k] = page::contour_box(contours.at(cand[k].first), contours.len(cand[k].first), det_w, det_h);
        items += size_t((bx[k].y1 - bx[k].y0) / SCORE_ROWS + 1);
    }
    const size_t bytes_boxes = align16(cand.size() * sizeof(ScoreBox)), bytes_work = align16(items * sizeof(ScoreWork));
    if (!pts_host.fit(npts * sizeof(int2), code) || !pts.fit(npts * sizeof(int2), code) ||
        !boxes_host.fit(bytes_boxes + bytes_work, code) || !boxes.fit(bytes_boxes + bytes_work, code) ||
        !scores_host.fit(items * sizeof(ScoreOut), code) || !scores.fit(items * sizeof(ScoreOut), code))
        return code;
    int2 *hp = pts_host.as<int2>();
    ScoreBox *hb = boxes_host.as<ScoreBox>();
    ScoreWork *hw = reinterpret_cast<ScoreWork *>(boxes_host.as<char>() + bytes_boxes);
    std::vector<size_t> first_item(cand.size() + 1, 0);
    size_t at = 0, item = 0;
    int words = 1;
    for (size_t k = 0; k < cand.size(); k++) {
        const size_t i = cand[k].first, n = contours.len(i);
        const Point *c = contours.at(i);
        for (size_t j = 0; j < n; j++) hp[at + j] = make_int2(c[j].x, c[j].y);
        const page::Box &b = bx[k];
        hb[k] = ScoreBox{b.x0, b.y0, b.x1, b.y1, int(at), int(n)};
        words = std::max(words, (b.x1 - b.x0 + 1 + 31) / 32);
        at += n;
        first_item[k] = item;
        for (int y = b.y0; y <= b.y1; y += SCORE_ROWS)
            hw[item++] = ScoreWork{int(k), y, std::min(b.y1, y + SCORE_ROWS - 1)};
    }
    first_item[cand.size()] = item;
    if (score_smem(words) > 200 * 1024) return fail(PPOCR_E_SIZE, "a contour wider than the box-score kernel takes");
    if (!cuda_ok(cudaMemcpyAsync(pts.p, pts_host.p, npts * sizeof(int2), cudaMemcpyHostToDevice, stream),
                 "copying contours in") ||
        !cuda_ok(cudaMemcpyAsync(boxes.p, boxes_host.p, bytes_boxes + bytes_work, cudaMemcpyHostToDevice, stream),
                 "copying contour boxes in"))
        return PPOCR_E_DEVICE;
    size_t out_len = 0;
    const float *prob = ppocr_model_lane_device_output(det, 0, 0, &out_len);
    ScoreArgs a{prob, int(det_w), pts.as<int2>(), boxes.as<ScoreBox>(),
                reinterpret_cast<const ScoreWork *>(boxes.as<char>() + bytes_boxes), scores.as<ScoreOut>(), words};
    launch_box_scores(a, int(items), stream);
    launches++;
    if (!cuda_ok(cudaGetLastError(), "launching the box scores")) return PPOCR_E_DEVICE;
    if (!cuda_ok(cudaMemcpyAsync(scores_host.p, scores.p, items * sizeof(ScoreOut), cudaMemcpyDeviceToHost,
                                 stream), "copying box scores out"))
        return PPOCR_E_DEVICE;
    int rc = sync(timeout_ms);
    if (rc) return rc;
    bool prob_here = false;
    const ScoreOut *so = scores_host.as<ScoreOut>();
    Clock clk(t_ns[T_BOXES]);
    for (size_t k = 0; k < cand.size(); k++) {
        ScoreOut o{0.0, 0.0, 0, 0};
        for (size_t j = first_item[k]; j < first_item[k + 1]; j++) {  // the slices in row order
            o.sum += so[j].sum;
            o.abs_sum += so[j].abs_sum;
            o.count += so[j].count;
            o.overflow |= so[j].overflow;
        }
        double mean = o.count ? o.sum / double(o.count) : 0.0;
        const double margin = 4.0 * U * o.abs_sum + 4.0 * U * std::fabs(mean);
        scored++;
        if (o.overflow || std::fabs(mean - opt.box_thresh) <= margin) {
            if (!prob_here) {  // the map, once, for the reference-order sums
                if (!prob_host.fit(out_len * sizeof(float), code)) return code;
                if (!cuda_ok(cudaMemcpyAsync(prob_host.p, prob, out_len * sizeof(float), cudaMemcpyDeviceToHost,
                                             stream), "copying the map out"))
                    return PPOCR_E_DEVICE;
                if ((rc = sync(timeout_ms))) return rc;
                prob_here = true;
            }
            const size_t i = cand[k].first;
            mean = page::contour_mean(prob_host.as<float>(), det_w, det_h, contours.at(i), contours.len(i));
            rescored++;
        }
        if (opt.box_thresh > mean) continue;
        Point corners[4];
        Quad q;
        if (page::grow_box(cand[k].second, det_w, det_h, prep.width, prep.height, opt.unclip_ratio, corners) &&
            page::order_and_clip(corners, prep.width, prep.height, q))
            found.push_back(q);
    }
    return PPOCR_OK;
}

// ocr.rs:436-530 recognise_on_gpu + read_on_gpu: every quad cropped from the
// detector's page (crop.rs:84-127), turned into its recogniser input
// (rec.rs:19-43, ocr.rs:534-549), read in runs of up to max_lanes lanes,
// decoded (rec.rs:144-161). An empty crop reads as no text. A lane's result
// does not depend on the run it is in, so runs larger than the reference's
// 16 give the same reads.
int ppocr_reader::recognise(const Quad *quads, size_t n, uint32_t timeout_ms) {
    reads.assign(n, {std::string(), 0.0});
    if (!have_page) return fail(PPOCR_E_ARG, "no page: detect one first");
    if (!cuda_ok(cudaSetDevice(device), "selecting the device")) return PPOCR_E_DEVICE;
    struct Lane {
        size_t quad;
        page::CropPlan plan;
        size_t cw, ch, width, rw, crop;
    };
    std::vector<Lane> all;
    auto prep_start = std::chrono::steady_clock::now();
    const auto prep_stop = [&] {
        t_ns[T_PREP] += uint64_t(std::chrono::duration_cast<std::chrono::nanoseconds>(
                                     std::chrono::steady_clock::now() - prep_start).count());
    };
    for (size_t i = 0; i < n; i++) {
        Lane L;
        L.quad = i;
        L.plan = page::plan_crop(quads[i]);
        if (!L.plan.width || !L.plan.height) continue;
        L.cw = L.plan.turns ? L.plan.height : L.plan.width;
        L.ch = L.plan.turns ? L.plan.width : L.plan.height;
        page::rec_widths(L.cw, L.ch, L.width, L.rw);
        all.push_back(L);
    }
    const size_t per_run = ppocr_model_max_lanes(rec);
    int code = PPOCR_OK;
    for (size_t r0 = 0; r0 < all.size(); r0 += per_run) {
        if (r0) prep_start = std::chrono::steady_clock::now();
        const size_t r1 = std::min(all.size(), r0 + per_run), k = r1 - r0;
        std::vector<std::pair<size_t, size_t>> sizes;
        std::vector<uint32_t> hw;
        size_t crop_bytes = 0;
        for (size_t j = r0; j < r1; j++) {
            sizes.emplace_back(48, all[j].width);
            hw.push_back(48);
            hw.push_back(uint32_t(all[j].width));
            all[j].crop = crop_bytes;
            crop_bytes += align16(all[j].cw * all[j].ch * 3);
        }
        if (sizes != rec_sizes) {
            int rc = ppocr_model_set_sizes(rec, hw.data(), k);
            if (rc) return rc;
            rec_sizes = sizes;
        }
        // descriptors: crop lines, their first pixels, recogniser lines, theirs
        const size_t off_cf = align16(k * sizeof(CropLine)), off_rl = off_cf + align16(k * sizeof(long)),
                     off_rf = off_rl + align16(k * sizeof(RecLine)), total = off_rf + align16(k * sizeof(long));
        if (!desc_host.fit(total, code) || !desc.fit(total, code) || !crops.fit(crop_bytes, code)) return code;
        char *hd = desc_host.as<char>();
        CropLine *cl = reinterpret_cast<CropLine *>(hd);
        long *cf = reinterpret_cast<long *>(hd + off_cf);
        RecLine *rl = reinterpret_cast<RecLine *>(hd + off_rl);
        long *rf = reinterpret_cast<long *>(hd + off_rf);
        long crop_px = 0, rec_px = 0;
        for (size_t j = 0; j < k; j++) {
            const Lane &L = all[r0 + j];
            std::memcpy(cl[j].m, L.plan.m, sizeof(cl[j].m));
            cl[j].width = int(L.plan.width);
            cl[j].height = int(L.plan.height);
            cl[j].turns = L.plan.turns ? 1 : 0;
            cl[j].out = long(L.crop);
            cf[j] = crop_px;
            crop_px += long(L.plan.width * L.plan.height);
            size_t len = 0;
            float *in = ppocr_model_lane_device_input(rec, j, &len);
            if (!in || len != 48 * L.width * 3) return fail(PPOCR_E_UNSUPPORTED, "the recogniser's input is not 48 x width x 3");
            rl[j] = RecLine{long(L.crop), int(L.cw), int(L.ch), int(L.rw), int(L.width), in,
                            1.0 / (48.0 / double(L.ch)), 1.0 / (double(L.rw) / double(L.cw))};
            rf[j] = rec_px;
            rec_px += long(48 * L.width);
        }
        if (!cuda_ok(cudaMemcpyAsync(desc.p, desc_host.p, total, cudaMemcpyHostToDevice, stream), "copying crop plans in"))
            return PPOCR_E_DEVICE;
        const char *dd = desc.as<char>();
        CropArgs ca{prepared, int(prep.width), int(prep.height), reinterpret_cast<const CropLine *>(dd),
                    reinterpret_cast<const long *>(dd + off_cf), int(k), crop_px, crops.as<uint8_t>(), {}};
        launch_crops(ca, stream);
        RecLinesArgs ra{crops.as<uint8_t>(), reinterpret_cast<const RecLine *>(dd + off_rl),
                        reinterpret_cast<const long *>(dd + off_rf), int(k), rec_px};
        launch_rec_lines(ra, stream);
        if (!cuda_ok(cudaGetLastError(), "launching the crops")) return PPOCR_E_DEVICE;
        prep_stop();
        int rc = ppocr_model_enqueue_device(rec);
        if (rc) return rc;
        launches += 2 + ppocr_model_launches(rec);
        // the lanes' outputs lie back to back: one copy
        size_t first_len = 0, out_floats = 0;
        const float *out0 = ppocr_model_lane_device_output(rec, 0, 0, &first_len);
        std::vector<size_t> lens(k);
        for (size_t j = 0; j < k; j++) {
            ppocr_model_lane_device_output(rec, j, 0, &lens[j]);
            out_floats += lens[j];
        }
        if (!rec_host.fit(out_floats * sizeof(float), code)) return code;
        if (!cuda_ok(cudaMemcpyAsync(rec_host.p, out0, out_floats * sizeof(float), cudaMemcpyDeviceToHost, stream),
                     "copying the reads out"))
            return PPOCR_E_DEVICE;
        if ((rc = sync(timeout_ms))) return rc;
        if ((rc = ppocr_model_wait(rec, timeout_ms))) return rc;
        const float *ho = rec_host.as<float>();
        Clock cd(t_ns[T_DECODE]);
        for (size_t j = 0; j < k; j++) {
            auto &out = reads[all[r0 + j].quad];
            out.second = page::ctc_decode(ho, lens[j] / 2, dict, out.first);
            ho += lens[j];
        }
    }
    return PPOCR_OK;
}

// ------------------------------------------------------------------- C ABI

extern "C" {

void ppocr_reader_options_default(ppocr_reader_options *o) {
    if (!o) return;
    *o = ppocr_reader_options{};
    o->thresh = 0.3f;  // DbOptions::default (det.rs:305-315)
    o->box_thresh = 0.5;
    o->unclip_ratio = 1.5;
    o->max_candidates = 1000;
    o->text_score = 0.3;  // main.rs:122
    o->min_side = 30;     // PageOptions::default (det.rs:142-152)
    o->max_side = 4096;
    o->width_height_ratio = 8.0;
    o->min_height = 30;
    o->limit_min = 0;  // Limit::Max (main.rs:120)
    const double mean[3] = {0.485, 0.456, 0.406}, std_[3] = {0.229, 0.224, 0.225};  // ocr.rs:24-25
    for (int c = 0; c < 3; c++) {
        o->mean[c] = mean[c];
        o->std[c] = std_[c];
    }
}

int ppocr_reader_create(const ppocr_model *det, const ppocr_model *rec, const char *characters, size_t len,
                        const ppocr_reader_options *options, ppocr_reader **out) {
    set_last_error("");
    if (!det || !rec || !out || (!characters && len)) return fail(PPOCR_E_ARG, "null argument");
    *out = nullptr;
    auto r = std::make_unique<ppocr_reader>();
    if (options)
        r->opt = *options;
    else
        ppocr_reader_options_default(&r->opt);
    if (!(r->opt.max_side > 0) || r->opt.min_side > r->opt.max_side)
        return fail(PPOCR_E_ARG, "page sides: 0 < min_side <= max_side");
    int rc = ppocr_model_share_weights(det, &r->det);
    if (rc) return rc;
    if ((rc = ppocr_model_share_weights(rec, &r->rec))) return rc;
    r->dict = page::Dictionary::from_metadata(characters, len);
    r->stream = static_cast<cudaStream_t>(ppocr_model_stream(r->det));
    if ((rc = ppocr_model_set_stream(r->rec, r->stream))) return rc;
    // The recogniser's lanes change with every page: direct launches instead
    // of a graph captured once per set of sizes. Readers run several pages at
    // once, so both networks size their grids for throughput.
    if ((rc = ppocr_model_set_options(r->det, PPOCR_OPT_THROUGHPUT))) return rc;
    if ((rc = ppocr_model_set_options(r->rec, PPOCR_OPT_NO_GRAPH | PPOCR_OPT_THROUGHPUT))) return rc;
    if (!cuda_ok(cudaGetDevice(&r->device), "reading the device") ||
        !cuda_ok(cudaEventCreateWithFlags(&r->ev, cudaEventDisableTiming), "creating an event"))
        return PPOCR_E_DEVICE;
    configure_page_kernels();
    *out = r.release();
    return PPOCR_OK;
}

void ppocr_reader_free(ppocr_reader *r) { delete r; }

void *ppocr_reader_stream(ppocr_reader *r) { return r ? r->stream : nullptr; }

uint8_t *ppocr_reader_page(ppocr_reader *r, size_t width, size_t height) {
    if (!r || !width || !height || width > (1u << 20) || height > (1u << 20)) {
        fail(PPOCR_E_ARG, "page sizes must be between 1 and 2^20");
        return nullptr;
    }
    int code = PPOCR_OK;
    cudaSetDevice(r->device);
    if (!r->page_host.fit(width * height * 3, code)) return nullptr;
    return r->page_host.as<uint8_t>();
}

int ppocr_reader_detect(ppocr_reader *r, const uint8_t *page, size_t width, size_t height, uint32_t timeout_ms) {
    set_last_error("");
    if (!r || (!page && width && height)) return fail(PPOCR_E_ARG, "null argument");
    if (width > (1u << 20) || height > (1u << 20)) return fail(PPOCR_E_SIZE, "page sides above 2^20");
    return r->detect(page, width, height, timeout_ms);
}

int ppocr_reader_detect_device(ppocr_reader *r, const uint8_t *page, size_t width, size_t height,
                               uint32_t timeout_ms) {
    set_last_error("");
    if (!r || (!page && width && height)) return fail(PPOCR_E_ARG, "null argument");
    if (width > (1u << 20) || height > (1u << 20)) return fail(PPOCR_E_SIZE, "page sides above 2^20");
    return r->detect(page, width, height, timeout_ms, true);
}

size_t ppocr_reader_launches(const ppocr_reader *r) { return r ? r->launches : 0; }

size_t ppocr_reader_box_count(const ppocr_reader *r) { return r ? r->found.size() : 0; }

const float *ppocr_reader_boxes(const ppocr_reader *r) {
    return r && !r->found.empty() ? &r->found[0][0].x : nullptr;
}

int ppocr_reader_prepared(const ppocr_reader *r, size_t *width, size_t *height, double *ratio_w, double *ratio_h,
                          size_t *pad_top) {
    if (!r || !r->have_page) return fail(PPOCR_E_ARG, "no page");
    if (width) *width = r->prep.width;
    if (height) *height = r->prep.height;
    if (ratio_w) *ratio_w = r->prep.ratio_w;
    if (ratio_h) *ratio_h = r->prep.ratio_h;
    if (pad_top) *pad_top = r->prep.pad_top;
    return PPOCR_OK;
}

int ppocr_reader_recognise(ppocr_reader *r, const float *quads, size_t n, uint32_t timeout_ms) {
    set_last_error("");
    if (!r || (!quads && n)) return fail(PPOCR_E_ARG, "null argument");
    std::vector<Quad> q(n);
    if (n) std::memcpy(q.data(), quads, n * sizeof(Quad));
    return r->recognise(q.data(), n, timeout_ms);
}

size_t ppocr_reader_text_count(const ppocr_reader *r) { return r ? r->reads.size() : 0; }

int ppocr_reader_text(const ppocr_reader *r, size_t i, const char **text, double *score) {
    if (!r || i >= r->reads.size()) return fail(PPOCR_E_ARG, "no such read");
    if (text) *text = r->reads[i].first.c_str();
    if (score) *score = r->reads[i].second;
    return PPOCR_OK;
}

// ocr.rs:234-263 Reader::read without the vertical re-read: detection, the
// boxes read, then page_lines (lib.rs:96-129): blank or low-scoring lines
// dropped (a NaN score is kept), boxes mapped back to the page as given.
int ppocr_reader_read(ppocr_reader *r, const uint8_t *page, size_t width, size_t height, uint32_t timeout_ms) {
    int rc = ppocr_reader_detect(r, page, width, height, timeout_ms);
    if (rc) return rc;
    if (!r->have_page) return PPOCR_OK;
    const std::vector<Quad> boxes = r->found;
    if ((rc = r->recognise(boxes.data(), boxes.size(), timeout_ms))) return rc;
    for (size_t i = 0; i < boxes.size(); i++) {
        const auto &rd = r->reads[i];
        if (page::is_blank(rd.first) || rd.second < r->opt.text_score) continue;
        r->lines.push_back(ppocr_reader::Line{
            page::to_page(boxes[i], r->prep.ratio_w, r->prep.ratio_h, r->prep.pad_top, width, height), rd.first,
            rd.second});
    }
    return PPOCR_OK;
}

size_t ppocr_reader_line_count(const ppocr_reader *r) { return r ? r->lines.size() : 0; }

int ppocr_reader_line(const ppocr_reader *r, size_t i, float quad[8], const char **text, double *score) {
    if (!r || i >= r->lines.size()) return fail(PPOCR_E_ARG, "no such line");
    if (quad) std::memcpy(quad, &r->lines[i].quad[0].x, 8 * sizeof(float));
    if (text) *text = r->lines[i].text.c_str();
    if (score) *score = r->lines[i].score;
    return PPOCR_OK;
}

int ppocr_reader_set_options(ppocr_reader *r, uint32_t options) {
    set_last_error("");
    if (!r) return fail(PPOCR_E_ARG, "null reader");
    int rc = ppocr_model_set_options(r->det, options | PPOCR_OPT_THROUGHPUT);
    if (rc) return rc;
    if ((rc = ppocr_model_set_options(r->rec, options | PPOCR_OPT_NO_GRAPH | PPOCR_OPT_THROUGHPUT))) return rc;
    r->det_w = r->det_h = 0;  // sizes are set again at the next page
    r->rec_sizes.clear();
    return PPOCR_OK;
}

int ppocr_reader_prob_map(ppocr_reader *r, float *out, size_t capacity, size_t *width, size_t *height) {
    set_last_error("");
    if (!r || !width || !height) return fail(PPOCR_E_ARG, "null argument");
    if (!r->have_page) return fail(PPOCR_E_ARG, "no page");
    *width = r->det_w;
    *height = r->det_h;
    if (!out || capacity < r->det_w * r->det_h) return fail(PPOCR_E_SIZE, "out holds fewer than the map's floats");
    size_t len = 0;
    const float *prob = ppocr_model_lane_device_output(r->det, 0, 0, &len);
    if (!cuda_ok(cudaSetDevice(r->device), "selecting the device") ||
        !cuda_ok(cudaMemcpyAsync(out, prob, len * sizeof(float), cudaMemcpyDeviceToHost, r->stream), "copying the map") ||
        !cuda_ok(cudaStreamSynchronize(r->stream), "copying the map"))
        return PPOCR_E_DEVICE;
    return PPOCR_OK;
}

int ppocr_reader_host_times(const ppocr_reader *r, double seconds[5]) {
    if (!r || !seconds) return fail(PPOCR_E_ARG, "null argument");
    for (int i = 0; i < ppocr_reader::T_COUNT; i++) seconds[i] = double(r->t_ns[i]) * 1e-9;
    return PPOCR_OK;
}

int ppocr_reader_stats(const ppocr_reader *r, size_t *scored, size_t *rescored) {
    if (!r) return fail(PPOCR_E_ARG, "null reader");
    if (scored) *scored = r->scored;
    if (rescored) *rescored = r->rescored;
    return PPOCR_OK;
}

// ---- host page steps

int ppocr_find_contours(const uint8_t *mask, size_t width, size_t height, int32_t *points, size_t points_cap,
                        size_t *starts, size_t starts_cap, size_t *contours, size_t *npoints) {
    set_last_error("");
    if ((!mask && width * height) || !contours || !npoints) return fail(PPOCR_E_ARG, "null argument");
    page::Contours cs;
    page::ContourScratch s;
    page::find_contours(mask, width, height, cs, s);
    *contours = cs.size();
    *npoints = cs.pts.size();
    if (cs.pts.size() > points_cap || cs.size() + 1 > starts_cap || (!points && !cs.pts.empty()) || !starts)
        return fail(PPOCR_E_SIZE, "the contours need " + std::to_string(cs.pts.size()) + " points and " +
                                      std::to_string(cs.size() + 1) + " starts");
    for (size_t i = 0; i < cs.pts.size(); i++) {
        points[2 * i] = cs.pts[i].x;
        points[2 * i + 1] = cs.pts[i].y;
    }
    for (size_t i = 0; i <= cs.size(); i++) starts[i] = cs.start[i];
    return PPOCR_OK;
}

int ppocr_contour_mean(const float *map, size_t width, size_t height, const int32_t *points, size_t n,
                       double *mean) {
    if (!map || !width || !height || (!points && n) || !mean) return fail(PPOCR_E_ARG, "null argument or empty map");
    *mean = page::contour_mean(map, width, height, reinterpret_cast<const Point *>(points), n);
    return PPOCR_OK;
}

int ppocr_min_area_rect(const int32_t *points, size_t n, float rect[5]) {
    if ((!points && n) || !rect) return fail(PPOCR_E_ARG, "null argument");
    const page::RotatedRect r = page::min_area_rect(reinterpret_cast<const Point *>(points), n);
    rect[0] = r.cx;
    rect[1] = r.cy;
    rect[2] = r.width;
    rect[3] = r.height;
    rect[4] = r.angle;
    return PPOCR_OK;
}

int ppocr_box_points(const float rect[5], float quad[8]) {
    if (!rect || !quad) return fail(PPOCR_E_ARG, "null argument");
    const Quad q = page::box_points(page::RotatedRect{rect[0], rect[1], rect[2], rect[3], rect[4]});
    std::memcpy(quad, &q[0].x, sizeof(q));
    return PPOCR_OK;
}

int ppocr_mini_box(const int32_t *points, size_t n, float quad[8], float *side) {
    if ((!points && n) || !quad || !side) return fail(PPOCR_E_ARG, "null argument");
    Quad q;
    *side = page::mini_box(reinterpret_cast<const Point *>(points), n, q);
    std::memcpy(quad, &q[0].x, sizeof(q));
    return PPOCR_OK;
}

int ppocr_unclip(const float quad[8], double ratio, int32_t *out, size_t cap, size_t *n) {
    if (!quad || !n) return fail(PPOCR_E_ARG, "null argument");
    Quad q;
    std::memcpy(&q[0].x, quad, sizeof(q));
    const std::vector<Point> ring = page::unclip(q, ratio);
    *n = ring.size();
    if (ring.size() > cap || (!out && !ring.empty()))
        return fail(PPOCR_E_SIZE, "the ring has " + std::to_string(ring.size()) + " points");
    for (size_t i = 0; i < ring.size(); i++) {
        out[2 * i] = ring[i].x;
        out[2 * i + 1] = ring[i].y;
    }
    return PPOCR_OK;
}

int ppocr_boxes_from_prob(const float *prob, size_t map_w, size_t map_h, size_t dest_w, size_t dest_h, float thresh,
                          double box_thresh, double unclip_ratio, size_t max_candidates, float *quads, size_t cap,
                          size_t *n) {
    if ((!prob && map_w * map_h) || !n) return fail(PPOCR_E_ARG, "null argument");
    page::DbOptions o;
    o.thresh = thresh;
    o.box_thresh = box_thresh;
    o.unclip_ratio = unclip_ratio;
    o.max_candidates = max_candidates;
    const std::vector<Quad> boxes = page::boxes_from_prob(prob, map_w, map_h, dest_w, dest_h, o);
    *n = boxes.size();
    if (boxes.size() > cap || (!quads && !boxes.empty()))
        return fail(PPOCR_E_SIZE, std::to_string(boxes.size()) + " boxes");
    if (!boxes.empty()) std::memcpy(quads, boxes.data(), boxes.size() * sizeof(Quad));
    return PPOCR_OK;
}

int ppocr_det_size(size_t width, size_t height, size_t limit_min, size_t *out_width, size_t *out_height) {
    if (!out_width || !out_height) return fail(PPOCR_E_ARG, "null argument");
    if (!page::det_size(width, height, limit_min, *out_width, *out_height))
        return fail(PPOCR_E_SIZE, "a side would vanish");
    return PPOCR_OK;
}

int ppocr_prepare_page(size_t width, size_t height, const ppocr_reader_options *o, size_t *out_width,
                       size_t *out_height, double *ratio_w, double *ratio_h, size_t *pad_top) {
    ppocr_reader_options d;
    if (!o) {
        ppocr_reader_options_default(&d);
        o = &d;
    }
    page::Prepared p;
    if (!page::prepare_page(width, height, o->min_side, o->max_side, o->width_height_ratio, o->min_height, p))
        return fail(PPOCR_E_SIZE, "no page at these sizes");
    if (out_width) *out_width = p.width;
    if (out_height) *out_height = p.height;
    if (ratio_w) *ratio_w = p.ratio_w;
    if (ratio_h) *ratio_h = p.ratio_h;
    if (pad_top) *pad_top = p.pad_top;
    return PPOCR_OK;
}

int ppocr_crop_size(const float quad[8], size_t *width, size_t *height) {
    if (!quad || !width || !height) return fail(PPOCR_E_ARG, "null argument");
    Quad q;
    std::memcpy(&q[0].x, quad, sizeof(q));
    const page::CropPlan c = page::plan_crop(q);
    *width = c.turns ? c.height : c.width;
    *height = c.turns ? c.width : c.height;
    return PPOCR_OK;
}

int ppocr_crop_text(const uint8_t *image, size_t width, size_t height, const float quad[8], uint8_t *out,
                    size_t capacity, void *stream) {
    if (!image || !quad || !out) return fail(PPOCR_E_ARG, "null argument");
    if (!width || !height || width > (1u << 20) || height > (1u << 20))
        return fail(PPOCR_E_SIZE, "image sizes must be between 1 and 2^20");
    Quad q;
    std::memcpy(&q[0].x, quad, sizeof(q));
    const page::CropPlan c = page::plan_crop(q);
    const size_t bytes = c.width * c.height * 3;
    if (capacity < bytes) return fail(PPOCR_E_SIZE, "out holds fewer than the crop's bytes");
    if (!bytes) return PPOCR_OK;
    if (c.width * c.height > (size_t(1) << 31)) return fail(PPOCR_E_SIZE, "the crop is too large");
    // One line: its plan travels in the kernel's parameters, nothing is
    // allocated or copied.
    CropArgs a{image, int(width), int(height), nullptr, nullptr, 1, long(c.width * c.height), out, {}};
    std::memcpy(a.single.m, c.m, sizeof(c.m));
    a.single.width = int(c.width);
    a.single.height = int(c.height);
    a.single.turns = c.turns ? 1 : 0;
    a.single.out = 0;
    launch_crops(a, static_cast<cudaStream_t>(stream));
    if (!cuda_ok(cudaGetLastError(), "launching the crop")) return PPOCR_E_DEVICE;
    return PPOCR_OK;
}

struct ppocr_dictionary {
    page::Dictionary d;
};

int ppocr_dictionary_load(const char *text, size_t len, ppocr_dictionary **out) {
    if ((!text && len) || !out) return fail(PPOCR_E_ARG, "null argument");
    *out = new ppocr_dictionary{page::Dictionary::from_metadata(text, len)};
    return PPOCR_OK;
}

size_t ppocr_dictionary_size(const ppocr_dictionary *d) { return d ? d->d.classes.size() : 0; }

const char *ppocr_dictionary_class(const ppocr_dictionary *d, size_t i, size_t *len) {
    if (!d || i >= d->d.classes.size()) return nullptr;
    if (len) *len = d->d.classes[i].size();
    return d->d.classes[i].data();
}

void ppocr_dictionary_free(ppocr_dictionary *d) { delete d; }

int ppocr_ctc_decode(const float *output, size_t steps, const ppocr_dictionary *d, char *text, size_t capacity,
                     size_t *len, double *score) {
    if ((!output && steps) || !d || !len || !score) return fail(PPOCR_E_ARG, "null argument");
    std::string t;
    *score = page::ctc_decode(output, steps, d->d, t);
    *len = t.size();
    if (t.size() + 1 > capacity || !text) return fail(PPOCR_E_SIZE, "the text needs " + std::to_string(t.size() + 1) + " bytes");
    std::memcpy(text, t.c_str(), t.size() + 1);
    return PPOCR_OK;
}

int ppocr_text_is_blank(const char *text, size_t len) {
    return page::is_blank(std::string(text ? text : "", text ? len : 0)) ? 1 : 0;
}

}  // extern "C"
