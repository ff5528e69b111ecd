/* ppocr_cuda.h — C ABI of libppocr_cuda.so, the B200 (sm_100a) backend of
 * the ppocr-native engine.
 *
 * It replaces the Vulkan `GpuModel` of ppocr-native
 * (`src/engine/gpu/mod.rs:81-291`) behind the same calls: a model is a
 * PPOCRPL1 plan loaded onto one GPU, run over one or more images ("lanes")
 * at a time, each lane with its own input height and width. Lanes of equal
 * size run as one batch. The library owns page-locked host buffers for
 * every lane's input and outputs; their pointers stay valid until the next
 * ppocr_model_set_sizes / ppocr_model_free.
 *
 * Every call returns a status (PPOCR_OK = 0) and never throws or aborts; the
 * reason for the last failure on the calling thread is ppocr_last_error().
 * On a failed resize the model keeps its previous sizes
 * (`src/engine/mod.rs:425-446`). Calls on one model are not thread-safe;
 * different models are independent.
 *
 * No PyTorch, Vulkan or CPU fallback sits on this path: a model that cannot
 * run on the GPU returns an error, and the caller decides what to do.
 */
#ifndef PPOCR_CUDA_H
#define PPOCR_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ppocr_model ppocr_model;

enum {
    PPOCR_OK = 0,
    PPOCR_E_PLAN = 1,        /* the plan file is unreadable, malformed or inconsistent */
    PPOCR_E_SIZE = 2,        /* the requested input size does not fit the plan */
    PPOCR_E_NOMEM = 3,       /* device or page-locked host memory ran out */
    PPOCR_E_DEVICE = 4,      /* a CUDA call failed or no usable device */
    PPOCR_E_TIMEOUT = 5,     /* the GPU did not finish within the timeout */
    PPOCR_E_UNSUPPORTED = 6, /* an operation this backend does not run */
    PPOCR_E_ARG = 7          /* a bad argument (null pointer, lane out of range) */
};

/* Bits of ppocr_model_set_options. */
enum {
    PPOCR_OPT_NO_FUSION = 1, /* run every plan operation as its own kernel */
    PPOCR_OPT_NO_GRAPH = 2,  /* launch kernels directly instead of replaying a CUDA graph */
    PPOCR_OPT_NO_TENSOR_CORES = 4, /* every contraction on the FP32 cores: the reference CPU engine's bits */
    PPOCR_OPT_THROUGHPUT = 8       /* size grids for several runs in flight: small tensor-core layers take few
                                      SMs (same results, longer latency alone, more pages per second together) */
};

/* Number of CUDA devices this process can use (0 when none). */
int ppocr_device_count(void);

/* Reason for the last failed call on this thread ("" after success). */
const char *ppocr_last_error(void);

/* Load and check a plan (replaces `GpuModel::load`, gpu/mod.rs:113-163),
 * with one lane at the size the plan was exported at. */
int ppocr_model_load(const char *plan_path, int device, ppocr_model **out);
/* The same from a plan held in memory. */
int ppocr_model_load_bytes(const void *bytes, size_t len, int device, ppocr_model **out);
/* A second model on the same device sharing the first one's weights
 * (`Model::try_clone`, src/engine/mod.rs:318). */
int ppocr_model_share_weights(const ppocr_model *src, ppocr_model **out);
void ppocr_model_free(ppocr_model *model);

/* The GPU's name (`GpuModel::device`, gpu/mod.rs:165-168). */
const char *ppocr_model_device_name(const ppocr_model *model);
/* 1 when the GPU shares memory with the CPU (`GpuModel::integrated`, :170-173). */
int ppocr_model_integrated(const ppocr_model *model);
/* Most lanes one run takes (`GpuModel::max_lanes`, :177-181). */
size_t ppocr_model_max_lanes(const ppocr_model *model);
size_t ppocr_model_output_count(const ppocr_model *model);

/* One lane of height x width (`GpuModel::set_input_size`, :175-177). */
int ppocr_model_set_input_size(ppocr_model *model, uint32_t height, uint32_t width);
/* One lane per (height, width) pair in hw_pairs[2*i], hw_pairs[2*i+1]
 * (`GpuModel::set_sizes`, :184-230). */
int ppocr_model_set_sizes(ppocr_model *model, const uint32_t *hw_pairs, size_t lanes);

/* The lane's HWC input in page-locked host memory, to be filled before each
 * run (`GpuModel::lane_input_mut`, :240-246); *len receives its floats. Its
 * contents after ppocr_model_set_sizes are unspecified (buffers are kept
 * across sizes, never cleared). */
float *ppocr_model_lane_input(ppocr_model *model, size_t lane, size_t *len);
/* Output `index` of the lane's last run (`GpuModel::lane_output`, :255-259). */
const float *ppocr_model_lane_output(const ppocr_model *model, size_t lane, size_t index, size_t *len);

/* Copy every lane's input to the GPU, run the network, copy the outputs
 * back and wait at most timeout_ms (0 = no limit) (`GpuModel::run`,
 * :262-290, whose fence wait has no limit, vk.rs:373-378). */
int ppocr_model_run(ppocr_model *model, uint32_t timeout_ms);
/* ppocr_model_run split in two, so that the host can prepare the next
 * batch while the GPU runs this one. */
int ppocr_model_enqueue(ppocr_model *model);
int ppocr_model_wait(ppocr_model *model, uint32_t timeout_ms);

/* Device-resident use, for callers whose inputs are produced on the GPU:
 * the lane's input / output tensors in device memory, and a run that copies
 * nothing (the outputs stay on the device). */
float *ppocr_model_lane_device_input(ppocr_model *model, size_t lane, size_t *len);
const float *ppocr_model_lane_device_output(const ppocr_model *model, size_t lane, size_t index, size_t *len);
int ppocr_model_enqueue_device(ppocr_model *model);
/* The cudaStream_t every kernel of this model runs on. */
void *ppocr_model_stream(ppocr_model *model);
/* Run this model on the caller's cudaStream_t (NULL: its own again), e.g.
 * to queue several models behind one another without host waits. The
 * caller keeps that stream alive while the model may still use it; freeing
 * the model waits only for the model's own work, not for the stream. */
int ppocr_model_set_stream(ppocr_model *model, void *stream);

/* PPOCR_OPT_* bits; takes effect at the next run. */
int ppocr_model_set_options(ppocr_model *model, uint32_t options);
/* Kernel launches one run makes at the current sizes (copies excluded). */
size_t ppocr_model_launches(const ppocr_model *model);
/* A text line describing step `i` of the fused schedule (NULL past the end). */
const char *ppocr_model_step_name(const ppocr_model *model, size_t i);

/* The CTC argmax head (plan kind ctcargmax, the recogniser's last layer)
 * over device buffers the caller owns, for callers that may not allocate
 * device memory: hosts that manage a fixed device-memory budget themselves,
 * or loops that must not stall on cudaMalloc / cudaFree, which can
 * synchronize the device. No counterpart in the reference (its engine always
 * allocates per model). x: [pixels][ci] time steps; w: ceil(vocab/16) panels
 * of [ci][16]; b: 16 * ceil(vocab/16) biases (-1e30 past vocab); y:
 * [pixels][2] = (best class as float, 1 / sum of exp). w must be 16-byte
 * aligned (its panels are read as 16-byte vectors), x, b and y 4-byte
 * aligned; a misaligned pointer returns PPOCR_E_ARG before any launch.
 * Enqueued on `stream` (a cudaStream_t; NULL is the default stream) on the
 * current device.
 * Allocates nothing: its scratch is a fixed 4 MiB array in the library's
 * device memory (3 floats per time step per 128 classes, 1 Mi floats in
 * all); larger calls return PPOCR_E_SIZE. The first call on a device looks
 * the array up and raises the kernels' shared-memory limits on that device
 * (no model needs to exist), so make it before any stream capture. All calls on a device
 * share the array: calls that overlap on the GPU race. */
int ppocr_ctc_argmax_noalloc(const float *x, const float *w, const float *b, float *y, size_t pixels,
                             size_t ci, size_t vocab, void *stream);

/* The detector's input on the GPU (replaces the CPU preparation of the page
 * before the detector runs: det_input_hwc, reference src/det.rs:230-292,
 * with resize_linear_rows, src/image.rs:91-142): `image` (device memory,
 * width x height RGB bytes, rows of width * 3) resized to out_width x
 * out_height by OpenCV's INTER_LINEAR in the reference's integer staging,
 * scaled to [0, 1] and normalized per channel ((x - mean[c]) / std[c] in
 * f64, rounded once to f32), written to `out` (device memory, out_height x
 * out_width x 3 floats: the detector's input layout; `capacity` floats
 * available, PPOCR_E_SIZE when fewer) on `stream` (NULL: the default
 * stream). The same bytes and bits as the reference's CPU path. Sizes from
 * 1 to 2^20; allocates nothing. */
int ppocr_det_input_hwc(const uint8_t *image, size_t width, size_t height, size_t out_width, size_t out_height,
                        const double *mean, const double *std, float *out, size_t capacity, void *stream);

/* The recogniser's input for one line crop on the GPU (replaces rec_input,
 * reference src/rec.rs:19-43, turned HWC as ocr.rs:534-549 rec_hwc does):
 * `crop` (device memory, width x height RGB bytes) resized to height 48 at
 * its aspect ratio (width rounded up, cut to the tensor), scaled to [-1, 1]
 * in f32 and zero-padded on the right to the tensor width
 * max(320, trunc(48 * width / height)), written to `out` (device memory,
 * 48 x tensor_width x 3 floats, `capacity` floats available) on `stream`.
 * *tensor_width receives the width; with out NULL only the width is
 * computed. The same bytes and bits as the reference's CPU path. Crop sizes
 * from 1 to 2^20; allocates nothing. */
int ppocr_rec_input_hwc(const uint8_t *crop, size_t width, size_t height, float *out, size_t capacity,
                        size_t *tensor_width, void *stream);

/* The DB postprocess's text mask on the GPU (the first line of
 * boxes_from_prob, reference src/det.rs:438): mask[i] = prob[i] > thresh,
 * compared in f32, for `pixels` values of the detector's probability map
 * (device memory in and out) on `stream`. Allocates nothing. */
int ppocr_db_mask(const float *prob, size_t pixels, float thresh, uint8_t *mask, void *stream);

/* ------------------------------------------------------------------------
 * Page reading: the steps around the two networks.
 *
 * The reference's library exposes its page steps as plain functions the
 * worker strings together (src/lib.rs:15-48, re-exports at :533-544); its
 * worker's Reader reads a page with them and the two networks
 * (src/bin/ppocr-native/ocr.rs:205-263). The host steps below are those
 * functions, bit for bit (border following, boxes, unclip, page sizes,
 * CTC decode, the dictionary); a reader runs the whole page on the GPU
 * where the step is data-parallel (page fit, detector input, text mask, box
 * scores, crops, recogniser inputs) and on the calling thread where it is
 * sequential. Quads are 8 floats: top-left, top-right, bottom-right,
 * bottom-left, (x, y) each. Images are RGB (or BGR: channel order is kept)
 * bytes, rows of width * 3.
 * ---------------------------------------------------------------------- */

/* The worker's options (det.rs:142-152 PageOptions, :305-315 DbOptions,
 * main.rs:112-122, ocr.rs:20-25 MEAN / STD). */
typedef struct {
    float thresh;              /* text pixel: prob > thresh (0.3) */
    double box_thresh;         /* mean probability a box needs (0.5) */
    double unclip_ratio;       /* growth: area * ratio / perimeter (1.5) */
    uint32_t max_candidates;   /* contours considered (1000) */
    double text_score;         /* lines scoring less are dropped (0.3) */
    uint32_t min_side, max_side;   /* page fit (30, 4096) */
    double width_height_ratio; /* vertical padding rule (8; -1 turns it off) */
    uint32_t min_height;       /* (30) */
    uint32_t limit_min;        /* 0: Limit::Max (960/1500/2000); else Limit::Min(limit_min) */
    double mean[3], std[3];    /* detector normalization per channel */
} ppocr_reader_options;

typedef struct ppocr_reader ppocr_reader;

void ppocr_reader_options_default(ppocr_reader_options *options);
/* A reader over a detector and a recogniser (an argmax recogniser: output
 * [steps][2] = (class, probability)) whose weights it shares, with the
 * recogniser's classes from `characters` (the model's metadata, one class
 * per line, as rec.rs:54-79 Dictionary::from_metadata). The reader makes
 * its own models and stream (replaces ocr.rs:114-201 Reader::load). */
int ppocr_reader_create(const ppocr_model *det, const ppocr_model *rec, const char *characters, size_t len,
                        const ppocr_reader_options *options, ppocr_reader **out);
void ppocr_reader_free(ppocr_reader *reader);
/* The cudaStream_t the reader runs on. */
void *ppocr_reader_stream(ppocr_reader *reader);
/* Page-locked host memory for a width x height page, valid until the next
 * call or ppocr_reader_free; a page written there and passed to
 * ppocr_reader_detect / _read is copied to the GPU at full speed (any other
 * host pointer works too, through the driver's staging). */
uint8_t *ppocr_reader_page(ppocr_reader *reader, size_t width, size_t height);
/* Detection (ocr.rs:205-231 Reader::detect): the page prepared (fit and
 * padding, det.rs:110-131), the detector at det_size, the DB postprocess
 * (det.rs:430-452). The boxes (on the prepared page, in reading order)
 * stay until the next call. A page with no usable size has no boxes. */
int ppocr_reader_detect(ppocr_reader *reader, const uint8_t *page, size_t width, size_t height,
                        uint32_t timeout_ms);
/* The same for a page already in device memory (read where it lies: keep
 * it unchanged until the next detection, or the recognition after it,
 * returns). */
int ppocr_reader_detect_device(ppocr_reader *reader, const uint8_t *page, size_t width, size_t height,
                               uint32_t timeout_ms);
/* Kernels the last detection and the recognitions after it launched. */
size_t ppocr_reader_launches(const ppocr_reader *reader);
size_t ppocr_reader_box_count(const ppocr_reader *reader);
const float *ppocr_reader_boxes(const ppocr_reader *reader);
/* The prepared page of the last detection: its size, the ratios back to
 * the page as given and the padding band (det.rs:28-38 PreparedPage). */
int ppocr_reader_prepared(const ppocr_reader *reader, size_t *width, size_t *height, double *ratio_w,
                          double *ratio_h, size_t *pad_top);
/* Recognition of n quads on the prepared page of the last detection
 * (ocr.rs:436-530 recognise_on_gpu / read_on_gpu): crops (crop.rs:84-127),
 * recogniser inputs (rec.rs:19-43), the recogniser, CTC decode
 * (rec.rs:144-161). Read i is quad i's text and score. */
int ppocr_reader_recognise(ppocr_reader *reader, const float *quads, size_t n, uint32_t timeout_ms);
size_t ppocr_reader_text_count(const ppocr_reader *reader);
int ppocr_reader_text(const ppocr_reader *reader, size_t i, const char **text, double *score);
/* A whole page (ocr.rs:234-263 Reader::read, without its vertical re-read
 * of low-scoring vertical lines): detection, the boxes read, then
 * page_lines (lib.rs:96-129): blank or low-scoring lines dropped, boxes
 * mapped back to the page as given. */
int ppocr_reader_read(ppocr_reader *reader, const uint8_t *page, size_t width, size_t height, uint32_t timeout_ms);
size_t ppocr_reader_line_count(const ppocr_reader *reader);
int ppocr_reader_line(const ppocr_reader *reader, size_t i, float quad[8], const char **text, double *score);
/* PPOCR_OPT_* bits for the reader's models (PPOCR_OPT_NO_TENSOR_CORES:
 * both networks in the reference CPU engine's exact arithmetic). */
int ppocr_reader_set_options(ppocr_reader *reader, uint32_t options);
/* The detector's probability map of the last detection (host memory,
 * capacity floats; *width x *height values). */
int ppocr_reader_prob_map(ppocr_reader *reader, float *out, size_t capacity, size_t *width, size_t *height);
/* Host seconds this reader has spent, summed over its calls, in: waits for
 * the GPU, border following, box geometry (minimum-area boxes, scores'
 * check, unclip, order), recogniser set-up (crop maps, lane sizes,
 * descriptors), CTC decoding. */
int ppocr_reader_host_times(const ppocr_reader *reader, double seconds[5]);
/* Contours the GPU scored, and how many of those the host scored again in
 * the reference's summation order because their mean lay within the
 * parallel sum's error bound of box_thresh. */
int ppocr_reader_stats(const ppocr_reader *reader, size_t *scored, size_t *rescored);

/* cv2.findContours(mask, RETR_LIST, CHAIN_APPROX_SIMPLE) (contour.rs:44-130):
 * contour i is points[2*starts[i] .. 2*starts[i+1]); *contours and *npoints
 * receive the counts, PPOCR_E_SIZE when the capacities are short. */
int ppocr_find_contours(const uint8_t *mask, size_t width, size_t height, int32_t *points, size_t points_cap,
                        size_t *starts, size_t starts_cap, size_t *contours, size_t *npoints);
/* The map's f64 mean inside a contour (contour.rs:142-199). */
int ppocr_contour_mean(const float *map, size_t width, size_t height, const int32_t *points, size_t n,
                       double *mean);
/* cv2.minAreaRect as OpenCV 5 computes it (geometry.rs:406-457):
 * rect = {cx, cy, width, height, angle in degrees}. */
int ppocr_min_area_rect(const int32_t *points, size_t n, float rect[5]);
/* cv2.boxPoints (geometry.rs:228-240). */
int ppocr_box_points(const float rect[5], float quad[8]);
/* RapidOCR's get_mini_boxes (geometry.rs:462-477): ordered corners and the
 * shorter side. */
int ppocr_mini_box(const int32_t *points, size_t n, float quad[8], float *side);
/* RapidOCR's unclip (geometry.rs:519-606, pyclipper's round offset): ring
 * points into out (cap points), their count in *n. */
int ppocr_unclip(const float quad[8], double ratio, int32_t *out, size_t cap, size_t *n);
/* The DB postprocess on the host (det.rs:430-452): quads in reading order
 * on a dest_w x dest_h page. */
int ppocr_boxes_from_prob(const float *prob, size_t map_w, size_t map_h, size_t dest_w, size_t dest_h, float thresh,
                          double box_thresh, double unclip_ratio, size_t max_candidates, float *quads, size_t cap,
                          size_t *n);
/* The detector input size (det.rs:166-193): limit_min 0 is Limit::Max. */
int ppocr_det_size(size_t width, size_t height, size_t limit_min, size_t *out_width, size_t *out_height);
/* prepare_page's sizes (det.rs:44-131) under `options` (NULL: defaults). */
int ppocr_prepare_page(size_t width, size_t height, const ppocr_reader_options *options, size_t *out_width,
                       size_t *out_height, double *ratio_w, double *ratio_h, size_t *pad_top);
/* The size of crop_text's result for a quad, turned when tall. */
int ppocr_crop_size(const float quad[8], size_t *width, size_t *height);
/* crop_text on the GPU (crop.rs:84-127): the quad straightened out of
 * `image` (device memory) by its projective map and Keys' bicubic taps,
 * turned a quarter counter-clockwise when 1.5 times taller than wide, into
 * `out` (device memory, capacity bytes) on `stream`. Allocates nothing. */
int ppocr_crop_text(const uint8_t *image, size_t width, size_t height, const float quad[8], uint8_t *out,
                    size_t capacity, void *stream);

/* The recogniser's classes (rec.rs:54-79): blank, the metadata's lines as
 * Python's str.splitlines splits them, a space. */
typedef struct ppocr_dictionary ppocr_dictionary;
int ppocr_dictionary_load(const char *text, size_t len, ppocr_dictionary **out);
size_t ppocr_dictionary_size(const ppocr_dictionary *d);
const char *ppocr_dictionary_class(const ppocr_dictionary *d, size_t i, size_t *len);
void ppocr_dictionary_free(ppocr_dictionary *d);
/* RapidOCR's greedy CTC decode of an argmax recogniser's [steps][2] output
 * (rec.rs:144-161, ocr.rs:551-560): UTF-8 text (NUL-terminated, capacity
 * bytes) and its score. */
int ppocr_ctc_decode(const float *output, size_t steps, const ppocr_dictionary *d, char *text, size_t capacity,
                     size_t *len, double *score);
/* 1 when the text is only white space (rec.rs:168-172). */
int ppocr_text_is_blank(const char *text, size_t len);

#ifdef __cplusplus
}
#endif
#endif
