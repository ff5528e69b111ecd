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
    PPOCR_OPT_NO_TENSOR_CORES = 4 /* every contraction on the FP32 cores: the reference CPU engine's bits */
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
 * run (`GpuModel::lane_input_mut`, :240-246); *len receives its floats. */
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

#ifdef __cplusplus
}
#endif
#endif
