/* TEST INFRASTRUCTURE ONLY: the CPU oracle for parity tests, smoke() and
 * bench.py's cpu_baseline / reference arm. The product library never links,
 * loads or calls it.
 *
 * A C restatement of ppocr-native's CPU engine (`src/engine/plan.rs`,
 * `conv.rs`, `layers.rs`, `kernels/` sources), executed op by op. The reference
 * schedules fused steps, but its own tests require every fused step to give
 * the bits of op-by-op execution (`src/engine/schedule.rs:642-664`), so the
 * op-by-op form is the definition.
 *
 * Pinning: the reference ships no network-level golden vectors (its engine
 * tests compare each kernel to an f64 definition); the Rust toolchain needed
 * to run the reference here is absent. This oracle is pinned to the same f64
 * definitions and bounds the reference's tests use (tests/test_oracle.py);
 * network-level parity against the reference binary is unpinned.
 */
#ifndef PPOCR_ORACLE_H
#define PPOCR_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct orc_plan orc_plan;

/* Parse and check a PPOCRPL1 plan (plan.rs:303-365); NULL on error with the
 * reason in err. The plan keeps its own copy of the weights. */
orc_plan *orc_load(const uint8_t *bytes, size_t len, char *err, size_t errlen);
void orc_free(orc_plan *p);
/* Re-derive every shape for an input height x width (plan.rs:383-398). */
int orc_set_size(orc_plan *p, size_t h, size_t w, char *err, size_t errlen);
size_t orc_input_len(const orc_plan *p);
size_t orc_output_count(const orc_plan *p);
size_t orc_output_len(const orc_plan *p, size_t k);
/* Run the plan over one HWC image; outputs[k] holds orc_output_len(k)
 * floats. threads <= 0 uses every core. Each output value is computed by one
 * thread in a fixed order, so any thread count gives the same bits. */
int orc_run(orc_plan *p, const float *input, float *const *outputs, int threads);

/* The timed CPU path on or off (register-tiled AVX2+FMA loops that give the
 * same bits as the plain ones); off by default. */
void orc_set_fast(int on);

/* Scalar definitions, exposed for the f64 checks. */
float orc_exp_neg(float z);
float orc_activation(int code, float x);
/* The detector's input from an 8-bit RGB image (iw x ih, pixels by rows,
 * channels together): resized to ow x oh by OpenCV's INTER_LINEAR in the
 * reference's integer staging, scaled to [0, 1] in f32 and normalized per
 * channel in f64, rounded once to f32, written channels together
 * (reference det.rs:230-292 det_input_hwc, image.rs:46-142). Returns 0, or
 * 1 for an empty size. */
int orc_det_input_hwc(const unsigned char *image, size_t iw, size_t ih, size_t ow, size_t oh, const double *mean,
                      const double *std, float *out);
/* The recogniser's input for one crop (cw x ch RGB bytes): its tensor width
 * (at least 320, the crop's aspect at height 48), and, when out is not null,
 * the crop resized to height 48 (width rounded up, cut to the tensor),
 * scaled to [-1, 1] in f32 and zero-padded on the right, channels together
 * (reference rec.rs:19-43 rec_input, ocr.rs:534-549 rec_hwc). Returns the
 * width, 0 for an empty crop. */
size_t orc_rec_input_hwc(const unsigned char *crop, size_t cw, size_t ch, float *out);

/* ---- host page steps (page_oracle.c): the reference's src/image.rs,
 * det.rs, contour.rs, geometry.rs, crop.rs, rec.rs and lib.rs restated. ---- */

/* cv2.resize INTER_LINEAR on RGB bytes (image.rs:91-142). 0 on success. */
int orc_resize_linear(const uint8_t *image, size_t iw, size_t ih, size_t ow, size_t oh, uint8_t *out);
/* np.rot90 of a w x h image (image.rs:145-155): out is h x w. */
void orc_rotate_ccw(const uint8_t *image, size_t w, size_t h, uint8_t *out);
/* det_size (det.rs:166-193): limit_min 0 for Limit::Max, else Limit::Min. */
int orc_det_size(size_t w, size_t h, size_t limit_min, size_t *ow, size_t *oh);
/* prepare_page's sizes (det.rs:44-131); 0 when there is no page. */
int orc_prepare_page(size_t w, size_t h, size_t min_side, size_t max_side, double whr, size_t min_height,
                     size_t *fw, size_t *fh, double *ratio_h, double *ratio_w, size_t *pad_top);

/* find_contours (contour.rs:44-130). */
typedef struct orc_contours orc_contours;
orc_contours *orc_find_contours(const uint8_t *mask, size_t width, size_t height);
size_t orc_contours_count(const orc_contours *c);
const int32_t *orc_contour(const orc_contours *c, size_t i, size_t *len);
void orc_contours_free(orc_contours *c);
/* contour_mean (contour.rs:142-199). */
double orc_contour_mean(const float *map, size_t width, size_t height, const int32_t *pts, size_t n);

/* min_area_rect (geometry.rs:406-457): {cx, cy, width, height, angle}. */
void orc_min_area_rect(const int32_t *pts, size_t n, float rect[5]);
/* RotatedRect::points (geometry.rs:228-240). */
void orc_box_points(const float rect[5], float quad[8]);
/* mini_box (geometry.rs:462-477): returns the shorter side. */
float orc_mini_box(const int32_t *pts, size_t n, float quad[8]);
/* unclip (geometry.rs:519-606): ring points, -1 when cap is short. */
long orc_unclip(const float quad[8], double ratio, int32_t *out, size_t cap);

/* contour_candidate (det.rs:342-372): 0 Small, 1 LowScore, 2 SmallAfterUnclip, 3 Kept. */
int orc_contour_candidate(const float *prob, size_t mw, size_t mh, const int32_t *contour, size_t n, size_t dw,
                          size_t dh, double box_thresh, double unclip_ratio, double *score, int32_t corners[8]);
/* order_and_clip (det.rs:377-396): 1 when kept. */
int orc_order_and_clip(const int32_t corners[8], size_t width, size_t height, float quad[8]);
/* sort_boxes (det.rs:407-421). */
void orc_sort_boxes(float *quads, size_t n);
/* boxes_from_prob (det.rs:430-452): the number of boxes; at most cap written. */
size_t orc_boxes_from_prob(const float *prob, size_t mw, size_t mh, size_t dw, size_t dh, float thresh,
                           double box_thresh, double unclip_ratio, size_t max_candidates, float *quads, size_t cap);

/* crop_text's size before the turn and whether it turns (crop.rs:85-86, 122). */
void orc_crop_size(const float quad[8], size_t *width, size_t *height, int *turns);
/* crop_text (crop.rs:84-127) into out (turned when tall). */
int orc_crop_text(const uint8_t *image, size_t iw, size_t ih, const float quad[8], uint8_t *out);

/* ctc_decode (rec.rs:144-161): the kept classes and the score. */
double orc_ctc_decode(const uint32_t *best, const float *prob, size_t n, uint32_t *kept, size_t *kept_n);
/* to_page (lib.rs:121-129). */
void orc_to_page(const float quad[8], double ratio_w, double ratio_h, size_t pad_top, size_t width, size_t height,
                 float out[8]);

#ifdef __cplusplus
}
#endif
#endif
