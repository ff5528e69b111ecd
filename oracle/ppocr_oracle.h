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

#ifdef __cplusplus
}
#endif
#endif
