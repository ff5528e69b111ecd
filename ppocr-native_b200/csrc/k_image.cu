// The detector's and the recogniser's inputs on the GPU. The detector's: an
// 8-bit RGB page image resized to the
// detector's size and normalized, written channels together as the model
// reads its input (reference det.rs:230-292 det_input_hwc, the resize of
// image.rs:46-142, which reproduces OpenCV's INTER_LINEAR).
//
// One thread per output pixel. Its two taps along each axis are computed
// the reference's way with correctly rounded IEEE operations (the source
// coordinate (d + 0.5) * src / dst - 0.5 in f64, rounded to f32, each weight
// rounded to 1/2048 on its own, ties to even), the four source pixels are
// blended with the reference's integer staging (the horizontal products
// kept at 1/2048, four bits of each row dropped before the vertical weight
// and sixteen after, the sum of the two rounded), and each byte becomes
// ((f64)(byte * (f32)(1/255)) - mean) / std rounded once to f32: the same
// bytes and bits as the CPU path.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <string>

#include "../../include/ppocr_cuda.h"
#include "image.cuh"
#include "kernels.hpp"

namespace ppocr {
void set_last_error(const std::string &msg);
}

using ppocr::Tap;

namespace {

struct ImageArgs {
    const uint8_t *image;
    float *out;
    int iw, ih, ow, oh;
    double mean[3], std[3];
};


__global__ void __launch_bounds__(256) det_input_kernel(const ImageArgs a) {
    // every output value is a function of its byte and channel alone: the
    // 3 x 256 of them, computed once per block
    __shared__ float norm[3][256];
    const float scale = __double2float_rn(__ddiv_rn(1.0, 255.0));
    for (int e = threadIdx.x; e < 3 * 256; e += blockDim.x) {
        const int c = e / 256, byte = e - c * 256;
        const float x = __fmul_rn(float(byte), scale);
        norm[c][byte] = __double2float_rn(__ddiv_rn(__dsub_rn(double(x), a.mean[c]), a.std[c]));
    }
    __syncthreads();
    const double sy = ppocr::resize_scale(a.ih, a.oh), sx = ppocr::resize_scale(a.iw, a.ow);
    const long total = long(a.ow) * a.oh;
    for (long i = long(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += long(gridDim.x) * blockDim.x) {
        const int oy = int(i / a.ow), ox = int(i - long(oy) * a.ow);
        const Tap ty = ppocr::resize_tap_scaled(a.ih, sy, oy), tx = ppocr::resize_tap_scaled(a.iw, sx, ox);
        const uint8_t *r0 = a.image + long(ty.near) * a.iw * 3, *r1 = a.image + long(ty.far) * a.iw * 3;
        float *o = a.out + i * 3;
#pragma unroll
        for (int c = 0; c < 3; c++) {
            const int p = int(r0[tx.near * 3 + c]) * tx.near_w + int(r0[tx.far * 3 + c]) * tx.far_w;
            const int q = int(r1[tx.near * 3 + c]) * tx.near_w + int(r1[tx.far * 3 + c]) * tx.far_w;
            const int v = (((p >> 4) * ty.near_w) >> 16) + (((q >> 4) * ty.far_w) >> 16);
            int byte = (v + 2) >> 2;
            byte = byte < 0 ? 0 : byte > 255 ? 255 : byte;
            o[c] = norm[c][byte];
        }
    }
}

// The recogniser's input: 48 rows x width, the crop resized to rw x 48 in
// the first rw columns, scaled to [-1, 1] as (v / 255 - 0.5) / 0.5 in f32,
// zeros after (reference rec.rs:19-43).
struct RecArgs {
    const uint8_t *crop;
    float *out;
    int cw, ch, rw, width;
};

__global__ void __launch_bounds__(256) rec_input_kernel(const RecArgs a) {
    const double sy = ppocr::resize_scale(a.ch, 48), sx = ppocr::resize_scale(a.cw, a.rw);
    const long total = long(a.width) * 48;
    for (long i = long(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += long(gridDim.x) * blockDim.x) {
        const int oy = int(i / a.width), ox = int(i - long(oy) * a.width);
        float *o = a.out + i * 3;
        if (ox >= a.rw) {
            o[0] = o[1] = o[2] = 0.0f;
            continue;
        }
        const Tap ty = ppocr::resize_tap_scaled(a.ch, sy, oy), tx = ppocr::resize_tap_scaled(a.cw, sx, ox);
        const uint8_t *r0 = a.crop + long(ty.near) * a.cw * 3, *r1 = a.crop + long(ty.far) * a.cw * 3;
#pragma unroll
        for (int c = 0; c < 3; c++) {
            const int p = int(r0[tx.near * 3 + c]) * tx.near_w + int(r0[tx.far * 3 + c]) * tx.far_w;
            const int q = int(r1[tx.near * 3 + c]) * tx.near_w + int(r1[tx.far * 3 + c]) * tx.far_w;
            const int v = (((p >> 4) * ty.near_w) >> 16) + (((q >> 4) * ty.far_w) >> 16);
            int byte = (v + 2) >> 2;
            byte = byte < 0 ? 0 : byte > 255 ? 255 : byte;
            o[c] = __fdiv_rn(__fsub_rn(__fdiv_rn(float(byte), 255.0f), 0.5f), 0.5f);
        }
    }
}

// The DB threshold: mask = prob > thresh, compared in f32 (reference
// det.rs:438), a grid-stride loop over the pixels.
__global__ void __launch_bounds__(256) db_mask_kernel(const float *prob, long n, float thresh, uint8_t *mask) {
    for (long i = long(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += long(gridDim.x) * blockDim.x)
        mask[i] = prob[i] > thresh ? 1 : 0;
}

}  // namespace

extern "C" int ppocr_db_mask(const float *prob, size_t pixels, float thresh, uint8_t *mask, void *stream) {
    if (!prob || !mask) {
        ppocr::set_last_error("ppocr_db_mask: null pointer");
        return PPOCR_E_ARG;
    }
    if (!pixels) return PPOCR_OK;
    long blocks = long((pixels + 255) / 256);
    if (blocks > 148L * 16) blocks = 148L * 16;
    db_mask_kernel<<<unsigned(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(prob, long(pixels), thresh, mask);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        ppocr::set_last_error(std::string("ppocr_db_mask: ") + cudaGetErrorString(e));
        return PPOCR_E_DEVICE;
    }
    return PPOCR_OK;
}

extern "C" int ppocr_rec_input_hwc(const uint8_t *crop, size_t width, size_t height, float *out, size_t capacity,
                                   size_t *tensor_width, void *stream) {
    if (!tensor_width || (out && !crop)) {
        ppocr::set_last_error("ppocr_rec_input_hwc: null pointer");
        return PPOCR_E_ARG;
    }
    if (!width || !height || width > (1u << 20) || height > (1u << 20)) {
        ppocr::set_last_error("ppocr_rec_input_hwc: crop sizes must be between 1 and 2^20");
        return PPOCR_E_SIZE;
    }
    // rec.rs:20-31: the tensor width truncates, the resized width rounds up
    // and is cut to the tensor
    const double h = double(height), w = double(width), rows = 48.0;
    const double ratio = 320.0 / rows > w / h ? 320.0 / rows : w / h;
    const size_t tw = size_t(rows * ratio);
    const double fitted = std::ceil(rows * (w / h));
    const size_t rw = fitted > double(tw) ? tw : size_t(fitted);
    *tensor_width = tw;
    if (!out) return PPOCR_OK;
    if (tw > (1u << 22) || capacity < 48 * tw * 3) {
        ppocr::set_last_error("ppocr_rec_input_hwc: out holds fewer than 48 x width x 3 floats");
        return PPOCR_E_SIZE;
    }
    RecArgs a;
    a.crop = crop;
    a.out = out;
    a.cw = int(width); a.ch = int(height); a.rw = int(rw); a.width = int(tw);
    const long total = long(tw) * 48;
    long blocks = (total + 255) / 256;
    if (blocks > 148L * 16) blocks = 148L * 16;
    rec_input_kernel<<<unsigned(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        ppocr::set_last_error(std::string("ppocr_rec_input_hwc: ") + cudaGetErrorString(e));
        return PPOCR_E_DEVICE;
    }
    return PPOCR_OK;
}

extern "C" int ppocr_det_input_hwc(const uint8_t *image, size_t width, size_t height, size_t out_width,
                                   size_t out_height, const double *mean, const double *std, float *out,
                                   size_t capacity, void *stream) {
    if (!image || !out || !mean || !std) {
        ppocr::set_last_error("ppocr_det_input_hwc: null pointer");
        return PPOCR_E_ARG;
    }
    if (!width || !height || !out_width || !out_height || width > (1u << 20) || height > (1u << 20) ||
        out_width > (1u << 20) || out_height > (1u << 20)) {
        ppocr::set_last_error("ppocr_det_input_hwc: sizes must be between 1 and 2^20");
        return PPOCR_E_SIZE;
    }
    if (capacity / 3 / out_width < out_height) {
        ppocr::set_last_error("ppocr_det_input_hwc: out holds fewer than out_height x out_width x 3 floats");
        return PPOCR_E_SIZE;
    }
    ImageArgs a;
    a.image = image;
    a.out = out;
    a.iw = int(width); a.ih = int(height); a.ow = int(out_width); a.oh = int(out_height);
    for (int c = 0; c < 3; c++) {
        a.mean[c] = mean[c];
        a.std[c] = std[c];
    }
    const long total = long(out_width) * long(out_height);
    long blocks = (total + 255) / 256;
    if (blocks > 148L * 16) blocks = 148L * 16;
    det_input_kernel<<<unsigned(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        ppocr::set_last_error(std::string("ppocr_det_input_hwc: ") + cudaGetErrorString(e));
        return PPOCR_E_DEVICE;
    }
    return PPOCR_OK;
}
