// Device helpers shared by the image kernels: OpenCV's INTER_LINEAR taps
// and blend in the reference's integer staging (ppocr-native
// src/image.rs:46-142), with correctly rounded IEEE operations so the bytes
// equal the CPU path's.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace ppocr {

struct Tap {
    int near, far, near_w, far_w;
};

// The f64 scale of a src -> dst resize, 1 / (dst / src), rounded as the
// reference rounds it (one value per axis: a kernel computes it once).
__device__ __forceinline__ double resize_scale(int src, int dst) {
    return __ddiv_rn(1.0, __ddiv_rn(double(dst), double(src)));
}

// Output coordinate d of a src -> dst resize whose scale is `scale`
// (resize_scale): source (d + 0.5) * scale - 0.5 in f64 rounded to f32,
// indices clamped to the edge, each weight rounded to 1/2048 on its own
// (ties to even).
__device__ __forceinline__ Tap resize_tap_scaled(int src, double scale, int d) {
    const float f = __double2float_rn(__dadd_rn(__dmul_rn(__dadd_rn(double(d), 0.5), scale), -0.5));
    const float fl = floorf(f);
    const float a = __fsub_rn(f, fl);
    const int s = int(fl), last = src - 1;
    Tap t;
    t.near = s < 0 ? 0 : s > last ? last : s;
    t.far = s + 1 < 0 ? 0 : s + 1 > last ? last : s + 1;
    t.near_w = __float2int_rn(__fmul_rn(__fsub_rn(1.0f, a), 2048.0f));
    t.far_w = __float2int_rn(__fmul_rn(a, 2048.0f));
    return t;
}

__device__ __forceinline__ Tap resize_tap(int src, int dst, int d) {
    return resize_tap_scaled(src, resize_scale(src, dst), d);
}

// One channel of one output byte from its two source rows (RGB bytes): the
// horizontal products kept at 1/2048, four bits of each row dropped before
// the vertical weight and sixteen after, the sum of the two rounded.
__device__ __forceinline__ int blend(const uint8_t *r0, const uint8_t *r1, const Tap &tx, const Tap &ty, int c) {
    const int p = int(r0[tx.near * 3 + c]) * tx.near_w + int(r0[tx.far * 3 + c]) * tx.far_w;
    const int q = int(r1[tx.near * 3 + c]) * tx.near_w + int(r1[tx.far * 3 + c]) * tx.far_w;
    const int v = (((p >> 4) * ty.near_w) >> 16) + (((q >> 4) * ty.far_w) >> 16);
    const int byte = (v + 2) >> 2;
    return byte < 0 ? 0 : byte > 255 ? 255 : byte;
}

}  // namespace ppocr
