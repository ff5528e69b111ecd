// Device arithmetic that reproduces the reference CPU engine's tier-3 bits.
//
// Every product, sum and fused multiply-add is written with a rounding
// intrinsic (__fmul_rn, __fadd_rn, __fmaf_rn), which the compiler never
// contracts or reorders, so each value goes through the same IEEE operations
// as the reference's scalar definition. The exponential is XNNPACK's
// published "p5-div" method as the reference restates it
// (`src/engine/kernels/activation.rs:7-60`), not CUDA's expf.
#pragma once

#include <cstdint>

namespace ppocr {

__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float ffma(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }

// Two independent fused multiply-adds in one instruction (sm_100's packed
// fma.rn.f32x2): each lane is rounded as __fmaf_rn rounds it, so the pair
// gives ffma's bits twice.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "mov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
        "mov.b64 {%0, %1}, rd;}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

// Rust's f32::clamp: NaN passes through.
__device__ __forceinline__ float clampf_(float v, float lo, float hi) {
    v = v < lo ? lo : v;
    return v > hi ? hi : v;
}

// exp(z) for z <= 0, 0 below the cutoff: activation.rs:37-60 with FMA.
__device__ __forceinline__ float exp_neg(float z) {
    const float bias = __uint_as_float(0x4b40007fu);
    float n = ffma(z, __uint_as_float(0x3fb8aa3bu), bias);
    float s = __uint_as_float(__float_as_uint(n) << 23);
    n = fsub(n, bias);
    float t = ffma(n, __uint_as_float(0xbf317218u), z);
    float p = ffma(__uint_as_float(0x3c07cfceu), t, __uint_as_float(0x3d2b9d0du));
    p = ffma(p, t, __uint_as_float(0x3e2aad40u));
    p = ffma(p, t, __uint_as_float(0x3efffee3u));
    p = ffma(p, t, __uint_as_float(0x3f7ffffbu));
    float e = ffma(fmul(t, s), p, s);
    return z < __uint_as_float(0xc2aeac4fu) ? 0.0f : e;
}

// A quotient: IEEE-rounded, or (QUICK) __fdividef's reciprocal and product,
// within 2 ulp, for callers whose sums already differ from the reference's
// by a few units and whose denominators lie in [1, 2^20]. QUICK forms serve
// the tensor-core epilogues only.
template <bool QUICK>
__device__ __forceinline__ float quot(float a, float b) {
    return QUICK ? __fdividef(a, b) : fdiv(a, b);
}

// activation.rs:151-159: e / (e + 1) for negative x, 1 minus it otherwise.
// QUICK: 1 / (1 + e^-x) with CUDA's __expf and __fdividef (a few ulp; 0 and
// 1 at the far ends as e^-x overflows or vanishes).
template <bool QUICK = false>
__device__ __forceinline__ float sigmoid_one(float x) {
    if (QUICK) return __fdividef(1.0f, 1.0f + __expf(-x));
    float e = exp_neg(__uint_as_float(__float_as_uint(x) | 0x80000000u));
    float f = fdiv(e, fadd(e, 1.0f));
    return (__float_as_uint(x) >> 31) ? f : fsub(1.0f, f);
}

// layers.rs:49-67: x * Phi(x) with the reference's rational fit.
template <bool QUICK = false>
__device__ __forceinline__ float gelu_one(float x) {
    float c = clampf_(x, -5.5f, 5.5f);
    float s = fmul(c, c);
    float p = __uint_as_float(0x32c36a3cu);
    p = ffma(p, s, __uint_as_float(0x36d52462u));
    p = ffma(p, s, __uint_as_float(0x39310738u));
    p = ffma(p, s, __uint_as_float(0x3b9943c9u));
    p = ffma(p, s, __uint_as_float(0x3d0aa93cu));
    p = ffma(p, s, __uint_as_float(0x3ecc4228u));
    float q = __uint_as_float(0x35a0b9e3u);
    q = ffma(q, s, __uint_as_float(0x389a737au));
    q = ffma(q, s, __uint_as_float(0x3af6ffc6u));
    q = ffma(q, s, __uint_as_float(0x3ceaaaeeu));
    q = ffma(q, s, __uint_as_float(0x3e80c788u));
    q = ffma(q, s, 1.0f);
    return fmul(x, clampf_(ffma(c, quot<QUICK>(p, q), 0.5f), 0.0f, 1.0f));
}

// The folded activation of `code` (reference conv.rs:36-72; code 7 is this
// library's hardswish, x * hardsigmoid(x)).
template <bool QUICK = false>
__device__ __forceinline__ float activate(int code, float v) {
    const float alpha = __uint_as_float(0x3e2aaaadu);  // layers.rs:42
    switch (code) {
    case 1: return clampf_(v, 0.0f, __int_as_float(0x7f800000));
    case 2: return sigmoid_one<QUICK>(v);
    case 3: return gelu_one<QUICK>(v);
    case 4: return fmul(v, sigmoid_one<QUICK>(v));
    case 5: return clampf_(fadd(fmul(v, alpha), 0.5f), 0.0f, 1.0f);
    case 6: return clampf_(fadd(fmul(v, 0.2f), 0.5f), 0.0f, 1.0f);
    case 7: return fmul(v, clampf_(fadd(fmul(v, alpha), 0.5f), 0.0f, 1.0f));
    default: return v;
    }
}

// The same with the code known at compile time, for hot epilogues.
template <int CODE, bool QUICK = false>
__device__ __forceinline__ float activate_t(float v) {
    return activate<QUICK>(CODE, v);
}

}  // namespace ppocr
