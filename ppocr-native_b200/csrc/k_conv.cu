// Dense convolution as an implicit GEMM on the FP32 pipes (sm_100a).
//
// GEMM view: M = output pixels of all lanes, Nc = oc output channels,
// K = kh*kw*C with k = (ky*kw + kx)*C + c, the order of the weights
// `[kh][kw][C][oc]` and of the reference's sums (`kernels/dense.rs:20-36`).
// A block owns a BM x BN output tile; its threads hold TM x TN accumulators
// each. K advances one (tap, BK-channel slice) tile at a time through
// double-buffered shared memory, the next tile prefetched into registers
// while the current one is multiplied. Every accumulator adds its k terms in
// increasing k with one fused multiply-add each, starting from the bias or
// from zero as the reference's tiles do, so each output carries the
// reference's bits.
//
// The A tile is gathered on the fly: a padded tap reads zero, and each of up
// to four sources is read nearest-upsampled by 2^shift in place, so the
// neck's upsample + concat never reach memory. A pointwise layer (1x1, unit
// stride, no padding, one source) reads A straight from its input, whose
// pixels are the output's. An SE gate (per lane and input channel)
// multiplies A as it is loaded; a residual add and a second activation run in
// the epilogue.
#include <algorithm>

#include "devmath.cuh"
#include "kernels.hpp"

namespace ppocr {

namespace {

constexpr int APAD = 4;

template <int TM, int TN, int TX, int TY, int BK>
struct Cfg {
    static constexpr int BM = TM * TY, BN = TN * TX, THREADS = TX * TY;
    static constexpr int AGROUPS = BM * BK / 4;  // float4 groups of the A tile
    static constexpr int ALOADS = (AGROUPS + THREADS - 1) / THREADS;
    static constexpr int BGROUPS = BK * BN / 4;  // float4 groups of the B tile (BN % 4 == 0)
    static constexpr int BLOADS = (BGROUPS + THREADS - 1) / THREADS;
    static constexpr size_t SMEM = sizeof(float) * (2 * BK * (BM + APAD) + 2 * BK * BN);
};

// One A-load slot, fixed for the whole K loop: its lane, the lane's input
// size and the top-left input tap (windowed), or its pixel (pointwise). The
// block keeps one per tile pixel in shared memory (`meta`) rather than each
// thread in registers.
struct Pixel {
    long m;
    int n, iy0, ix0, ih, iw;
    bool ok;
};

// Shared form of a Pixel: {lane, iy0, ix0, ih << 16 | iw}; ih 0 marks a
// pixel past the end.
__device__ __forceinline__ Pixel unpack(int4 md, long m) {
    Pixel p;
    p.m = m;
    p.n = md.x;
    p.iy0 = md.y;
    p.ix0 = md.z;
    p.ih = md.w >> 16;
    p.iw = md.w & 0xffff;
    p.ok = p.ih != 0;
    return p;
}

// Four channels c..c+3 of A for one slot at tap (ky, kx).
template <bool PW>
__device__ __forceinline__ void load_a_group(const ConvArgs &a, const Pixel &px, int ky, int kx, int c, bool vec4,
                                             float v[4]) {
    v[0] = v[1] = v[2] = v[3] = 0.0f;
    if (!px.ok) return;
    if (PW) {
        // pointwise: the input pixel is the output pixel, one source
        if (vec4) {
            if (c >= a.C) return;
            float4 q = __ldg(reinterpret_cast<const float4 *>(a.src[0].p + px.m * a.C + c));
            v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
        } else {
#pragma unroll
            for (int e = 0; e < 4; e++)
                if (c + e < a.C) v[e] = __ldg(a.src[0].p + px.m * a.C + c + e);
        }
        if (a.gate) {
            const float *g = a.gate + (long)px.n * a.C + c;
#pragma unroll
            for (int e = 0; e < 4; e++)
                if (c + e < a.C) v[e] = fmul(v[e], __ldg(g + e));
        }
        return;
    }
    int iy = px.iy0 + ky, ix = px.ix0 + kx;
    if (iy < 0 || iy >= px.ih || ix < 0 || ix >= px.iw) return;
    const LaneInfo &L = a.lanes[px.n];
    if (vec4) {
        // All four channels lie in one source (every source has c % 4 == 0).
        if (c >= a.C) return;
        int start = 0, s = 0;
        while (s + 1 < a.nsrc && c >= start + a.src[s].c) { start += a.src[s].c; s++; }
        const ConvSource &src = a.src[s];
        int sh = src.shift;
        int ws = px.iw >> sh;
        long off = (__ldg(&L.spix0[s]) + (long)(iy >> sh) * ws + (ix >> sh)) * src.c + (c - start);
        float4 q = __ldg(reinterpret_cast<const float4 *>(src.p + off));
        v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
        if (a.gate) {
            const float *g = a.gate + (long)px.n * a.C + c;
            v[0] = fmul(v[0], g[0]); v[1] = fmul(v[1], g[1]);
            v[2] = fmul(v[2], g[2]); v[3] = fmul(v[3], g[3]);
        }
        return;
    }
#pragma unroll
    for (int e = 0; e < 4; e++) {
        int ce = c + e;
        if (ce >= a.C) break;
        int start = 0, s = 0;
        while (s + 1 < a.nsrc && ce >= start + a.src[s].c) { start += a.src[s].c; s++; }
        const ConvSource &src = a.src[s];
        int sh = src.shift;
        int ws = px.iw >> sh;
        long off = (__ldg(&L.spix0[s]) + (long)(iy >> sh) * ws + (ix >> sh)) * src.c + (ce - start);
        float x = __ldg(src.p + off);
        if (a.gate) x = fmul(x, a.gate[(long)px.n * a.C + ce]);
        v[e] = x;
    }
}

// At most 128 registers a thread, so that two 256-thread (or four
// 128-thread) blocks share an SM.
template <int TM, int TN, int TX, int TY, int BK, bool PW>
__global__ void __launch_bounds__(TX *TY, 65536 / (TX * TY * 128)) conv_gemm(const ConvArgs a, int ctiles, int ntiles_k, bool vec4,
                                                    bool bvec4) {
    using C = Cfg<TM, TN, TX, TY, BK>;
    constexpr int BM = C::BM, BN = C::BN;
    extern __shared__ __align__(16) float smem[];
    float *As = smem;                          // [2][BK][BM + APAD]
    float *Bs = smem + 2 * BK * (BM + APAD);   // [2][BK][BN]
    __shared__ int4 meta[BM];

    const int tid = threadIdx.x;
    const int tx = tid % TX, ty = tid / TX;
    const long M = a.M;
    const long m0 = (long)blockIdx.x * BM;
    const int n0 = blockIdx.y * BN;

    // Where each pixel of the tile reads, once per block.
    for (int p = tid; p < BM; p += C::THREADS) {
        long m = m0 + p;
        int4 md = make_int4(0, 0, 0, 0);
        if (m < M) {
            md.w = 1 << 16;  // in range (pointwise reads need no more)
            if (!PW || a.gate) {
                int n = find_lane(a.lanes, a.nl, m);
                md.x = n;
                if (!PW) {
                    const LaneInfo &L = a.lanes[n];
                    int ow = __ldg(&L.ow);
                    int r = int(m - __ldg(&L.pix0));
                    int oy = r / ow, ox = r - oy * ow;
                    md.y = oy * a.sh - a.pt;
                    md.z = ox * a.sw - a.pl;
                    md.w = (__ldg(&L.ih) << 16) | __ldg(&L.iw);
                }
            }
        }
        meta[p] = md;
    }
    __syncthreads();

    float ra[C::ALOADS][4];
    float4 rb[C::BLOADS];

    auto fetch = [&](int t) {
        int tap = PW ? 0 : t / ctiles;
        int c0 = (t - tap * ctiles) * BK;
        int ky = PW ? 0 : tap / a.kw;
        int kx = PW ? 0 : tap - ky * a.kw;
#pragma unroll
        for (int l = 0; l < C::ALOADS; l++) {
            int g = tid + l * C::THREADS;
            int am = g / (BK / 4), aq = g % (BK / 4);
            if (g < C::AGROUPS) {
                Pixel px = unpack(meta[am], m0 + am);
                load_a_group<PW>(a, px, ky, kx, c0 + aq * 4, vec4, ra[l]);
            }
        }
#pragma unroll
        for (int l = 0; l < C::BLOADS; l++) {
            int g = tid + l * C::THREADS;
            int kk = (g * 4) / BN, nn = (g * 4) - kk * BN;
            int c = c0 + kk, n = n0 + nn;
            float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
            if (g < C::BGROUPS && c < a.C) {
                const float *src = a.w + ((long)tap * a.C + c) * a.oc + n;
                if (bvec4 && n + 3 < a.oc) {
                    q = __ldg(reinterpret_cast<const float4 *>(src));
                } else {
                    if (n < a.oc) q.x = __ldg(src);
                    if (n + 1 < a.oc) q.y = __ldg(src + 1);
                    if (n + 2 < a.oc) q.z = __ldg(src + 2);
                    if (n + 3 < a.oc) q.w = __ldg(src + 3);
                }
            }
            rb[l] = q;
        }
    };
    auto stash = [&](int buf) {
        float *Ab = As + buf * BK * (BM + APAD);
        float *Bb = Bs + buf * BK * BN;
#pragma unroll
        for (int l = 0; l < C::ALOADS; l++) {
            int g = tid + l * C::THREADS;
            int am = g / (BK / 4), aq = g % (BK / 4);
            if (g < C::AGROUPS) {
#pragma unroll
                for (int e = 0; e < 4; e++) Ab[(aq * 4 + e) * (BM + APAD) + am] = ra[l][e];
            }
        }
#pragma unroll
        for (int l = 0; l < C::BLOADS; l++) {
            int g = tid + l * C::THREADS;
            if (g < C::BGROUPS) *reinterpret_cast<float4 *>(Bb + g * 4) = rb[l];
        }
    };

    // Accumulators, seeded with the bias where the reference takes it first.
    float acc[TM][TN];
    bool first[TM];
#pragma unroll
    for (int i = 0; i < TM; i++) {
        long m = m0 + ty * TM + i;
        bool f = a.bias_mode == BIAS_FIRST;
        if (a.bias_mode == BIAS_FIRST_BUT_ROW_TAIL && m < M) {
            const LaneInfo &L = a.lanes[find_lane(a.lanes, a.nl, m)];
            int ow = __ldg(&L.ow);
            int ox = int((m - __ldg(&L.pix0)) % ow);
            f = ox < ow - ow % 4;
        }
        first[i] = f;
#pragma unroll
        for (int j = 0; j < TN; j++) {
            int n = n0 + tx * TN + j;
            acc[i][j] = (f && a.b && n < a.oc) ? __ldg(a.b + n) : 0.0f;
        }
    }

    fetch(0);
    stash(0);
    __syncthreads();
    for (int t = 0; t < ntiles_k; t++) {
        const int buf = t & 1;
        if (t + 1 < ntiles_k) fetch(t + 1);
        const float *Ab = As + buf * BK * (BM + APAD) + ty * TM;
        const float *Bb = Bs + buf * BK * BN + tx * TN;
#pragma unroll
        for (int kk = 0; kk < BK; kk++) {
            float fa[TM], fb[TN];
#pragma unroll
            for (int i = 0; i < TM; i += 4) {
                float4 q = *reinterpret_cast<const float4 *>(Ab + kk * (BM + APAD) + i);
                fa[i] = q.x; fa[i + 1] = q.y; fa[i + 2] = q.z; fa[i + 3] = q.w;
            }
            if (TN % 4 == 0) {
#pragma unroll
                for (int j = 0; j < TN; j += 4) {
                    float4 q = *reinterpret_cast<const float4 *>(Bb + kk * BN + j);
                    fb[j] = q.x; fb[j + 1] = q.y; fb[j + 2] = q.z; fb[j + 3] = q.w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < TN; j += 2) {
                    float2 q = *reinterpret_cast<const float2 *>(Bb + kk * BN + j);
                    fb[j] = q.x; fb[j + 1] = q.y;
                }
            }
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < TN; j++) acc[i][j] = ffma(fb[j], fa[i], acc[i][j]);
        }
        if (t + 1 < ntiles_k) stash(buf ^ 1);
        __syncthreads();
    }

    // Epilogue: bias last where due, activation, residual, second activation.
#pragma unroll
    for (int i = 0; i < TM; i++) {
        long m = m0 + ty * TM + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < TN; j++) {
            int n = n0 + tx * TN + j;
            if (n >= a.oc) continue;
            float v = acc[i][j];
            if (!first[i] && a.b) v = fadd(v, __ldg(a.b + n));
            v = activate(a.act, v);
            if (a.res) v = activate(a.act2, fadd(v, __ldg(a.res + m * a.oc + n)));
            a.y[m * a.oc + n] = v;
        }
    }
}

// A pointwise layer over per-lane vectors (a squeeze-and-excite branch: one
// pixel per lane). Block (b, r) takes output channels 32b..32b+31 of pixels
// 8r..8r+7, one thread each: its threads first copy that weight slice and
// those (gated) input vectors to shared memory together, many loads in
// flight; then each output is one thread's chain of k terms added in
// increasing k with one fused multiply-add each, from the bias or from zero,
// as conv_gemm's accumulators do, so the two give the same bits.
constexpr int VEC_COLS = 32, VEC_ROWS = 8;

__global__ void __launch_bounds__(VEC_COLS *VEC_ROWS) conv_vector_kernel(const ConvArgs a) {
    extern __shared__ float vsm[];
    float *ws = vsm;                   // [C][32]
    float *xs = vsm + a.C * VEC_COLS;  // [8][C]
    const int n0 = blockIdx.x * VEC_COLS;
    const long m0 = (long)blockIdx.y * VEC_ROWS;
    const int cols = min(VEC_COLS, a.oc - n0);
    const int rows = int(min((long)VEC_ROWS, a.M - m0));
    // staged eight loads at a time, so that their latencies overlap
    constexpr int BATCH = 8;
    const int wn = a.C * VEC_COLS;
    for (int e0 = threadIdx.x; e0 < wn; e0 += BATCH * blockDim.x) {
        float v[BATCH];
#pragma unroll
        for (int u = 0; u < BATCH; u++) {
            const int e = e0 + u * blockDim.x, k = e / VEC_COLS, j = e - k * VEC_COLS;
            v[u] = (e < wn && j < cols) ? __ldg(a.w + (long)k * a.oc + n0 + j) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < BATCH; u++)
            if (e0 + u * blockDim.x < wn) ws[e0 + u * blockDim.x] = v[u];
    }
    const int xn = rows * a.C;
    for (int e0 = threadIdx.x; e0 < xn; e0 += BATCH * blockDim.x) {
        float v[BATCH];
#pragma unroll
        for (int u = 0; u < BATCH; u++) {
            const int e = e0 + u * blockDim.x, r = e / a.C, k = e - r * a.C;
            v[u] = 0.0f;
            if (e < xn) {
                v[u] = __ldg(a.src[0].p + (m0 + r) * a.C + k);
                if (a.gate) v[u] = fmul(v[u], __ldg(a.gate + (long)find_lane(a.lanes, a.nl, m0 + r) * a.C + k));
            }
        }
#pragma unroll
        for (int u = 0; u < BATCH; u++)
            if (e0 + u * blockDim.x < xn) xs[e0 + u * blockDim.x] = v[u];
    }
    __syncthreads();
    const int r = threadIdx.x / VEC_COLS, j = threadIdx.x % VEC_COLS;
    if (r >= rows || j >= cols) return;
    const long m = m0 + r;
    const int n = n0 + j;
    const bool first = a.bias_mode == BIAS_FIRST;
    float acc = (first && a.b) ? __ldg(a.b + n) : 0.0f;
    const float *xm = xs + r * a.C;
#pragma unroll 8
    for (int k = 0; k < a.C; k++) acc = ffma(ws[k * VEC_COLS + j], xm[k], acc);
    if (!first && a.b) acc = fadd(acc, __ldg(a.b + n));
    acc = activate(a.act, acc);
    if (a.res) acc = activate(a.act2, fadd(acc, __ldg(a.res + m * a.oc + n)));
    a.y[m * a.oc + n] = acc;
}

// A stem pixel's NB outputs, activated and stored four at a time.
template <int NB, bool QUICK>
__device__ __forceinline__ void stem_store(int act, const float acc[NB], float *y) {
#pragma unroll
    for (int j = 0; j < NB; j += 4)
        *reinterpret_cast<float4 *>(y + j) =
            make_float4(activate<QUICK>(act, acc[j]), activate<QUICK>(act, acc[j + 1]),
                        activate<QUICK>(act, acc[j + 2]), activate<QUICK>(act, acc[j + 3]));
}

// An RGB stem (three input channels, bias first, kh * kw <= 9): one thread
// per output pixel holds its kh*kw*3 input values and all NB outputs; the
// weights sit in shared memory, read by every thread at once (broadcast).
// Each output adds its k terms in increasing k = (ky*kw + kx)*3 + c with one
// fused multiply-add each, padded taps as zeros, from the bias, as
// conv_gemm's accumulators do, so the two give the same bits.
template <int NB>
__global__ void __launch_bounds__(128) stem_kernel(const ConvArgs a) {
    __shared__ __align__(16) float ws[27 * NB];
    __shared__ float bs[NB];
    const int K = a.kh * a.kw * 3;
    for (int e = threadIdx.x; e < K * NB; e += blockDim.x) ws[e] = __ldg(a.w + e);
    for (int e = threadIdx.x; e < NB; e += blockDim.x) bs[e] = a.b ? __ldg(a.b + e) : 0.0f;
    __syncthreads();
    const float *x = a.src[0].p;
    for (long m = (long)blockIdx.x * blockDim.x + threadIdx.x; m < a.M; m += (long)gridDim.x * blockDim.x) {
        const int n = find_lane(a.lanes, a.nl, m);
        const LaneInfo &L = a.lanes[n];
        const int ow = __ldg(&L.ow), ih = __ldg(&L.ih), iw = __ldg(&L.iw);
        const int q = int(m - __ldg(&L.pix0));
        const int oy = q / ow, ox = q - oy * ow;
        const int iy0 = oy * a.sh - a.pt, ix0 = ox * a.sw - a.pl;
        const float *xl = x + __ldg(&L.ipix0) * 3;
        float in[27];  // taps past kh x kw stay zero and are never used
#pragma unroll
        for (int t = 0; t < 9; t++) {
            const bool tap = t < a.kh * a.kw;
            const int ty = tap ? t / a.kw : 0;
            const int iy = iy0 + ty, ix = ix0 + (tap ? t - ty * a.kw : 0);
            const bool ok = tap && iy >= 0 && iy < ih && ix >= 0 && ix < iw;
            const float *p = xl + ((long)iy * iw + ix) * 3;
            in[3 * t] = ok ? __ldg(p) : 0.0f;
            in[3 * t + 1] = ok ? __ldg(p + 1) : 0.0f;
            in[3 * t + 2] = ok ? __ldg(p + 2) : 0.0f;
        }
        float acc[NB];
#pragma unroll
        for (int j = 0; j < NB; j++) acc[j] = bs[j];
#pragma unroll
        for (int k = 0; k < 27; k++) {
            if (k >= K) break;
#pragma unroll
            for (int j = 0; j < NB; j += 4) {
                const float4 w4 = *reinterpret_cast<const float4 *>(ws + k * NB + j);  // broadcast
                acc[j] = ffma(w4.x, in[k], acc[j]);
                acc[j + 1] = ffma(w4.y, in[k], acc[j + 1]);
                acc[j + 2] = ffma(w4.z, in[k], acc[j + 2]);
                acc[j + 3] = ffma(w4.w, in[k], acc[j + 3]);
            }
        }
        float *y = a.y + m * NB;
        if (a.quick)
            stem_store<NB, true>(a.act, acc, y);
        else
            stem_store<NB, false>(a.act, acc, y);
    }
}

// A 3x3 stride-2 RGB stem by row segments: a block computes STEM_SEG
// consecutive outputs of one output row (grid y: the row over all lanes,
// grid x: the segment). The three input rows under the segment are staged
// in shared memory with coalesced loads (zeros outside the image; each row
// padded to a multiple of four floats, so that a pixel's nine values of a
// kernel row read as four 8-byte loads and one 4-byte load, conflict free),
// each thread computes STEM_CH channels of one or two pixels (stem_px; bias
// first, then the 27 terms in increasing k = (ky * 3 + kx) * 3 + c, padded
// taps as zeros: the same bits as stem_kernel; the channel pairs go through
// packed FMAs), and the segment's
// outputs, contiguous in the packed output, leave through shared memory as
// coalesced 16-byte stores.
constexpr int STEM_SEG = 128;
constexpr int STEM_CH = 12;  // channels per thread
// Pixels per thread: two for the 48-channel stem (a weight float4 then
// serves both), one for the 24-channel one (which measured faster with 256
// threads a block than with 128); 256 threads either way.
__host__ __device__ constexpr int stem_px(int nb) { return nb >= 48 ? 2 : 1; }
__host__ __device__ constexpr int stem_threads(int nb) { return STEM_SEG / stem_px(nb) * (nb / STEM_CH); }

template <int N, int ACT, bool QUICK>
__device__ __forceinline__ void stem_activate(const float acc[N], float *out) {
#pragma unroll
    for (int j = 0; j < N; j += 4)
        *reinterpret_cast<float4 *>(out + j) =
            make_float4(activate_t<ACT, QUICK>(acc[j]), activate_t<ACT, QUICK>(acc[j + 1]),
                        activate_t<ACT, QUICK>(acc[j + 2]), activate_t<ACT, QUICK>(acc[j + 3]));
}

template <int NB, bool QUICK>
__global__ void __launch_bounds__(256) stem_rows_kernel(const ConvArgs a) {
    static_assert(NB % STEM_CH == 0, "whole channel groups");
    constexpr int PX = stem_px(NB), THREADS = stem_threads(NB);
    constexpr int SPAN = 2 * STEM_SEG + 1;        // staged input columns
    constexpr int RF = 3 * SPAN;                  // floats of one staged row
    constexpr int RS = (RF + 3) / 4 * 4;          // padded row stride
    constexpr int OS = NB + 4;                    // padded smem output row (conflict-free 16-byte stores)
    __shared__ __align__(16) float ws[27 * NB];
    __shared__ float bs[NB];
    __shared__ __align__(16) float xin[3 * RS];
    __shared__ __align__(16) float yout[STEM_SEG * OS];
    const int tid = threadIdx.x;
    const LaneInfo &L = a.lanes[find_row_lane(a.lanes, a.nl, blockIdx.y)];
    const int ow = __ldg(&L.ow), ih = __ldg(&L.ih), iw = __ldg(&L.iw);
    const int oy = int(blockIdx.y - __ldg(&L.row0));
    const int ox0 = int(blockIdx.x) * STEM_SEG;
    if (ox0 >= ow) return;  // a narrower lane's row
    const int cnt = ow - ox0 < STEM_SEG ? ow - ox0 : STEM_SEG;
    for (int e = tid; e < 27 * NB; e += THREADS) ws[e] = __ldg(a.w + e);
    for (int e = tid; e < NB; e += THREADS) bs[e] = a.b ? __ldg(a.b + e) : 0.0f;
    const float *xl = a.src[0].p + __ldg(&L.ipix0) * 3;
    const int iy0 = oy * 2 - a.pt, ix0 = ox0 * 2 - a.pl;
    // each staged row is one run of RF floats of the input row (zeros
    // outside the image): all of a thread's loads in flight at once
    constexpr int PER = (RF + THREADS - 1) / THREADS;
    const int lo = (ix0 < 0 ? -ix0 : 0) * 3, hi = (iw - ix0 < SPAN ? iw - ix0 : SPAN) * 3;
    float v[3][PER];
#pragma unroll
    for (int r = 0; r < 3; r++) {
        const bool row_ok = (unsigned)(iy0 + r) < (unsigned)ih;
        const float *src = xl + ((long)(iy0 + r) * iw + ix0) * 3;
#pragma unroll
        for (int u = 0; u < PER; u++) {
            const int j = tid + u * THREADS;
            v[r][u] = (row_ok && j >= lo && j < hi) ? __ldg(src + j) : 0.0f;
        }
    }
#pragma unroll
    for (int r = 0; r < 3; r++)
#pragma unroll
        for (int u = 0; u < PER; u++) {
            const int j = tid + u * THREADS;
            if (j < RS) xin[r * RS + j] = j < RF ? v[r][u] : 0.0f;
        }
    __syncthreads();
    constexpr int GAP = STEM_SEG / PX;  // a thread's pixels: q, q + GAP, ...
    const int q = tid % GAP, g = tid / GAP;
    if (q < cnt) {
        float acc[PX][STEM_CH];
#pragma unroll
        for (int i = 0; i < PX; i++)
#pragma unroll
            for (int j = 0; j < STEM_CH; j++) acc[i][j] = bs[g * STEM_CH + j];
#pragma unroll
        for (int ky = 0; ky < 3; ky++) {
            // the nine values (kx, c) of kernel row ky under each pixel
            float in[PX][9];
#pragma unroll
            for (int i = 0; i < PX; i++) {
                const float *r = xin + ky * RS + 6 * (q + i * GAP);
#pragma unroll
                for (int e = 0; e < 8; e += 2) {
                    const float2 t = *reinterpret_cast<const float2 *>(r + e);
                    in[i][e] = t.x;
                    in[i][e + 1] = t.y;
                }
                in[i][8] = r[8];
            }
#pragma unroll
            for (int t = 0; t < 9; t++) {
                const int k = ky * 9 + t;
#pragma unroll
                for (int j = 0; j < STEM_CH; j += 4) {
                    const float4 w4 = *reinterpret_cast<const float4 *>(ws + k * NB + g * STEM_CH + j);  // broadcast
                    const float2 wa = make_float2(w4.x, w4.y), wb = make_float2(w4.z, w4.w);
#pragma unroll
                    for (int i = 0; i < PX; i++) {
                        const float2 xv = make_float2(in[i][t], in[i][t]);
                        float2 r = ffma2(wa, xv, make_float2(acc[i][j], acc[i][j + 1]));
                        acc[i][j] = r.x;
                        acc[i][j + 1] = r.y;
                        r = ffma2(wb, xv, make_float2(acc[i][j + 2], acc[i][j + 3]));
                        acc[i][j + 2] = r.x;
                        acc[i][j + 3] = r.y;
                    }
                }
            }
        }
        // one branch on the activation per thread, not per value
#pragma unroll
        for (int i = 0; i < PX; i++) {
            if (q + i * GAP >= cnt) break;
            float *out = yout + (q + i * GAP) * OS + g * STEM_CH;
            switch (a.act) {
            case 1: stem_activate<STEM_CH, 1, QUICK>(acc[i], out); break;
            case 2: stem_activate<STEM_CH, 2, QUICK>(acc[i], out); break;
            case 3: stem_activate<STEM_CH, 3, QUICK>(acc[i], out); break;
            case 4: stem_activate<STEM_CH, 4, QUICK>(acc[i], out); break;
            case 5: stem_activate<STEM_CH, 5, QUICK>(acc[i], out); break;
            case 6: stem_activate<STEM_CH, 6, QUICK>(acc[i], out); break;
            case 7: stem_activate<STEM_CH, 7, QUICK>(acc[i], out); break;
            default: stem_activate<STEM_CH, 0, QUICK>(acc[i], out); break;
            }
        }
    }
    __syncthreads();
    float *dst = a.y + (__ldg(&L.pix0) + (long)oy * ow + ox0) * NB;
    for (int e = tid; e < cnt * (NB / 4); e += THREADS) {
        const int px = e / (NB / 4), c4 = e - px * (NB / 4);
        reinterpret_cast<float4 *>(dst)[e] = *reinterpret_cast<const float4 *>(yout + px * OS + 4 * c4);
    }
}

template <int NB>
void run_stem_rows(const ConvArgs &a, cudaStream_t s) {
    const dim3 grid(unsigned((a.max_ow + STEM_SEG - 1) / STEM_SEG), unsigned(a.out_rows));
    constexpr int THREADS = stem_threads(NB);
    if (a.quick)
        stem_rows_kernel<NB, true><<<grid, THREADS, 0, s>>>(a);
    else
        stem_rows_kernel<NB, false><<<grid, THREADS, 0, s>>>(a);
}

template <int TM, int TN, int TX, int TY, int BK>
int run(const ConvArgs &a, cudaStream_t s, bool vec4, bool pw) {
    using C = Cfg<TM, TN, TX, TY, BK>;
    static_assert(TM % 4 == 0 && TN % 2 == 0 && C::BN % 4 == 0 && BK % 4 == 0, "tile shape");
    int ctiles = (a.C + BK - 1) / BK;
    int taps = a.kh * a.kw;
    dim3 grid((unsigned)((a.M + C::BM - 1) / C::BM), (unsigned)((a.oc + C::BN - 1) / C::BN));
    bool bvec4 = a.oc % 4 == 0;
    if (pw)
        conv_gemm<TM, TN, TX, TY, BK, true><<<grid, C::THREADS, C::SMEM, s>>>(a, ctiles, ctiles, vec4, bvec4);
    else
        conv_gemm<TM, TN, TX, TY, BK, false><<<grid, C::THREADS, C::SMEM, s>>>(a, ctiles, taps * ctiles, vec4, bvec4);
    return 1;
}

template <int TM, int TN, int TX, int TY, int BK>
void allow() {
    using C = Cfg<TM, TN, TX, TY, BK>;
    cudaFuncSetAttribute(conv_gemm<TM, TN, TX, TY, BK, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         int(C::SMEM));
    cudaFuncSetAttribute(conv_gemm<TM, TN, TX, TY, BK, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         int(C::SMEM));
}

// Output pixels under which a layer is short of blocks for 148 SMs: it then
// takes the tile with fewer pixels per block.
constexpr long SMALL_M = 148L * 2 * 128;

}  // namespace

void configure_conv_kernels() {
    cudaFuncSetAttribute(conv_vector_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    allow<8, 8, 16, 16, 8>();
    allow<4, 8, 16, 16, 16>();
    allow<8, 6, 16, 16, 8>();
    allow<4, 6, 16, 16, 16>();
    allow<8, 4, 16, 16, 8>();
    allow<8, 6, 8, 32, 8>();
    allow<4, 6, 8, 32, 16>();
    allow<8, 6, 4, 32, 8>();
    allow<4, 6, 4, 32, 16>();
    allow<4, 4, 4, 64, 16>();
    allow<4, 2, 4, 64, 16>();
    allow<4, 4, 8, 32, 16>();
    allow<8, 6, 4, 32, 4>();
    allow<8, 6, 8, 32, 4>();
}

// Tile per output width: the widest per-thread tiles (8 pixels) on layers
// with enough pixels to fill the SMs, 4 pixels per thread on smaller ones;
// K slices of 8 channels for the wide tiles, 16 for the narrow ones, which
// keeps every variant near or under 128 registers.
int launch_conv(const ConvArgs &a, cudaStream_t s) {
    bool vec4 = true;
    for (int i = 0; i < a.nsrc; i++) vec4 = vec4 && (a.src[i].c % 4 == 0);
    bool pw = a.kh == 1 && a.kw == 1 && a.sh == 1 && a.sw == 1 && a.pt == 0 && a.pl == 0 && a.nsrc == 1 &&
              a.src[0].shift == 0;
    bool small = a.M < SMALL_M;
    int oc = a.oc;
    // RGB stems (bias first): the direct kernel
    if (a.C == 3 && a.nsrc == 1 && !a.src[0].shift && a.bias_mode == BIAS_FIRST && !a.gate && !a.res &&
        a.kh * a.kw <= 9 && (oc == 24 || oc == 48)) {
        if (a.kh == 3 && a.kw == 3 && a.sh == 2 && a.sw == 2 && a.out_rows > 0 && a.out_rows < 65536 && a.max_ow > 0) {
            oc == 24 ? run_stem_rows<24>(a, s) : run_stem_rows<48>(a, s);
            return 1;
        }
        const long blocks = std::min<long>((a.M + 127) / 128, 148L * 16);
        if (oc == 24)
            stem_kernel<24><<<unsigned(blocks), 128, 0, s>>>(a);
        else
            stem_kernel<48><<<unsigned(blocks), 128, 0, s>>>(a);
        return 1;
    }
    // other three- or four-channel inputs: K slices of 4
    if (a.C <= 4 && oc == 24) return run<8, 6, 4, 32, 4>(a, s, vec4, pw);
    if (a.C <= 4 && oc == 48) return run<8, 6, 8, 32, 4>(a, s, vec4, pw);
    if (oc % 128 == 0) return small ? run<4, 8, 16, 16, 16>(a, s, vec4, pw) : run<8, 8, 16, 16, 8>(a, s, vec4, pw);
    if (oc % 96 == 0) return small ? run<4, 6, 16, 16, 16>(a, s, vec4, pw) : run<8, 6, 16, 16, 8>(a, s, vec4, pw);
    if (oc % 64 == 0) return run<8, 4, 16, 16, 8>(a, s, vec4, pw);
    if (oc % 48 == 0) return small ? run<4, 6, 8, 32, 16>(a, s, vec4, pw) : run<8, 6, 8, 32, 8>(a, s, vec4, pw);
    if (oc % 24 == 0) return small ? run<4, 6, 4, 32, 16>(a, s, vec4, pw) : run<8, 6, 4, 32, 8>(a, s, vec4, pw);
    if (oc <= 8) return run<4, 2, 4, 64, 16>(a, s, vec4, pw);
    if (oc <= 16) return run<4, 4, 4, 64, 16>(a, s, vec4, pw);
    if (oc <= 32) return run<4, 4, 8, 32, 16>(a, s, vec4, pw);
    return run<8, 4, 16, 16, 8>(a, s, vec4, pw);
}

size_t conv_vector_smem(const ConvArgs &a) { return sizeof(float) * size_t(a.C) * (VEC_COLS + VEC_ROWS); }

bool conv_vector_supported(const ConvArgs &a) { return conv_vector_smem(a) <= 200 * 1024; }

int launch_conv_vector(const ConvArgs &a, cudaStream_t s) {
    dim3 grid(unsigned((a.oc + VEC_COLS - 1) / VEC_COLS), unsigned((a.M + VEC_ROWS - 1) / VEC_ROWS));
    conv_vector_kernel<<<grid, VEC_COLS * VEC_ROWS, conv_vector_smem(a), s>>>(a);
    return 1;
}

}  // namespace ppocr
