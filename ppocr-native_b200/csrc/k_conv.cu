// Dense convolution as an implicit GEMM on the FP32 pipes (sm_100a).
//
// GEMM view: M = output pixels of all lanes, Nc = oc output channels,
// K = kh*kw*C with k = (ky*kw + kx)*C + c, the order of the weights
// `[kh][kw][C][oc]` and of the reference's sums (`kernels/dense.rs:20-36`).
// A block owns a BM x BN output tile; its threads hold TM x TN accumulators
// each. K advances one (tap, BK-channel slice) tile at a time, staged through
// double-buffered shared memory with the next tile prefetched into registers.
// Every accumulator adds its k terms in increasing k with one fused
// multiply-add each, starting from the bias or from zero as the reference's
// tiles do, so each output carries the reference's bits.
//
// The A tile is gathered on the fly: a padded tap reads zero, and each of up
// to four sources is read nearest-upsampled by 2^shift in place, so the
// neck's upsample + concat never reach memory. An SE gate (per lane and input
// channel) multiplies A as it is loaded; a residual add and a second
// activation run in the epilogue.
#include "devmath.cuh"
#include "kernels.hpp"

namespace ppocr {

namespace {

constexpr int BK = 8;
constexpr int APAD = 4;

template <int TM, int TN, int TX, int TY>
struct Cfg {
    static constexpr int BM = TM * TY, BN = TN * TX, THREADS = TX * TY;
    static constexpr int AGROUPS = BM * BK / 4;  // float4 groups of the A tile
    static constexpr int ALOADS = (AGROUPS + THREADS - 1) / THREADS;
    static constexpr int BELEMS = BK * BN;
    static constexpr int BLOADS = (BELEMS + THREADS - 1) / THREADS;
};

// Pixel coordinates of one A-load slot, fixed for the whole K loop: its
// lane, the lane's input size, and the top-left input tap.
struct Pixel {
    int n, iy0, ix0, ih, iw;
    bool ok;
};

__device__ __forceinline__ void load_a_group(const ConvArgs &a, const Pixel &px, int tap, int c, bool vec4,
                                             float v[4]) {
    v[0] = v[1] = v[2] = v[3] = 0.0f;
    if (!px.ok) return;
    int ky = tap / a.kw, kx = tap - ky * a.kw;
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

template <int TM, int TN, int TX, int TY>
__global__ void __launch_bounds__(TX *TY) conv_gemm(const ConvArgs a, int ctiles, int ntiles_k, bool vec4,
                                                    bool bvec4) {
    using C = Cfg<TM, TN, TX, TY>;
    constexpr int BM = C::BM, BN = C::BN;
    __shared__ __align__(16) float As[2][BK][BM + APAD];
    __shared__ __align__(16) float Bs[2][BK][BN];

    const int tid = threadIdx.x;
    const int tx = tid % TX, ty = tid / TX;
    const long M = a.M;
    const long m0 = (long)blockIdx.x * BM;
    const int n0 = blockIdx.y * BN;

    // A-load slots of this thread.
    Pixel px[C::ALOADS];
    int am[C::ALOADS], aq[C::ALOADS];
#pragma unroll
    for (int l = 0; l < C::ALOADS; l++) {
        int g = tid + l * C::THREADS;
        am[l] = g / (BK / 4);
        aq[l] = g % (BK / 4);
        long m = m0 + am[l];
        px[l].ok = g < C::AGROUPS && m < M;
        if (px[l].ok) {
            int n = find_lane(a.lanes, a.nl, m);
            const LaneInfo &L = a.lanes[n];
            int ow = __ldg(&L.ow);
            int r = int(m - __ldg(&L.pix0));
            int oy = r / ow, ox = r - oy * ow;
            px[l].n = n;
            px[l].ih = __ldg(&L.ih);
            px[l].iw = __ldg(&L.iw);
            px[l].iy0 = oy * a.sh - a.pt;
            px[l].ix0 = ox * a.sw - a.pl;
        } else {
            px[l].n = px[l].iy0 = px[l].ix0 = px[l].ih = px[l].iw = 0;
        }
    }

    float ra[C::ALOADS][4];
    float rb[C::BLOADS];

    auto fetch = [&](int t) {
        int tap = t / ctiles;
        int c0 = (t - tap * ctiles) * BK;
#pragma unroll
        for (int l = 0; l < C::ALOADS; l++) load_a_group(a, px[l], tap, c0 + aq[l] * 4, vec4, ra[l]);
        if (bvec4) {
#pragma unroll
            for (int l = 0; l < C::BLOADS; l += 4) {
                int e = (tid + (l / 4) * C::THREADS) * 4;
                if (l < C::BLOADS) {
                    int kk = e / BN, nn = e - kk * BN;
                    int c = c0 + kk, n = n0 + nn;
                    float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (e < C::BELEMS && c < a.C && n < a.oc)
                        q = __ldg(reinterpret_cast<const float4 *>(a.w + ((long)tap * a.C + c) * a.oc + n));
                    rb[l] = q.x;
                    if (l + 1 < C::BLOADS) rb[l + 1] = q.y;
                    if (l + 2 < C::BLOADS) rb[l + 2] = q.z;
                    if (l + 3 < C::BLOADS) rb[l + 3] = q.w;
                }
            }
        } else {
#pragma unroll
            for (int l = 0; l < C::BLOADS; l++) {
                int e = tid + l * C::THREADS;
                int kk = e / BN, nn = e - kk * BN;
                int c = c0 + kk, n = n0 + nn;
                rb[l] = (e < C::BELEMS && c < a.C && n < a.oc) ? __ldg(a.w + ((long)tap * a.C + c) * a.oc + n) : 0.0f;
            }
        }
    };
    auto stash = [&](int buf) {
#pragma unroll
        for (int l = 0; l < C::ALOADS; l++) {
            int g = tid + l * C::THREADS;
            if (g < C::AGROUPS) {
#pragma unroll
                for (int e = 0; e < 4; e++) As[buf][aq[l] * 4 + e][am[l]] = ra[l][e];
            }
        }
        if (bvec4) {
#pragma unroll
            for (int l = 0; l < C::BLOADS; l += 4) {
                int e = (tid + (l / 4) * C::THREADS) * 4;
                if (l < C::BLOADS && e < C::BELEMS) {
                    int kk = e / BN, nn = e - kk * BN;
                    float *d = &Bs[buf][kk][nn];
                    d[0] = rb[l];
                    if (l + 1 < C::BLOADS) d[1] = rb[l + 1];
                    if (l + 2 < C::BLOADS) d[2] = rb[l + 2];
                    if (l + 3 < C::BLOADS) d[3] = rb[l + 3];
                }
            }
        } else {
#pragma unroll
            for (int l = 0; l < C::BLOADS; l++) {
                int e = tid + l * C::THREADS;
                if (e < C::BELEMS) Bs[buf][e / BN][e % BN] = rb[l];
            }
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
        int buf = t & 1;
        if (t + 1 < ntiles_k) fetch(t + 1);
#pragma unroll
        for (int kk = 0; kk < BK; kk++) {
            float fa[TM], fb[TN];
#pragma unroll
            for (int i = 0; i < TM; i++) fa[i] = As[buf][kk][ty * TM + i];
#pragma unroll
            for (int j = 0; j < TN; j++) fb[j] = Bs[buf][kk][tx * TN + j];
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

template <int TM, int TN, int TX, int TY>
int run(const ConvArgs &a, cudaStream_t s, bool vec4) {
    using C = Cfg<TM, TN, TX, TY>;
    long M = a.M;
    int ctiles = (a.C + BK - 1) / BK;
    int taps = a.kh * a.kw;
    dim3 grid((unsigned)((M + C::BM - 1) / C::BM), (unsigned)((a.oc + C::BN - 1) / C::BN));
    bool bvec4 = (a.oc % 4 == 0) && (C::BN % 4 == 0) && (C::BLOADS % 4 == 0) &&
                 (C::BELEMS % (4 * C::THREADS) == 0);
    conv_gemm<TM, TN, TX, TY><<<grid, C::THREADS, 0, s>>>(a, ctiles, taps * ctiles, vec4, bvec4);
    return 1;
}

}  // namespace

int launch_conv(const ConvArgs &a, cudaStream_t s) {
    bool vec4 = true;
    for (int i = 0; i < a.nsrc; i++) vec4 = vec4 && (a.src[i].c % 4 == 0);
    int oc = a.oc;
    if (oc % 128 == 0) return run<8, 8, 16, 16>(a, s, vec4);
    if (oc % 96 == 0) return run<8, 6, 16, 16>(a, s, vec4);
    if (oc % 64 == 0) return run<8, 4, 16, 16>(a, s, vec4);
    if (oc % 48 == 0) return run<4, 6, 8, 32>(a, s, vec4);
    if (oc % 24 == 0) return run<4, 6, 4, 64>(a, s, vec4);
    if (oc <= 8) return run<4, 2, 4, 64>(a, s, vec4);
    if (oc <= 16) return run<4, 4, 4, 64>(a, s, vec4);
    if (oc <= 32) return run<4, 4, 8, 32>(a, s, vec4);
    return run<8, 4, 16, 16>(a, s, vec4);
}

}  // namespace ppocr
