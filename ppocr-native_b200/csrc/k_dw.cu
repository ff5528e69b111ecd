// Depthwise convolution, alone and feeding a pointwise GEMM tile from shared
// memory (sm_100a, FP32 pipes).
//
// Each depthwise output starts from its bias and adds its taps in kernel
// row-major order, one fused multiply-add each (reference
// `src/engine/conv.rs:244-339`, `kernels/depthwise.rs:12-45`), skipping taps
// that fall in the padding. In the fused kernel a block computes the
// depthwise outputs of BM consecutive pixels for every channel into shared
// memory, then runs the pointwise GEMM over them for every output channel:
// the depthwise map never reaches HBM.
#include <algorithm>
#include <cstdint>
#include <mutex>

#include "devmath.cuh"
#include "kernels.hpp"

namespace ppocr {

namespace {

// Where output pixel m of a depthwise layer reads: its lane's input, the
// lane's input size and the output coordinates.
struct DwPixel {
    const float *xn;
    int ih, iw, oy, ox;
};

__device__ __forceinline__ DwPixel dw_locate(const DwArgs &a, long m) {
    const LaneInfo &L = a.lanes[find_lane(a.lanes, a.nl, m)];
    DwPixel p;
    int ow = __ldg(&L.ow);
    int r = int(m - __ldg(&L.pix0));
    p.oy = r / ow;
    p.ox = r - p.oy * ow;
    p.ih = __ldg(&L.ih);
    p.iw = __ldg(&L.iw);
    p.xn = a.x + __ldg(&L.ipix0) * a.c;
    return p;
}

// Depthwise outputs of `count` channels (1 or 4) of one pixel, into v.
template <int VEC>
__device__ __forceinline__ void dw_pixel(const DwArgs &a, const DwPixel &px, int c, float v[VEC]) {
#pragma unroll
    for (int e = 0; e < VEC; e++) v[e] = a.b ? __ldg(a.b + c + e) : 0.0f;
    const float *xn = px.xn;
    for (int ky = 0; ky < a.kh; ky++) {
        int iy = px.oy * a.sh - a.pt + ky;
        if (iy < 0 || iy >= px.ih) continue;
        for (int kx = 0; kx < a.kw; kx++) {
            int ix = px.ox * a.sw - a.pl + kx;
            if (ix < 0 || ix >= px.iw) continue;
            const float *src = xn + ((long)iy * px.iw + ix) * a.c + c;
            const float *w = a.w + (ky * a.kw + kx) * a.c + c;
            if (VEC == 4) {
                float4 q = __ldg(reinterpret_cast<const float4 *>(src));
                float4 g = __ldg(reinterpret_cast<const float4 *>(w));
                v[0] = ffma(g.x, q.x, v[0]);
                v[1] = ffma(g.y, q.y, v[1]);
                v[2] = ffma(g.z, q.z, v[2]);
                v[3] = ffma(g.w, q.w, v[3]);
            } else {
                v[0] = ffma(__ldg(w), __ldg(src), v[0]);
            }
        }
    }
    if (a.quick) {
#pragma unroll
        for (int e = 0; e < VEC; e++) v[e] = activate<true>(a.act, v[e]);
    } else {
#pragma unroll
        for (int e = 0; e < VEC; e++) v[e] = activate(a.act, v[e]);
    }
}

template <int VEC>
__global__ void __launch_bounds__(256) dw_kernel(const DwArgs a) {
    long groups = a.M * (a.c / VEC);
    for (long g = (long)blockIdx.x * blockDim.x + threadIdx.x; g < groups; g += (long)gridDim.x * blockDim.x) {
        int cg = a.c / VEC;
        long m = g / cg;
        int c = int(g - m * cg) * VEC;
        float v[VEC];
        dw_pixel<VEC>(a, dw_locate(a, m), c, v);
        float *dst = a.y + m * a.c + c;
        if (VEC == 4)
            *reinterpret_cast<float4 *>(dst) = make_float4(v[0], v[1], v[2], v[3]);
        else
            dst[0] = v[0];
    }
}

// The first n outputs of a run, activated, four channels each.
template <int ACT, bool QUICK>
__device__ __forceinline__ void dw_store(const float4 (&v)[DW_RUN], float *dst, int c, int n) {
#pragma unroll
    for (int j = 0; j < DW_RUN; j++) {
        if (j >= n) break;
        const float4 o = make_float4(activate_t<ACT, QUICK>(v[j].x), activate_t<ACT, QUICK>(v[j].y),
                                     activate_t<ACT, QUICK>(v[j].z), activate_t<ACT, QUICK>(v[j].w));
        *reinterpret_cast<float4 *>(dst + (long)j * c) = o;
    }
}

// Depthwise outputs of DW_RUN consecutive pixels of one output row for four
// channels per thread: the input columns under the run are loaded once per
// kernel row (a window of (DW_RUN - 1) * S + K float4s) and shared by the
// run's outputs, and the thread's channels stay fixed across the grid-stride
// loop, so its weights and bias are loaded once (kept in registers for
// K = 3). Each output keeps the reference order: bias, then the taps inside
// the image in kernel row-major order. A block holds `per_block` runs of all
// c / 4 channel groups, the groups of one run on consecutive threads so that
// a warp's loads cover whole pixels.
// Weights: 3x3 stride 1 reads them from shared memory (fewer registers:
// three blocks per SM), 3x3 stride 2 holds them in registers, 5x5 reads them
// through L1 (each measured fastest its way).
template <int K, int S>
struct DwWeights {
    static constexpr bool SMEM = K == 3 && S == 1;
    static constexpr bool HOLD = K == 3 && S == 2;
    static constexpr int MIN_BLOCKS = SMEM || (K == 5 && S == 1) ? 3 : 2;
};

template <int K, int S, bool QUICK>
__global__ void __launch_bounds__(256, DwWeights<K, S>::MIN_BLOCKS) dw_row_kernel(const DwArgs a, int per_block) {
    constexpr int WC = (DW_RUN - 1) * S + K;  // window columns
    constexpr bool SMEM = DwWeights<K, S>::SMEM, HOLD = DwWeights<K, S>::HOLD;
    extern __shared__ __align__(16) float dw_ws[];  // SMEM: [K * K][c], the layer's weights
    if (SMEM) {
        for (int e = threadIdx.x; e < K * K * a.c; e += blockDim.x) dw_ws[e] = __ldg(a.w + e);
        __syncthreads();
    }
    const int cg = a.c >> 2;
    const int slot = threadIdx.x / cg;
    if (slot >= per_block) return;
    const int c = (threadIdx.x - slot * cg) * 4;
    const float4 zero = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const float4 bias = a.b ? __ldg(reinterpret_cast<const float4 *>(a.b + c)) : zero;
    float4 wr[HOLD ? K * K : 1];
    if (HOLD) {
#pragma unroll
        for (int t = 0; t < K * K; t++) wr[t] = __ldg(reinterpret_cast<const float4 *>(a.w + t * a.c + c));
    }
    for (long run = (long)blockIdx.x * per_block + slot; run < a.runs; run += (long)gridDim.x * per_block) {
        const LaneInfo &L = a.lanes[find_run_lane(a.lanes, a.nl, run)];
        const int ow = __ldg(&L.ow), ih = __ldg(&L.ih), iw = __ldg(&L.iw);
        const int rpr = (ow + DW_RUN - 1) / DW_RUN;
        const int r = int(run - __ldg(&L.run0));
        const int oy = r / rpr;
        const int ox0 = (r - oy * rpr) * DW_RUN;
        const int ix0 = ox0 * S - a.pl;
        unsigned cols = 0;  // window columns inside the image
#pragma unroll
        for (int i = 0; i < WC; i++)
            if (ix0 + i >= 0 && ix0 + i < iw) cols |= 1u << i;
        const float *xn = a.x + __ldg(&L.ipix0) * a.c + c;
        float4 v[DW_RUN];
#pragma unroll
        for (int j = 0; j < DW_RUN; j++) v[j] = bias;
#pragma unroll
        for (int ky = 0; ky < K; ky++) {
            const int iy = oy * S - a.pt + ky;
            if (iy < 0 || iy >= ih) continue;
            const float *row = xn + ((long)iy * iw + ix0) * a.c;
            float4 win[WC];
#pragma unroll
            for (int i = 0; i < WC; i++)
                win[i] = (cols >> i & 1u) ? __ldg(reinterpret_cast<const float4 *>(row + (long)i * a.c)) : zero;
#pragma unroll
            for (int kx = 0; kx < K; kx++) {
                const float4 g = HOLD   ? wr[HOLD ? ky * K + kx : 0]
                                 : SMEM ? *reinterpret_cast<const float4 *>(dw_ws + (ky * K + kx) * a.c + c)
                                        : __ldg(reinterpret_cast<const float4 *>(a.w + (ky * K + kx) * a.c + c));
#pragma unroll
                for (int j = 0; j < DW_RUN; j++) {
                    if (!(cols >> (j * S + kx) & 1u)) continue;
                    const float4 q = win[j * S + kx];
                    const float2 lo = ffma2(make_float2(g.x, g.y), make_float2(q.x, q.y), make_float2(v[j].x, v[j].y));
                    const float2 hi = ffma2(make_float2(g.z, g.w), make_float2(q.z, q.w), make_float2(v[j].z, v[j].w));
                    v[j] = make_float4(lo.x, lo.y, hi.x, hi.y);
                }
            }
        }
        float *dst = a.y + (__ldg(&L.pix0) + (long)oy * ow + ox0) * a.c + c;
        const int n = ow - ox0 < DW_RUN ? ow - ox0 : DW_RUN;
        if constexpr (K == 5) {
            // (the 5x5 kernels keep the per-value branch: the per-run one
            // costs them registers)
#pragma unroll
            for (int j = 0; j < DW_RUN; j++) {
                if (j >= n) break;
                const float4 o = make_float4(activate<QUICK>(a.act, v[j].x), activate<QUICK>(a.act, v[j].y),
                                             activate<QUICK>(a.act, v[j].z), activate<QUICK>(a.act, v[j].w));
                *reinterpret_cast<float4 *>(dst + (long)j * a.c) = o;
            }
            continue;
        }
        // one branch on the activation per run, not per value
        switch (a.act) {
        case 1: dw_store<1, QUICK>(v, dst, a.c, n); break;
        case 2: dw_store<2, QUICK>(v, dst, a.c, n); break;
        case 3: dw_store<3, QUICK>(v, dst, a.c, n); break;
        case 4: dw_store<4, QUICK>(v, dst, a.c, n); break;
        case 5: dw_store<5, QUICK>(v, dst, a.c, n); break;
        case 6: dw_store<6, QUICK>(v, dst, a.c, n); break;
        case 7: dw_store<7, QUICK>(v, dst, a.c, n); break;
        default: dw_store<0, QUICK>(v, dst, a.c, n); break;
        }
    }
}

// Resident 256-thread blocks per SM of each row-run instance (register
// bound), found once per process by configure_dw_kernels.
int g_row_resident[2][2][2];  // [K == 5][S == 2][QUICK]
int g_sms = 148;

template <int K, int S, bool QUICK>
void note_residency() {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, dw_row_kernel<K, S, QUICK>, 256, 0) != cudaSuccess || n < 1)
        n = 1;
    g_row_resident[K == 5][S == 2][QUICK] = n;
}

// One wave: at most as many blocks as can be resident at once, each looping
// over its share of the runs (keeping its weights).
template <int K, int S>
void run_dw_rows(const DwArgs &a, cudaStream_t s) {
    const int cg = a.c / 4;
    const int per_block = 256 / cg;
    long blocks = (a.runs + per_block - 1) / per_block;
    const size_t smem = DwWeights<K, S>::SMEM ? sizeof(float) * K * K * a.c : 0;
    int per_sm = g_row_resident[K == 5][S == 2][a.quick ? 1 : 0];
    if (long(per_sm) * long(smem + 1024) > 220L * 1024) per_sm = int(220L * 1024 / long(smem + 1024));
    const long wave = long(g_sms) * (per_sm < 1 ? 1 : per_sm);
    if (blocks > wave) blocks = wave;
    if (blocks < 1) blocks = 1;
    if (a.quick)
        dw_row_kernel<K, S, true><<<(unsigned)blocks, cg * per_block, smem, s>>>(a, per_block);
    else
        dw_row_kernel<K, S, false><<<(unsigned)blocks, cg * per_block, smem, s>>>(a, per_block);
}

constexpr int BK = 8;
constexpr int DPAD = 4;

// Fused depthwise -> pointwise. Threads TX x TY, each TM pixels x TN output
// channels of the current BN-wide output slice; BM = TM*TY pixels per block.
template <int TM, int TN, int TX, int TY>
__global__ void __launch_bounds__(TX *TY) dw_pw_kernel(const DwPwArgs a) {
    constexpr int BM = TM * TY, BN = TN * TX, THREADS = TX * TY;
    constexpr int BELEMS = BK * BN;
    constexpr int BLOADS = (BELEMS + THREADS - 1) / THREADS;
    extern __shared__ __align__(16) float smem[];
    const DwArgs &d = a.dw;
    const int C = d.c;
    float *Ds = smem;                              // [C][BM + DPAD]
    float *Bs = smem + (long)C * (BM + DPAD);      // [2][BK][BN]

    const int tid = threadIdx.x;
    const int tx = tid % TX, ty = tid / TX;
    const long M = d.M;
    const long m0 = (long)blockIdx.x * BM;

    // Phase 1: the depthwise tile, [channel][pixel].
    const bool vec = (C % 4) == 0;
    const int cg = vec ? C / 4 : C;
    for (int g = tid; g < BM * cg; g += THREADS) {
        int p = g / cg, c = (g - p * cg) * (vec ? 4 : 1);
        long m = m0 + p;
        if (m < M) {
            DwPixel px = dw_locate(d, m);
            if (vec) {
                float v[4];
                dw_pixel<4>(d, px, c, v);
#pragma unroll
                for (int e = 0; e < 4; e++) Ds[(c + e) * (BM + DPAD) + p] = v[e];
            } else {
                float v[1];
                dw_pixel<1>(d, px, c, v);
                Ds[c * (BM + DPAD) + p] = v[0];
            }
        } else {
            for (int e = 0; e < (vec ? 4 : 1); e++) Ds[(c + e) * (BM + DPAD) + p] = 0.0f;
        }
    }

    // Phase 2: pointwise GEMM over the tile, one BN slice at a time.
    const int ktiles = (C + BK - 1) / BK;
    float rb[BLOADS];
    for (int n0 = 0; n0 < a.oc; n0 += BN) {
        auto fetch = [&](int t) {
            int c0 = t * BK;
#pragma unroll
            for (int l = 0; l < BLOADS; l++) {
                int e = tid + l * THREADS;
                int kk = e / BN, nn = e - kk * BN;
                int c = c0 + kk, n = n0 + nn;
                rb[l] = (e < BELEMS && c < C && n < a.oc) ? __ldg(a.w2 + (long)c * a.oc + n) : 0.0f;
            }
        };
        auto stash = [&](int buf) {
#pragma unroll
            for (int l = 0; l < BLOADS; l++) {
                int e = tid + l * THREADS;
                if (e < BELEMS) Bs[buf * BELEMS + e] = rb[l];
            }
        };
        float acc[TM][TN];
        bool first[TM];
#pragma unroll
        for (int i = 0; i < TM; i++) {
            long m = m0 + ty * TM + i;
            bool f = a.bias_mode2 == BIAS_FIRST;
            if (a.bias_mode2 == BIAS_FIRST_BUT_ROW_TAIL && m < M) {
                DwPixel px = dw_locate(d, m);
                int ow = __ldg(&d.lanes[find_lane(d.lanes, d.nl, m)].ow);
                f = px.ox < ow - ow % 4;
            }
            first[i] = f;
#pragma unroll
            for (int j = 0; j < TN; j++) {
                int n = n0 + tx * TN + j;
                acc[i][j] = (f && a.b2 && n < a.oc) ? __ldg(a.b2 + n) : 0.0f;
            }
        }
        __syncthreads();  // the depthwise tile is complete; Bs is free
        fetch(0);
        stash(0);
        __syncthreads();
        for (int t = 0; t < ktiles; t++) {
            int buf = t & 1;
            if (t + 1 < ktiles) fetch(t + 1);
            int c0 = t * BK;
#pragma unroll
            for (int kk = 0; kk < BK; kk++) {
                if (c0 + kk >= C) break;
                float fa[TM], fb[TN];
                const float *arow = Ds + (c0 + kk) * (BM + DPAD) + ty * TM;
#pragma unroll
                for (int i = 0; i < TM; i++) fa[i] = arow[i];
#pragma unroll
                for (int j = 0; j < TN; j++) fb[j] = Bs[buf * BELEMS + kk * BN + tx * TN + j];
#pragma unroll
                for (int i = 0; i < TM; i++)
#pragma unroll
                    for (int j = 0; j < TN; j++) acc[i][j] = ffma(fb[j], fa[i], acc[i][j]);
            }
            if (t + 1 < ktiles) stash(buf ^ 1);
            __syncthreads();
        }
#pragma unroll
        for (int i = 0; i < TM; i++) {
            long m = m0 + ty * TM + i;
            if (m >= M) continue;
#pragma unroll
            for (int j = 0; j < TN; j++) {
                int n = n0 + tx * TN + j;
                if (n >= a.oc) continue;
                float v = acc[i][j];
                if (!first[i] && a.b2) v = fadd(v, __ldg(a.b2 + n));
                v = activate(a.act2, v);
                if (a.res) v = activate(a.act3, fadd(v, __ldg(a.res + m * a.oc + n)));
                a.y[m * a.oc + n] = v;
            }
        }
    }
}

template <int TM, int TN, int TX, int TY>
size_t dw_pw_smem(int C) {
    constexpr int BM = TM * TY, BN = TN * TX;
    return sizeof(float) * ((size_t)C * (BM + DPAD) + 2 * BK * BN);
}

template <int TM, int TN, int TX, int TY>
int run_dw_pw(const DwPwArgs &a, cudaStream_t s) {
    constexpr int BM = TM * TY;
    size_t smem = dw_pw_smem<TM, TN, TX, TY>(a.dw.c);
    long M = a.dw.M;
    dw_pw_kernel<TM, TN, TX, TY><<<(unsigned)((M + BM - 1) / BM), TX * TY, smem, s>>>(a);
    return 1;
}


// ---------------------------------------------------------------- row tiles

constexpr int TILE_THREADS = 256;

// Fused depthwise -> pointwise for narrow layers, by row tiles. A block
// keeps both layers' weights in shared memory for its whole life and walks
// tiles of TP consecutive output pixels of one row (TP * N = 256 * OPT):
//  1. the depthwise outputs of the tile, four channels per thread, taps read
//     through L1 (neighbouring outputs share them), into shared memory
//     [pixel][c] (row stride c + 1: the pointwise reads are conflict-free);
//  2. the pointwise outputs, OPT consecutive channels of one pixel per
//     thread, each a chain of c fused multiply-adds in channel order from
//     shared memory, then bias (first or last, as the reference's tiles put
//     it), activation, residual, and 16-byte stores: a warp writes whole
//     consecutive pixels.
// The depthwise map never leaves the chip. Every output is formed in the
// reference's order (depthwise: bias, then the taps inside the image in
// kernel row-major order; pointwise: the channel chain), so the results are
// the exact FP32 kernels' bits; QUICK selects the tensor-core mode's
// activation quotient.
template <int K, int S, int OPT, bool QUICK>
__global__ void __launch_bounds__(TILE_THREADS) dwpw_tile_kernel(const DwPwArgs a) {
    extern __shared__ __align__(16) float sm[];
    const DwArgs &d = a.dw;
    const int C = d.c, N = a.oc, tid = threadIdx.x;
    const int TP = TILE_THREADS * OPT / N, XS = C + 1, groups = N / OPT;
    float *wpw = sm;              // [C][N]
    float *wdw = wpw + C * N;     // [K * K][C]
    float *bdw = wdw + K * K * C; // [C]
    float *bpw = bdw + C;         // [N]
    float *xs = bpw + N;          // [TP][C + 1]
    for (int i = tid; i < C * N; i += TILE_THREADS) wpw[i] = __ldg(a.w2 + i);
    for (int i = tid; i < K * K * C; i += TILE_THREADS) wdw[i] = __ldg(d.w + i);
    for (int i = tid; i < C; i += TILE_THREADS) bdw[i] = d.b ? __ldg(d.b + i) : 0.0f;
    for (int i = tid; i < N; i += TILE_THREADS) bpw[i] = a.b2 ? __ldg(a.b2 + i) : 0.0f;
    __syncthreads();
    const int cg = C / 4;
    const bool first = a.bias_mode2 == BIAS_FIRST;
    const long tiles = a.rows * a.segs;
    for (long t = blockIdx.x; t < tiles; t += gridDim.x) {
        const long r = t / a.segs;
        const int seg = int(t - r * a.segs);
        const LaneInfo &L = d.lanes[d.nl > 1 ? find_row_lane(d.lanes, d.nl, r) : 0];
        const int ow = __ldg(&L.ow), ox0 = seg * TP;
        if (ox0 >= ow) continue;  // the whole block: this lane's row is shorter
        const int oy = int(r - __ldg(&L.row0)), ih = __ldg(&L.ih), iw = __ldg(&L.iw);
        const int np = min(TP, ow - ox0);
        const float *xn = d.x + __ldg(&L.ipix0) * C;
        // 1. depthwise
        for (int item = tid; item < np * cg; item += TILE_THREADS) {
            const int p = item / cg, c = (item - p * cg) * 4;
            const int ox = ox0 + p;
            float v0 = bdw[c], v1 = bdw[c + 1], v2 = bdw[c + 2], v3 = bdw[c + 3];
#pragma unroll
            for (int ky = 0; ky < K; ky++) {
                const int iy = oy * S - d.pt + ky;
                if (iy < 0 || iy >= ih) continue;
                const float *row = xn + long(iy) * iw * C + c;
#pragma unroll
                for (int kx = 0; kx < K; kx++) {
                    const int ix = ox * S - d.pl + kx;
                    if (ix < 0 || ix >= iw) continue;
                    const float4 q = __ldg(reinterpret_cast<const float4 *>(row + long(ix) * C));
                    const float4 w = *reinterpret_cast<const float4 *>(wdw + (ky * K + kx) * C + c);
                    v0 = ffma(w.x, q.x, v0);
                    v1 = ffma(w.y, q.y, v1);
                    v2 = ffma(w.z, q.z, v2);
                    v3 = ffma(w.w, q.w, v3);
                }
            }
            float *xp = xs + p * XS + c;
            xp[0] = activate<QUICK>(d.act, v0);
            xp[1] = activate<QUICK>(d.act, v1);
            xp[2] = activate<QUICK>(d.act, v2);
            xp[3] = activate<QUICK>(d.act, v3);
        }
        __syncthreads();
        // 2. pointwise
        const int p = tid / groups, n0 = (tid - p * groups) * OPT;
        if (p < np) {
            float acc[OPT];
#pragma unroll
            for (int j = 0; j < OPT; j++) acc[j] = first ? bpw[n0 + j] : 0.0f;
            const float *xp = xs + p * XS;
#pragma unroll 4
            for (int k = 0; k < C; k++) {
                const float x = xp[k];
                const float4 *wk = reinterpret_cast<const float4 *>(wpw + k * N + n0);
#pragma unroll
                for (int j4 = 0; j4 < OPT / 4; j4++) {
                    const float4 w = wk[j4];
                    acc[4 * j4] = ffma(w.x, x, acc[4 * j4]);
                    acc[4 * j4 + 1] = ffma(w.y, x, acc[4 * j4 + 1]);
                    acc[4 * j4 + 2] = ffma(w.z, x, acc[4 * j4 + 2]);
                    acc[4 * j4 + 3] = ffma(w.w, x, acc[4 * j4 + 3]);
                }
            }
            const long m = __ldg(&L.pix0) + long(oy) * ow + ox0 + p;
#pragma unroll
            for (int j4 = 0; j4 < OPT / 4; j4++) {
                float v[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    float u = acc[4 * j4 + e];
                    if (!first && a.b2) u = fadd(u, bpw[n0 + 4 * j4 + e]);
                    v[e] = activate<QUICK>(a.act2, u);
                }
                if (a.res) {
                    const float4 q = __ldg(reinterpret_cast<const float4 *>(a.res + m * N + n0 + 4 * j4));
                    v[0] = activate<QUICK>(a.act3, fadd(v[0], q.x));
                    v[1] = activate<QUICK>(a.act3, fadd(v[1], q.y));
                    v[2] = activate<QUICK>(a.act3, fadd(v[2], q.z));
                    v[3] = activate<QUICK>(a.act3, fadd(v[3], q.w));
                }
                *reinterpret_cast<float4 *>(a.y + m * N + n0 + 4 * j4) = make_float4(v[0], v[1], v[2], v[3]);
            }
        }
        __syncthreads();  // the tile's depthwise outputs are read; the next tile may write them
    }
}

int tile_opt(int N) { return N == 24 ? 12 : 24; }

size_t dwpw_tile_smem(const DwPwArgs &a) {
    const int C = a.dw.c, N = a.oc, K = a.dw.kh, TP = TILE_THREADS * tile_opt(N) / N;
    return sizeof(float) * (size_t(C) * N + size_t(K) * K * C + C + N + size_t(TP) * (C + 1));
}

template <int K, int S, int OPT, bool QUICK>
int run_dwpw_tile(const DwPwArgs &a, cudaStream_t s) {
    static int per_sm[2] = {0, 0};  // blocks per SM at the last smem size, found once per size
    static size_t at_smem = 0;
    static std::mutex mu;
    const size_t smem = dwpw_tile_smem(a);
    int resident;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (at_smem != smem || !per_sm[0]) {
            int n = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, dwpw_tile_kernel<K, S, OPT, QUICK>, TILE_THREADS,
                                                              smem) != cudaSuccess || n < 1)
                n = 1;
            per_sm[0] = n;
            at_smem = smem;
        }
        resident = per_sm[0];
    }
    const long tiles = a.rows * a.segs;
    const long blocks = std::max(1L, std::min(tiles, long(g_sms) * resident));
    dwpw_tile_kernel<K, S, OPT, QUICK><<<unsigned(blocks), TILE_THREADS, smem, s>>>(a);
    return 1;
}

}  // namespace

int launch_dw(const DwArgs &a, cudaStream_t s) {
    // square 3x3 and 5x5 kernels of stride 1 or 2 over whole float4s: row runs
    if (a.c % 4 == 0 && a.c <= 1024 && size_t(a.kh) * a.kw * a.c * 4 <= 48 * 1024 && a.runs > 0 && a.kh == a.kw && a.sh == a.sw && (a.kh == 3 || a.kh == 5) &&
        (a.sh == 1 || a.sh == 2)) {
        if (a.kh == 3)
            a.sh == 1 ? run_dw_rows<3, 1>(a, s) : run_dw_rows<3, 2>(a, s);
        else
            a.sh == 1 ? run_dw_rows<5, 1>(a, s) : run_dw_rows<5, 2>(a, s);
        return 1;
    }
    long work = a.M * (a.c % 4 == 0 ? a.c / 4 : a.c);
    long blocks = (work + 255) / 256;
    if (blocks > 148L * 64) blocks = 148L * 64;
    if (blocks < 1) blocks = 1;
    if (a.c % 4 == 0)
        dw_kernel<4><<<(unsigned)blocks, 256, 0, s>>>(a);
    else
        dw_kernel<1><<<(unsigned)blocks, 256, 0, s>>>(a);
    return 1;
}

template <int TM, int TN, int TX, int TY>
void allow_smem() {
    cudaFuncSetAttribute(dw_pw_kernel<TM, TN, TX, TY>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
}

template <int K, int S>
void allow_tile() {
    cudaFuncSetAttribute(dwpw_tile_kernel<K, S, 12, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
    cudaFuncSetAttribute(dwpw_tile_kernel<K, S, 12, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
    cudaFuncSetAttribute(dwpw_tile_kernel<K, S, 24, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
    cudaFuncSetAttribute(dwpw_tile_kernel<K, S, 24, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
}

// Raise the dynamic shared-memory ceiling of every fused instance; once per
// device, with that device current.
void configure_dw_kernels() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
        sms > 0)
        g_sms = sms;
    note_residency<3, 1, false>();
    note_residency<3, 1, true>();
    note_residency<3, 2, false>();
    note_residency<3, 2, true>();
    note_residency<5, 1, false>();
    note_residency<5, 1, true>();
    note_residency<5, 2, false>();
    note_residency<5, 2, true>();
    allow_smem<8, 6, 16, 16>();
    allow_smem<8, 4, 16, 16>();
    allow_smem<8, 3, 16, 16>();
    allow_smem<8, 3, 8, 16>();
    allow_smem<8, 2, 16, 16>();
    allow_smem<8, 4, 32, 8>();
    allow_smem<8, 3, 32, 8>();
    allow_smem<8, 2, 32, 8>();
    allow_tile<3, 1>();
    allow_tile<3, 2>();
    allow_tile<5, 1>();
    allow_tile<5, 2>();
}

bool dw_pw_supported(const DwPwArgs &a) {
    // The depthwise tile of 128 (or 64) pixels x C channels must fit.
    size_t smem = a.dw.c <= 192 ? dw_pw_smem<8, 4, 16, 16>(a.dw.c) : dw_pw_smem<8, 4, 32, 8>(a.dw.c);
    return smem <= 200 * 1024;
}


bool dwpw_tile_supported(const DwPwArgs &a) {
    const DwArgs &d = a.dw;
    const bool shape = (d.c == 24 || d.c == 48 || d.c == 96) && (a.oc == 24 || a.oc == 48 || a.oc == 96 || a.oc == 192) &&
                       d.kh == d.kw && (d.kh == 3 || d.kh == 5) && d.sh == d.sw && (d.sh == 1 || d.sh == 2);
    if (!shape || a.rows < 1 || a.segs < 1) return false;
    const auto aligned = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    return aligned(d.x) && aligned(d.w) && aligned(a.y) && (!a.res || aligned(a.res)) &&
           dwpw_tile_smem(a) <= 100 * 1024;
}

int dwpw_tile_pixels(const DwPwArgs &a) { return TILE_THREADS * tile_opt(a.oc) / a.oc; }

int launch_dwpw_tile(const DwPwArgs &a, bool quick, cudaStream_t s) {
    const int K = a.dw.kh, S = a.dw.sh, opt = tile_opt(a.oc);
#define PPOCR_TILE(KK, SS, OO)                                                                       \
    if (K == KK && S == SS && opt == OO)                                                             \
        return quick ? run_dwpw_tile<KK, SS, OO, true>(a, s) : run_dwpw_tile<KK, SS, OO, false>(a, s);
    PPOCR_TILE(3, 1, 12)
    PPOCR_TILE(3, 1, 24)
    PPOCR_TILE(3, 2, 12)
    PPOCR_TILE(3, 2, 24)
    PPOCR_TILE(5, 1, 12)
    PPOCR_TILE(5, 1, 24)
    PPOCR_TILE(5, 2, 12)
    PPOCR_TILE(5, 2, 24)
#undef PPOCR_TILE
    return 0;
}

int launch_dw_pw(const DwPwArgs &a, cudaStream_t s) {
    // 128 pixels per block up to 192 channels, else 64; the output slice is
    // 16 (or 32) threads x TN channels.
    if (a.dw.c <= 192) {
        if (a.oc % 96 == 0) return run_dw_pw<8, 6, 16, 16>(a, s);
        if (a.oc % 64 == 0) return run_dw_pw<8, 4, 16, 16>(a, s);
        if (a.oc % 48 == 0) return run_dw_pw<8, 3, 16, 16>(a, s);
        if (a.oc % 24 == 0) return run_dw_pw<8, 3, 8, 16>(a, s);
        return run_dw_pw<8, 2, 16, 16>(a, s);
    }
    if (a.oc % 128 == 0) return run_dw_pw<8, 4, 32, 8>(a, s);
    if (a.oc % 96 == 0) return run_dw_pw<8, 3, 32, 8>(a, s);
    return run_dw_pw<8, 2, 32, 8>(a, s);
}

}  // namespace ppocr
