// The layers around the convolutions (sm_100a): elementwise passes, pools,
// the f64 channel mean, LayerNorm, multi-head attention, the CTC head and
// the transposed convolution. Each follows the reference's arithmetic
// (`src/engine/layers.rs`, `kernels/elementwise.rs`); where a reduction is
// split across threads the split is noted.
#include <cfloat>

#include "devmath.cuh"
#include "kernels.hpp"

namespace ppocr {

namespace {

unsigned grid_for(long work, int threads = 256) {
    long blocks = (work + threads - 1) / threads;
    if (blocks > 148L * 32) blocks = 148L * 32;
    return (unsigned)(blocks < 1 ? 1 : blocks);
}

// ----------------------------------------------------------------- eltwise

// Four values (VEC) or one at a time; index arithmetic in 32 bits when the
// tensor allows (SMALL), 64 otherwise.
template <int VEC>
__device__ __forceinline__ void load_vec(const float *p, float v[VEC]) {
    if (VEC == 4) {
        const float4 q = __ldg(reinterpret_cast<const float4 *>(p));
        v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
    } else {
        v[0] = __ldg(p);
    }
}

template <int VEC, bool SMALL>
__global__ void __launch_bounds__(256) elt_kernel(const EltArgs a) {
    const int cout = a.mode == ELT_CONCAT ? a.c + a.c2 : a.c;
    const long total = a.M * cout / VEC;
    for (long g = (long)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (long)gridDim.x * blockDim.x) {
        const long e = g * VEC;
        const long m = SMALL ? long(unsigned(e) / unsigned(cout)) : e / cout;
        const int c = int(e - m * cout);
        float v[VEC];
        switch (a.mode) {
        case ELT_ADD: {
            float p[VEC], q[VEC];
            load_vec<VEC>(a.x + e, p);
            load_vec<VEC>(a.x2 + e, q);
#pragma unroll
            for (int k = 0; k < VEC; k++) v[k] = activate(a.act, fadd(p[k], q[k]));
            break;
        }
        case ELT_CHANNELMUL:
        case ELT_GATE_ADD: {
            const int n = a.nl > 1 ? find_lane(a.lanes, a.nl, m) : 0;
            float x[VEC], g[VEC];
            load_vec<VEC>(a.x + e, x);
            load_vec<VEC>(a.x2 + (long)n * a.c + c, g);
#pragma unroll
            for (int k = 0; k < VEC; k++) {
                const float p = fmul(x[k], g[k]);
                v[k] = a.mode == ELT_CHANNELMUL ? p : activate(a.act, fadd(p, x[k]));
            }
            break;
        }
        case ELT_UPSAMPLE:
        case ELT_UPSAMPLE_ADD:
        case ELT_GATE_UPSAMPLE_ADD: {
            const int n = a.nl > 1 ? find_lane(a.lanes, a.nl, m) : 0;
            const LaneInfo &L = a.lanes[n];
            const int ow = __ldg(&L.ow);
            const int r = int(m - __ldg(&L.pix0));
            const int oy = r / ow, ox = r - oy * ow;
            const long ip = __ldg(&L.ipix0) + (long)(oy / a.sh) * __ldg(&L.iw) + ox / a.sw;
            float u[VEC];
            load_vec<VEC>(a.x + ip * a.c + c, u);
            if (a.mode == ELT_UPSAMPLE) {
#pragma unroll
                for (int k = 0; k < VEC; k++) v[k] = u[k];
            } else {
                float q[VEC];
                load_vec<VEC>(a.x2 + e, q);
                if (a.mode == ELT_GATE_UPSAMPLE_ADD) {
                    // the full-size input as the gate-add would have written it
                    float gg[VEC];
                    load_vec<VEC>(a.g + (long)n * a.c + c, gg);
#pragma unroll
                    for (int k = 0; k < VEC; k++) q[k] = activate(a.act, fadd(fmul(q[k], gg[k]), q[k]));
                }
#pragma unroll
                for (int k = 0; k < VEC; k++) v[k] = fadd(q[k], u[k]);
            }
            break;
        }
        default: {  // ELT_CONCAT: c, a.c and a.c2 are multiples of VEC
            if (c < a.c)
                load_vec<VEC>(a.x + m * a.c + c, v);
            else
                load_vec<VEC>(a.x2 + m * a.c2 + (c - a.c), v);
        }
        }
        if (VEC == 4)
            *reinterpret_cast<float4 *>(a.y + e) = make_float4(v[0], v[1], v[2], v[3]);
        else
            a.y[e] = v[0];
    }
}

// ------------------------------------------------------------------- pools

// Max pool: windows cut short at the bottom and right edges, the first tap
// copied and later ones kept only when greater (conv.rs:404-440). Average
// pool: whole windows, taps summed in row-major order then divided
// (layers.rs:443-463).
// VEC channels per thread (4 when c % 4 == 0: float4 loads and stores, one
// lane search per four values); each channel keeps its own order.
template <int VEC>
__global__ void __launch_bounds__(256) pool_kernel(const PoolArgs a) {
    const int cg = a.c / VEC;
    const long total = a.M * cg;
    for (long g = (long)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (long)gridDim.x * blockDim.x) {
        const long m = g / cg;
        const int c = int(g - m * cg) * VEC;
        const LaneInfo &L = a.lanes[find_lane(a.lanes, a.nl, m)];
        const int ow = __ldg(&L.ow), ih = __ldg(&L.ih), iw = __ldg(&L.iw);
        const int r = int(m - __ldg(&L.pix0));
        const int oy = r / ow, ox = r - oy * ow;
        const float *xn = a.x + __ldg(&L.ipix0) * a.c + c;
        float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // the first VEC used
        bool seeded = false;
        for (int ky = 0; ky < a.kh; ky++) {
            const int iy = oy * a.sh + ky;
            if (iy >= ih) continue;
            for (int kx = 0; kx < a.kw; kx++) {
                const int ix = ox * a.sw + kx;
                if (ix >= iw) continue;
                const float *src = xn + ((long)iy * iw + ix) * a.c;
                float x[4];
                if (VEC == 4) {
                    const float4 q = __ldg(reinterpret_cast<const float4 *>(src));
                    x[0] = q.x; x[1] = q.y; x[2] = q.z; x[3] = q.w;
                } else {
                    x[0] = __ldg(src);
                }
#pragma unroll
                for (int e = 0; e < VEC; e++) {
                    if (a.average)
                        v[e] = fadd(v[e], x[e]);
                    else if (!seeded || x[e] > v[e])
                        v[e] = x[e];
                }
                seeded = true;
            }
        }
        float *dst = a.y + m * a.c + c;
#pragma unroll
        for (int e = 0; e < VEC; e++) {
            if (a.average) v[e] = fdiv(v[e], float(a.kh * a.kw));
            if (VEC == 1) dst[e] = v[e];
        }
        if (VEC == 4) *reinterpret_cast<float4 *>(dst) = make_float4(v[0], v[1], v[2], v[3]);
    }
}

// -------------------------------------------------------------------- mean

// Stage 1: each block sums a run of pixels of one lane, per channel, in f64.
// The reference sums all pixels in order in f64 (layers.rs:387-406); the
// split into runs changes only f64 rounding, far below the f32 result's.
__global__ void __launch_bounds__(256) mean_partial_kernel(const MeanArgs a) {
    extern __shared__ double sums[];  // [rows][c]
    const int n = blockIdx.y, chunk = blockIdx.x;
    const int rows = blockDim.x / a.c;  // pixels summed side by side
    const int t = threadIdx.x;
    const LaneInfo &L = a.lanes[n];
    const int hw = __ldg(&L.ih) * __ldg(&L.iw);
    const int chunks = mean_chunks(hw, a.c);  // a.chunks is the most of any lane
    if (chunk >= chunks) return;
    const int per = (hw + chunks - 1) / chunks;
    const int p0 = chunk * per, p1 = min(hw, p0 + per);
    const float *x = a.x + __ldg(&L.ipix0) * a.c;
    if (rows >= 1) {
        int row = t / a.c, c = t - row * a.c;
        double s = 0.0;
        if (row < rows) {
            int p = p0 + row;
            // eight independent loads in flight, added in pixel order
            for (; p + 7 * rows < p1; p += 8 * rows) {
                float v[8];
#pragma unroll
                for (int u = 0; u < 8; u++) v[u] = __ldg(x + (long)(p + u * rows) * a.c + c);
#pragma unroll
                for (int u = 0; u < 8; u++) s += (double)v[u];
            }
            for (; p < p1; p += rows) s += (double)x[(long)p * a.c + c];
            sums[row * a.c + c] = s;
        }
        __syncthreads();
        if (t < a.c) {
            double total = 0.0;
            for (int r = 0; r < rows; r++) total += sums[r * a.c + t];
            a.partial[((long)n * a.chunks + chunk) * a.c + t] = total;
        }
    } else {
        for (int c = t; c < a.c; c += blockDim.x) {
            double s = 0.0;
            int p = p0;
            for (; p + 3 < p1; p += 4) {
                const float v0 = x[(long)p * a.c + c], v1 = x[(long)(p + 1) * a.c + c];
                const float v2 = x[(long)(p + 2) * a.c + c], v3 = x[(long)(p + 3) * a.c + c];
                s += (double)v0;
                s += (double)v1;
                s += (double)v2;
                s += (double)v3;
            }
            for (; p < p1; p++) s += (double)x[(long)p * a.c + c];
            a.partial[((long)n * a.chunks + chunk) * a.c + c] = s;
        }
    }
}

// Stage 2: one block per (lane, 32 channels); 32 rows of threads sum the
// lane's runs strided, then their 32 partials are added in row order.
__global__ void __launch_bounds__(1024) mean_final_kernel(const MeanArgs a) {
    __shared__ double part[32][33];
    const int n = blockIdx.y, c = blockIdx.x * 32 + threadIdx.x % 32, row = threadIdx.x / 32;
    const int hw = a.lanes[n].ih * a.lanes[n].iw;
    const int chunks = mean_chunks(hw, a.c);
    double s = 0.0;
    if (c < a.c) {
        // eight loads in flight, added in run order
        const double *pp = a.partial + (long)n * a.chunks * a.c + c;
        int k = row;
        for (; k + 7 * 32 < chunks; k += 8 * 32) {
            double v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v[u] = pp[(long)(k + 32 * u) * a.c];
#pragma unroll
            for (int u = 0; u < 8; u++) s += v[u];
        }
        for (; k < chunks; k += 32) s += pp[(long)k * a.c];
    }
    part[row][threadIdx.x % 32] = s;
    __syncthreads();
    if (row == 0 && c < a.c) {
        double total = 0.0;
        for (int r = 0; r < 32; r++) total += part[r][threadIdx.x];
        a.y[(long)n * a.c + c] = (float)(total / (double)hw);
    }
}

// --------------------------------------------------------------- layernorm

// One warp per pixel. The pixel's values go through shared memory and every
// lane then forms the same sums in channel order, as the reference does
// (layers.rs:467-479), so the result carries its bits.
__global__ void __launch_bounds__(128) layernorm_kernel(const LayerNormArgs a) {
    extern __shared__ float vals[];  // [4 warps][c]
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const long p = (long)blockIdx.x * 4 + warp;
    if (p >= a.pixels) return;
    float *v = vals + warp * a.c;
    const float *x = a.x + p * a.c;
    for (int k = lane; k < a.c; k += 32) v[k] = x[k];
    __syncwarp();
    float s = 0.0f;
    for (int k = 0; k < a.c; k++) s = fadd(s, v[k]);
    float m = fdiv(s, float(a.c));
    float q = 0.0f;
    for (int k = 0; k < a.c; k++) {
        float d = fsub(v[k], m);
        q = fadd(q, fmul(d, d));
    }
    float var = fdiv(q, float(a.c));
    float r = __fsqrt_rn(fadd(var, a.w[2 * a.c]));
    for (int k = lane; k < a.c; k += 32)
        a.y[p * a.c + k] = fadd(fmul(fdiv(fsub(v[k], m), r), a.w[k]), a.w[a.c + k]);
}

// The tensor-core mode's LayerNorm (tolerance, not bits): one warp per
// pixel, each lane summing its channels (k = lane, lane + 32, ...), the
// partial sums folded to lane 0 by shuffles and broadcast from it, so every
// lane normalizes with the same mean and deviation; the mean first, then the
// squared deviations from it, as the exact kernel does.
__global__ void __launch_bounds__(256) layernorm_fast_kernel(const LayerNormArgs a) {
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const long p = (long)blockIdx.x * 8 + warp;
    if (p >= a.pixels) return;
    const float *x = a.x + p * a.c;
    constexpr int PER = 16;  // up to 512 channels
    float v[PER];
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const int k = lane + 32 * j;
        v[j] = k < a.c ? __ldg(x + k) : 0.0f;
        s += v[j];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_down_sync(0xffffffffu, s, off);
    const float m = __shfl_sync(0xffffffffu, s, 0) / float(a.c);
    float q = 0.0f;
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const int k = lane + 32 * j;
        const float d = v[j] - m;
        if (k < a.c) q = fmaf(d, d, q);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) q += __shfl_down_sync(0xffffffffu, q, off);
    const float var = __shfl_sync(0xffffffffu, q, 0) / float(a.c);
    const float r = 1.0f / sqrtf(var + a.w[2 * a.c]);
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const int k = lane + 32 * j;
        if (k < a.c) a.y[p * a.c + k] = fmaf((v[j] - m) * r, __ldg(a.w + k), __ldg(a.w + a.c + k));
    }
}

// --------------------------------------------------------------- attention

// One block per (lane, head, run of ATT_Q queries), one thread per query. Per
// query, as the reference (layers.rs:488-522 with softmax_row :254-294):
// scores (q * scale) . k summed over the head dimension in order; the
// maximum; the exponentials summed in 8 lanes (element j in lane j % 8) over
// whole groups of eight, the lanes folded in order, the rest added one at a
// time; each probability e * (1 / sum); the output sum of v * p over the
// keys in order. Scores and exponentials are recomputed per pass instead of
// stored (the same operations give the same bits), four keys at a time so
// that their independent chains overlap; every running sum still takes its
// terms in key order.
constexpr int ATT_Q = 128;

template <int HD>
__global__ void __launch_bounds__(ATT_Q) attention_kernel(const AttentionArgs a) {
    extern __shared__ float kv[];  // K [t][hd], V [t][hd]
    const int n = blockIdx.x / a.heads, h = blockIdx.x % a.heads;
    const LaneInfo &L = a.lanes[n];
    const int hd = HD > 0 ? HD : a.c / a.heads, t = L.iw, c = a.c;
    const int s = blockIdx.y * ATT_Q + threadIdx.x;
    if (blockIdx.y * ATT_Q >= t) return;
    float *K = kv, *V = kv + t * hd;
    const float *x = a.x + L.ipix0 * 3 * c;
    for (int i = threadIdx.x; i < t * hd; i += blockDim.x) {
        int j = i / hd, d = i - j * hd;
        K[i] = x[(long)j * 3 * c + c + h * hd + d];
        V[i] = x[(long)j * 3 * c + 2 * c + h * hd + d];
    }
    __syncthreads();
    if (s >= t) return;
    const float scale = a.scale[0];
    constexpr int MAXHD = HD > 0 ? HD : 64;
    float q[MAXHD];
#pragma unroll
    for (int d = 0; d < MAXHD; d++)
        if (d < hd) q[d] = fmul(x[(long)s * 3 * c + h * hd + d], scale);
    auto score = [&](int j) {
        float acc = 0.0f;
        const float *k = K + j * hd;
#pragma unroll
        for (int d = 0; d < MAXHD; d++)
            if (d < hd) acc = ffma(k[d], q[d], acc);
        return acc;
    };
    float mx = -FLT_MAX;
    bool any = false;
    int j = 0;
    for (; j + 4 <= t; j += 4) {
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; u++) v[u] = score(j + u);
#pragma unroll
        for (int u = 0; u < 4; u++) {
            if (!any || v[u] > mx) mx = v[u];
            any = true;
        }
    }
    for (; j < t; j++) {
        float v = score(j);
        if (!any || v > mx) mx = v;
        any = true;
    }
    const int body = t / 8 * 8;
    float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j0 = 0; j0 < body; j0 += 8)
#pragma unroll
        for (int l = 0; l < 8; l++) lanes[l] = fadd(lanes[l], exp_neg(fsub(score(j0 + l), mx)));
    float sum = 0.0f;
#pragma unroll
    for (int l = 0; l < 8; l++) sum = fadd(sum, lanes[l]);
    for (int jj = body; jj < t; jj++) sum = fadd(sum, exp_neg(fsub(score(jj), mx)));
    float r = fdiv(1.0f, sum);
    float out[MAXHD];
#pragma unroll
    for (int d = 0; d < MAXHD; d++) out[d] = 0.0f;
    j = 0;
    for (; j + 4 <= t; j += 4) {
        float p[4];
#pragma unroll
        for (int u = 0; u < 4; u++) p[u] = fmul(exp_neg(fsub(score(j + u), mx)), r);
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const float *v = V + (j + u) * hd;
#pragma unroll
            for (int d = 0; d < MAXHD; d++)
                if (d < hd) out[d] = ffma(v[d], p[u], out[d]);
        }
    }
    for (; j < t; j++) {
        float p = fmul(exp_neg(fsub(score(j), mx)), r);
        const float *v = V + j * hd;
#pragma unroll
        for (int d = 0; d < MAXHD; d++)
            if (d < hd) out[d] = ffma(v[d], p, out[d]);
    }
    float *y = a.y + (L.pix0 + s) * c + h * hd;
#pragma unroll
    for (int d = 0; d < MAXHD; d++)
        if (d < hd) y[d] = out[d];
}

// The tensor-core mode's attention (head size 15): a block per (lane, head,
// 32 queries), eight threads per query taking keys j = l mod 8. K and V of
// the lane and head are staged in shared memory, each row padded to 20
// floats (a key's 15 values read as four 16-byte loads; the eight keys of a
// query's threads fall in distinct banks). One pass over the keys with an
// online softmax (a running maximum; the sum and the value row rescaled by
// exp(old - new) when it rises, __expf), then the eight threads' states merge
// by shuffles and the row is divided by the sum. Within a few ulp of the
// two-pass exact kernel, in another order.
constexpr int ATT_FAST_Q = 32;  // queries per block (x 8 threads)
constexpr int ATT_ROW = 20;     // padded K / V row (floats)

template <int HD>
__global__ void __launch_bounds__(ATT_FAST_Q * 8) attention_fast_kernel(const AttentionArgs a) {
    static_assert(HD <= 16, "one row is four float4s");
    extern __shared__ __align__(16) float kv[];  // K [t][ATT_ROW], V [t][ATT_ROW]
    const int n = blockIdx.x / a.heads, h = blockIdx.x % a.heads;
    const LaneInfo &L = a.lanes[n];
    const int t = L.iw, c = a.c;
    if (blockIdx.y * ATT_FAST_Q >= t) return;
    float *K = kv, *V = kv + t * ATT_ROW;
    const float *x = a.x + L.ipix0 * 3 * c;
    for (int i0 = threadIdx.x; i0 < t * ATT_ROW; i0 += 4 * blockDim.x) {
        float kk[4], vv[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int i = i0 + u * blockDim.x, j = i / ATT_ROW, d = i - j * ATT_ROW;
            const bool in = i < t * ATT_ROW && d < HD;
            kk[u] = in ? __ldg(x + (long)j * 3 * c + c + h * HD + d) : 0.0f;
            vv[u] = in ? __ldg(x + (long)j * 3 * c + 2 * c + h * HD + d) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 4; u++)
            if (i0 + u * blockDim.x < t * ATT_ROW) {
                K[i0 + u * blockDim.x] = kk[u];
                V[i0 + u * blockDim.x] = vv[u];
            }
    }
    __syncthreads();
    const int l = threadIdx.x % 8;
    const int s = blockIdx.y * ATT_FAST_Q + threadIdx.x / 8;
    const bool live = s < t;
    const float scale = a.scale[0];
    float q[16];
#pragma unroll
    for (int d = 0; d < 16; d++) q[d] = live && d < HD ? x[(long)s * 3 * c + h * HD + d] * scale : 0.0f;
    float m = -FLT_MAX, sum = 0.0f, o[16];
#pragma unroll
    for (int d = 0; d < 16; d++) o[d] = 0.0f;
    for (int j = l; j < t; j += 8) {
        const float4 *k4 = reinterpret_cast<const float4 *>(K + j * ATT_ROW);
        float acc = 0.0f;
#pragma unroll
        for (int g = 0; g < 4; g++) {
            const float4 kq = k4[g];
            acc = fmaf(kq.x, q[4 * g], acc);
            acc = fmaf(kq.y, q[4 * g + 1], acc);
            acc = fmaf(kq.z, q[4 * g + 2], acc);
            acc = fmaf(kq.w, q[4 * g + 3], acc);
        }
        if (acc > m) {
            const float f = __expf(m - acc);  // 0 on the first key
            sum *= f;
#pragma unroll
            for (int d = 0; d < 16; d++) o[d] *= f;
            m = acc;
        }
        const float p = __expf(acc - m);
        sum += p;
        const float4 *v4 = reinterpret_cast<const float4 *>(V + j * ATT_ROW);
#pragma unroll
        for (int g = 0; g < 4; g++) {
            const float4 vq = v4[g];
            o[4 * g] = fmaf(vq.x, p, o[4 * g]);
            o[4 * g + 1] = fmaf(vq.y, p, o[4 * g + 1]);
            o[4 * g + 2] = fmaf(vq.z, p, o[4 * g + 2]);
            o[4 * g + 3] = fmaf(vq.w, p, o[4 * g + 3]);
        }
    }
    // the eight threads' states: rescaled to the query's maximum, then summed
    float mq = m;
#pragma unroll
    for (int off = 4; off > 0; off >>= 1) mq = fmaxf(mq, __shfl_xor_sync(0xffffffffu, mq, off));
    const float f = sum > 0.0f ? __expf(m - mq) : 0.0f;  // a thread without keys holds nothing
    sum *= f;
#pragma unroll
    for (int d = 0; d < HD; d++) o[d] *= f;
#pragma unroll
    for (int off = 4; off > 0; off >>= 1) {
        sum += __shfl_xor_sync(0xffffffffu, sum, off);
#pragma unroll
        for (int d = 0; d < HD; d++) o[d] += __shfl_xor_sync(0xffffffffu, o[d], off);
    }
    if (!live) return;
    const float r = 1.0f / sum;
    float *y = a.y + (L.pix0 + s) * c + h * HD;
    // the eight threads write two outputs each
#pragma unroll
    for (int d = 0; d < HD; d++)
        if (d % 8 == l) y[d] = o[d] * r;
}

// --------------------------------------------------------------------- ctc

constexpr int CTC_PX = 64;     // pixels (time steps) per block
constexpr int CTC_COLS = 128;  // columns (8 panels) per block
constexpr int CTC_THREADS = 256;
constexpr int CTC_TP = 4;      // pixels per thread
constexpr int CTC_TC = 8;      // columns per thread (two runs of 4)

// Logits of CTC_PX pixels x CTC_COLS columns as a GEMM tile: the block's
// inputs [ci][CTC_PX] and weight panels [ci][CTC_COLS] sit in shared memory,
// each thread holds 4 pixels x 8 columns. Every logit starts from its bias
// and adds the inputs in order (layers.rs:771-777), so it carries the
// reference's bits. The block then reduces its columns per pixel to (max,
// sum exp(logit - max), first column reaching max) with warp shuffles. The
// reference runs one online softmax per pixel over all panels in order;
// merging per-block states instead changes only the rounding of the sum
// (argmax and maximum are exact).
__global__ void __launch_bounds__(CTC_THREADS) ctc_logits_kernel(const CtcArgs a) {
    extern __shared__ __align__(16) float sm[];
    float *xs = sm;                       // [ci][CTC_PX]
    float *ws = sm + a.ci * CTC_PX;       // [ci][CTC_COLS]
    const int p0 = blockIdx.x * CTC_PX, cb = blockIdx.y;
    const int col0 = cb * CTC_COLS;
    for (int i = threadIdx.x; i < a.ci * CTC_PX; i += CTC_THREADS) {
        int p = i / a.ci, k = i - p * a.ci;  // coalesced over k
        xs[k * CTC_PX + p] = p0 + p < a.pixels ? __ldg(a.x + (long)(p0 + p) * a.ci + k) : 0.0f;
    }
    // Panels j = col / 16 hold [ci][16] contiguous floats each.
    for (int i = threadIdx.x; i < a.ci * CTC_COLS / 4; i += CTC_THREADS) {
        int e = i * 4;
        int panel = e / (a.ci * 16), r = e - panel * a.ci * 16;
        int k = r / 16, c16 = r - k * 16;
        int col = col0 + panel * 16 + c16;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (col < a.cols)
            v = __ldg(reinterpret_cast<const float4 *>(a.w + ((long)(col >> 4) * a.ci + k) * 16 + c16));
        *reinterpret_cast<float4 *>(ws + k * CTC_COLS + panel * 16 + c16) = v;
    }
    __syncthreads();
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;  // 16 column groups x 16 pixel groups
    // Columns of this thread: 4 at tx*4 and 4 at 64 + tx*4, so a half-warp
    // reads 256 contiguous bytes of each weight row.
    int cols[CTC_TC];
#pragma unroll
    for (int j = 0; j < CTC_TC; j++) cols[j] = col0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
    float acc[CTC_TP][CTC_TC];
#pragma unroll
    for (int j = 0; j < CTC_TC; j++) {
        float b = cols[j] < a.cols ? __ldg(a.b + cols[j]) : -FLT_MAX;
#pragma unroll
        for (int i = 0; i < CTC_TP; i++) acc[i][j] = b;
    }
    for (int k = 0; k < a.ci; k++) {
        float4 xv = *reinterpret_cast<const float4 *>(xs + k * CTC_PX + ty * CTC_TP);
        float4 w0 = *reinterpret_cast<const float4 *>(ws + k * CTC_COLS + tx * 4);
        float4 w1 = *reinterpret_cast<const float4 *>(ws + k * CTC_COLS + 64 + tx * 4);
        float x4[4] = {xv.x, xv.y, xv.z, xv.w};
        float w8[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < CTC_TP; i++)
#pragma unroll
            for (int j = 0; j < CTC_TC; j++) acc[i][j] = ffma(w8[j], x4[i], acc[i][j]);
    }
#pragma unroll
    for (int i = 0; i < CTC_TP; i++) {
        const int p = p0 + ty * CTC_TP + i;
        float m = -FLT_MAX;
        int best = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < CTC_TC; j++) {
            bool live = cols[j] < a.vocab;
            float v = acc[i][j];
            if (live && (v > m || (v == m && cols[j] < best))) { m = v; best = cols[j]; }
            if (a.probs && live && p < a.pixels) a.y[(long)p * a.vocab + cols[j]] = v;
        }
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < CTC_TC; j++)
            if (cols[j] < a.vocab) s = fadd(s, exp_neg(fsub(acc[i][j], m)));
        // Combine the 16 column groups of this pixel (lanes of a half-warp).
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) {
            float m2 = __shfl_xor_sync(0xffffffffu, m, off);
            float s2 = __shfl_xor_sync(0xffffffffu, s, off);
            int b2 = __shfl_xor_sync(0xffffffffu, best, off);
            float mm = m2 > m ? m2 : m;
            float sa = m > -FLT_MAX ? fmul(s, exp_neg(fsub(m, mm))) : 0.0f;
            float sb = m2 > -FLT_MAX ? fmul(s2, exp_neg(fsub(m2, mm))) : 0.0f;
            // a fixed order for the pair, whichever lane computes it
            s = (tx & off) ? fadd(sb, sa) : fadd(sa, sb);
            best = (m2 > m || (m2 == m && b2 < best)) ? b2 : best;
            m = mm;
        }
        if (tx == 0 && p < a.pixels) {
            float *st = a.partial + ((long)p * a.col_blocks + cb) * 3;
            st[0] = m;
            st[1] = s;
            st[2] = __int_as_float(best);
        }
    }
}

// Merge the column blocks of each pixel in order: the largest maximum, the
// rescaled sums, the smallest column holding the maximum (layers.rs:813-832).
__global__ void ctc_merge_kernel(const CtcArgs a) {
    int p = blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= a.pixels) return;
    const float *st = a.partial + (long)p * a.col_blocks * 3;
    float m = -FLT_MAX;
    int best = 0x7fffffff;
    for (int b = 0; b < a.col_blocks; b++) {
        float v = st[b * 3];
        int col = __float_as_int(st[b * 3 + 2]);
        if (v > m || (v == m && col < best)) { m = v; best = col; }
    }
    float s = 0.0f;
    for (int b = 0; b < a.col_blocks; b++)
        if (st[b * 3] > -FLT_MAX) s = fadd(s, fmul(st[b * 3 + 1], exp_neg(fsub(st[b * 3], m))));
    float r = fdiv(1.0f, s);
    if (a.probs) {
        for (int c = 0; c < a.vocab; c++) {
            float *v = a.y + (long)p * a.vocab + c;
            *v = fmul(exp_neg(fsub(*v, m)), r);
        }
    } else {
        a.y[2 * p] = (float)best;
        a.y[2 * p + 1] = r;
    }
}

// ------------------------------------------------------------ convtranspose

// Non-overlapping transposed convolution (layers.rs:595-680): each input
// pixel's channels times w [ic][kh][kw][oc] give its kh x kw block of
// outputs. One thread per (input pixel, 4 output columns of the block); the
// bias first or last as a pointwise layer of kh*kw*oc columns takes it.
__global__ void __launch_bounds__(256) convt_kernel(const ConvTArgs a) {
    const int cols = a.kh * a.kw * a.oc;
    const int cg = (cols + 3) / 4;
    const long total = a.Min * cg;
    for (long g = (long)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (long)gridDim.x * blockDim.x) {
        long pix = g / cg;
        int c0 = int(g - pix * cg) * 4;
        const float *x = a.x + pix * a.ic;
        float acc[4];
#pragma unroll
        for (int j = 0; j < 4; j++) acc[j] = (a.b && a.bias_first && c0 + j < cols) ? a.b[c0 + j] : 0.0f;
        for (int i = 0; i < a.ic; i++) {
            float xv = x[i];
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (c0 + j < cols) acc[j] = ffma(a.w[(long)i * cols + c0 + j], xv, acc[j]);
        }
        const LaneInfo &L = a.lanes[find_lane(a.lanes, a.nl, pix, true)];
        int iw = __ldg(&L.iw), ow = iw * a.kw;
        int r = int(pix - __ldg(&L.ipix0));
        int iy = r / iw, ix = r - iy * iw;
        long obase = __ldg(&L.pix0);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            int col = c0 + j;
            if (col >= cols) break;
            float v = acc[j];
            if (a.b && !a.bias_first) v = fadd(v, a.b[col]);
            v = activate(a.act, v);
            int tap = col / a.oc, o = col - tap * a.oc;
            int ky = tap / a.kw, kx = tap - ky * a.kw;
            long oy = (long)iy * a.kh + ky, ox = (long)ix * a.kw + kx;
            a.y[(obase + oy * ow + ox) * a.oc + o] = v;
        }
    }
}

}  // namespace

// ------------------------------------------------------------------ gather

// One thread per (pixel, 4 channels), grid-strided; every source's channel
// count is a multiple of 4.
__global__ void __launch_bounds__(256) gather_kernel(const GatherArgs a) {
    const int groups = a.C / 4;
    const long total = a.M * groups;
    for (long g = (long)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (long)gridDim.x * blockDim.x) {
        const long m = g / groups;
        const int c = int(g - m * groups) * 4;
        const int n = find_lane(a.lanes, a.nl, m, true);
        const LaneInfo &L = a.lanes[n];
        const int iw = __ldg(&L.iw);
        const int q = int(m - __ldg(&L.ipix0));
        const int iy = q / iw, ix = q - iy * iw;
        int start = 0, s = 0;
        while (s + 1 < a.nsrc && c >= start + a.src[s].c) {
            start += a.src[s].c;
            s++;
        }
        const ConvSource &src = a.src[s];
        const int sh = src.shift;
        const long pix = __ldg(&L.spix0[s]) + (long)(iy >> sh) * (iw >> sh) + (ix >> sh);
        const float4 v = __ldg(reinterpret_cast<const float4 *>(src.p + pix * src.c + (c - start)));
        *reinterpret_cast<float4 *>(a.y + m * a.C + c) = v;
    }
}

int launch_gather(const GatherArgs &a, cudaStream_t s) {
    gather_kernel<<<grid_for(a.M * (a.C / 4)), 256, 0, s>>>(a);
    return 1;
}

int launch_elt(const EltArgs &a, cudaStream_t s) {
    const int cout = a.mode == ELT_CONCAT ? a.c + a.c2 : a.c;
    const auto aligned = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    const bool vec = cout % 4 == 0 && a.c % 4 == 0 && (a.mode != ELT_CONCAT || a.c2 % 4 == 0) && aligned(a.x) &&
                     aligned(a.y) && (!a.x2 || aligned(a.x2)) && (!a.g || aligned(a.g));
    const long total = a.M * cout;
    const bool small = total < (1L << 31);
    if (vec)
        small ? elt_kernel<4, true><<<grid_for(total / 4), 256, 0, s>>>(a)
              : elt_kernel<4, false><<<grid_for(total / 4), 256, 0, s>>>(a);
    else
        small ? elt_kernel<1, true><<<grid_for(total), 256, 0, s>>>(a)
              : elt_kernel<1, false><<<grid_for(total), 256, 0, s>>>(a);
    return 1;
}

int launch_pool(const PoolArgs &a, cudaStream_t s) {
    const bool vec = a.c % 4 == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(a.y) & 15) == 0;
    if (vec)
        pool_kernel<4><<<grid_for(a.M * (a.c / 4)), 256, 0, s>>>(a);
    else
        pool_kernel<1><<<grid_for(a.M * a.c), 256, 0, s>>>(a);
    return 1;
}


int launch_mean(const MeanArgs &a, cudaStream_t s) {
    int threads = 256;
    int rows = a.c <= threads ? threads / a.c : 0;
    size_t smem = rows ? sizeof(double) * rows * a.c : 0;
    mean_partial_kernel<<<dim3(a.chunks, a.nl), threads, smem, s>>>(a);
    mean_final_kernel<<<dim3((a.c + 31) / 32, a.nl), 1024, 0, s>>>(a);
    return 2;
}

int launch_layernorm(const LayerNormArgs &a, cudaStream_t s) {
    if (a.fast && a.c <= 512)
        layernorm_fast_kernel<<<(a.pixels + 7) / 8, 256, 0, s>>>(a);
    else
        layernorm_kernel<<<(a.pixels + 3) / 4, 128, sizeof(float) * 4 * a.c, s>>>(a);
    return 1;
}

bool attention_supported(int t, int c, int heads) {
    int hd = c / heads;
    return hd <= 64 && (size_t)2 * t * hd * sizeof(float) <= 160 * 1024;
}

int launch_attention(const AttentionArgs &a, cudaStream_t s) {
    int hd = a.c / a.heads;
    size_t smem = sizeof(float) * 2 * a.tmax * hd;
    dim3 grid(unsigned(a.nl * a.heads), unsigned((a.tmax + ATT_Q - 1) / ATT_Q));
    const size_t fast_smem = sizeof(float) * 2 * a.tmax * ATT_ROW;
    if (hd == 15 && a.fast && fast_smem <= 160 * 1024) {
        dim3 fgrid(unsigned(a.nl * a.heads), unsigned((a.tmax + ATT_FAST_Q - 1) / ATT_FAST_Q));
        attention_fast_kernel<15><<<fgrid, ATT_FAST_Q * 8, fast_smem, s>>>(a);
    } else if (hd == 15)  // PP-OCRv6's 8 heads of 15 (tools/export_ocr.py:654)
        attention_kernel<15><<<grid, ATT_Q, smem, s>>>(a);
    else
        attention_kernel<0><<<grid, ATT_Q, smem, s>>>(a);
    return 1;
}

int ctc_col_blocks(int cols) { return (cols + CTC_COLS - 1) / CTC_COLS; }

bool ctc_supported(int ci) { return (size_t)ci * (CTC_PX + CTC_COLS) * sizeof(float) <= 200 * 1024; }

void configure_misc_kernels() {
    cudaFuncSetAttribute(ctc_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    // K and V of one lane and head (attention_supported: at most 160 KB)
    cudaFuncSetAttribute(attention_kernel<15>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    cudaFuncSetAttribute(attention_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    cudaFuncSetAttribute(attention_fast_kernel<15>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
}

int launch_ctc(const CtcArgs &a, cudaStream_t s) {
    dim3 grid((a.pixels + CTC_PX - 1) / CTC_PX, a.col_blocks);
    size_t smem = sizeof(float) * (size_t)a.ci * (CTC_PX + CTC_COLS);
    ctc_logits_kernel<<<grid, CTC_THREADS, smem, s>>>(a);
    ctc_merge_kernel<<<(a.pixels + 127) / 128, 128, 0, s>>>(a);
    return 2;
}

// A 2x2 transposed conv to one channel (the DB head's last layer): one
// thread per input pixel, its channels read as float4s, the 4 x ic weights
// in shared memory, the same sums in the same order as convt_kernel; the
// 2x2 output block leaves as two float2 stores.
__global__ void __launch_bounds__(256) convt_2x2x1_kernel(const ConvTArgs a) {
    __shared__ __align__(16) float ws[256 * 4];
    for (int e = threadIdx.x; e < a.ic * 4; e += blockDim.x) ws[e] = __ldg(a.w + e);
    __syncthreads();
    float bias[4];
#pragma unroll
    for (int j = 0; j < 4; j++) bias[j] = a.b ? __ldg(a.b + j) : 0.0f;
    for (long pix = (long)blockIdx.x * blockDim.x + threadIdx.x; pix < a.Min; pix += (long)gridDim.x * blockDim.x) {
        const float4 *x = reinterpret_cast<const float4 *>(a.x + pix * a.ic);
        float acc[4];
#pragma unroll
        for (int j = 0; j < 4; j++) acc[j] = a.bias_first ? bias[j] : 0.0f;
        for (int i4 = 0; i4 < a.ic / 4; i4++) {
            const float4 xv = __ldg(x + i4);
            const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const float4 w = *reinterpret_cast<const float4 *>(ws + (4 * i4 + u) * 4);
                acc[0] = ffma(w.x, xs[u], acc[0]);
                acc[1] = ffma(w.y, xs[u], acc[1]);
                acc[2] = ffma(w.z, xs[u], acc[2]);
                acc[3] = ffma(w.w, xs[u], acc[3]);
            }
        }
        const LaneInfo &L = a.lanes[a.nl > 1 ? find_lane(a.lanes, a.nl, pix, true) : 0];
        const int iw = __ldg(&L.iw), ow = iw * 2;
        const int r = int(pix - __ldg(&L.ipix0));
        const int iy = r / iw, ix = r - iy * iw;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            v[j] = acc[j];
            if (a.b && !a.bias_first) v[j] = fadd(v[j], bias[j]);
            v[j] = activate(a.act, v[j]);
        }
        float *y = a.y + __ldg(&L.pix0) + (long)(2 * iy) * ow + 2 * ix;
        *reinterpret_cast<float2 *>(y) = make_float2(v[0], v[1]);       // ky = 0: kx = 0, 1
        *reinterpret_cast<float2 *>(y + ow) = make_float2(v[2], v[3]);  // ky = 1
    }
}

int launch_convt(const ConvTArgs &a, cudaStream_t s) {
    const auto aligned = [](const void *p, int n) { return (reinterpret_cast<uintptr_t>(p) & (n - 1)) == 0; };
    if (a.kh == 2 && a.kw == 2 && a.oc == 1 && a.ic % 4 == 0 && a.ic <= 256 && aligned(a.x, 16) &&
        aligned(a.y, 8)) {
        convt_2x2x1_kernel<<<grid_for(a.Min), 256, 0, s>>>(a);
        return 1;
    }
    int cols = a.kh * a.kw * a.oc;
    long total = a.Min * ((cols + 3) / 4);
    convt_kernel<<<grid_for(total), 256, 0, s>>>(a);
    return 1;
}

}  // namespace ppocr
