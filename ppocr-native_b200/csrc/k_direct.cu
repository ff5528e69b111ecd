// Windowed dense convolution straight from a shared-memory halo tile
// (sm_100a, FP32 pipes): the detector's 3x3 neck and head convolutions and
// the RGB stems.
//
// A block computes TR output rows x 128 output columns of one lane, for all
// `oc` output channels (24 per warp group). It stages the input window those
// outputs read — (TR-1)*sh + kh rows x 127*sw + kw columns — one chunk of CH
// channels at a time in shared memory, with the chunk's weights, and every
// tap then reads its A values from there instead of gathering them from
// global memory. Each lane owns 4 pixels of a row (x = lane + 32 i) and 24
// output channels: per (tap, channel) 4 shared loads of A and 6 broadcast
// float4 loads of B feed 96 fused multiply-adds.
//
// Order of each output's sum: channel chunks in order, within a chunk the
// taps in kernel row-major order, within a tap the chunk's channels in order,
// one FMA each. When the input has at most CH channels (every stem, every
// recogniser layer) that is exactly the reference's order, tap-major then
// channel (`kernels/dense.rs:104-141`), and the bits match; wider inputs (the
// detector's 96-channel 3x3 layers) differ from it by rounding only.
//
// Up to four sources, each read nearest-upsampled by 2^shift, make the
// channels (the neck's upsample + concat, never written out); padding and
// the window's overhang read zero.
#include "devmath.cuh"
#include "kernels.hpp"

namespace ppocr {

namespace {

constexpr int TW = 128;  // output columns per block
constexpr int OCG = 24;  // output channels per warp group

struct DirectShape {
    int tr;  // output rows per block
    int ch;  // channels per chunk
};

__host__ __device__ inline DirectShape direct_shape(int oc, int C, int sh) {
    DirectShape d;
    d.tr = oc == 24 ? 8 : 4;  // 256 threads either way
    d.ch = C <= 4 ? C : (sh == 1 ? 16 : 8);
    return d;
}

// Floats of the halo chunk, rounded up so that the weights after it start on
// a 16-byte boundary (they are read as float4).
__host__ __device__ inline size_t halo_floats(int hr, int hw, int chp) {
    return ((size_t)hr * hw * chp + 3) / 4 * 4;
}

// Shared floats of one block: the halo chunk (channel stride ch | 1, odd, so
// neighbouring pixels fall in different banks) and the chunk's weights.
__host__ __device__ inline size_t direct_smem(int oc, int C, int kh, int kw, int sh, int sw) {
    DirectShape d = direct_shape(oc, C, sh);
    int hr = (d.tr - 1) * sh + kh, hw = (TW - 1) * sw + kw;
    int chp = d.ch | 1;
    return sizeof(float) * (halo_floats(hr, hw, chp) + (size_t)kh * kw * d.ch * oc);
}

template <int NG>  // output channel groups of 24
__global__ void __launch_bounds__(256) conv_direct_kernel(const ConvArgs a) {
    extern __shared__ __align__(16) float smem[];
    const DirectShape d = direct_shape(a.oc, a.C, a.sh);
    const int TR = d.tr, CH = d.ch, CHP = CH | 1;
    const int HR = (TR - 1) * a.sh + a.kh, HW = (TW - 1) * a.sw + a.kw;
    float *halo = smem;                          // [HR][HW][CHP]
    float *Ws = smem + halo_floats(HR, HW, CHP); // [kh*kw][CH][oc]

    // This block's lane and output tile.
    const long tile = blockIdx.x;
    int n = 0;
    {
        int lo = 0, hi = a.nl - 1;
        while (lo < hi) {
            int mid = (lo + hi + 1) >> 1;
            if (__ldg(&a.lanes[mid].tile0) <= tile) lo = mid; else hi = mid - 1;
        }
        n = lo;
    }
    const LaneInfo &L = a.lanes[n];
    const int ih = __ldg(&L.ih), iw = __ldg(&L.iw), oh = __ldg(&L.oh), ow = __ldg(&L.ow);
    const int tiles_x = (ow + TW - 1) / TW;
    const int t = int(tile - __ldg(&L.tile0));
    const int oy0 = (t / tiles_x) * TR, ox0 = (t % tiles_x) * TW;
    const int iy0 = oy0 * a.sh - a.pt, ix0 = ox0 * a.sw - a.pl;

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int g = warp % NG;       // output channel group
    const int r = warp / NG;       // output row within the tile
    const int oy = oy0 + r;
    const int taps = a.kh * a.kw;

    // Accumulators of 4 pixels x 24 channels, bias first where due.
    float acc[4][OCG];
    bool first[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        int ox = ox0 + lane + 32 * i;
        bool f = a.bias_mode == BIAS_FIRST;
        if (a.bias_mode == BIAS_FIRST_BUT_ROW_TAIL) f = ox < ow - ow % 4;
        first[i] = f;
#pragma unroll
        for (int j = 0; j < OCG; j++) acc[i][j] = (f && a.b) ? __ldg(a.b + g * OCG + j) : 0.0f;
    }

    const int nthreads = blockDim.x;
    for (int c0 = 0; c0 < a.C; c0 += CH) {
        const int cn = min(CH, a.C - c0);
        __syncthreads();  // the previous chunk is no longer read
        // Halo chunk: pixel (hy, hx) of the window, channels c0 .. c0+cn.
        for (int e = threadIdx.x; e < HR * HW * cn; e += nthreads) {
            int c = e % cn, p = e / cn;
            int hy = p / HW, hx = p - hy * HW;
            int iy = iy0 + hy, ix = ix0 + hx;
            float v = 0.0f;
            if (iy >= 0 && iy < ih && ix >= 0 && ix < iw) {
                int cc = c0 + c, start = 0, s = 0;
                while (s + 1 < a.nsrc && cc >= start + a.src[s].c) { start += a.src[s].c; s++; }
                const ConvSource &src = a.src[s];
                int sh = src.shift;
                long off = (__ldg(&L.spix0[s]) + (long)(iy >> sh) * (iw >> sh) + (ix >> sh)) * src.c + (cc - start);
                v = __ldg(src.p + off);
            }
            halo[(size_t)p * CHP + c] = v;
        }
        // Weights of the chunk: [tap][c][oc].
        for (int e = threadIdx.x; e < taps * cn * a.oc; e += nthreads) {
            int o = e % a.oc, rest = e / a.oc;
            int c = rest % cn, tap = rest / cn;
            Ws[((size_t)tap * CH + c) * a.oc + o] = __ldg(a.w + ((long)tap * a.C + c0 + c) * a.oc + o);
        }
        __syncthreads();
        if (oy < oh) {
            for (int tap = 0; tap < taps; tap++) {
                const int ky = tap / a.kw, kx = tap - ky * a.kw;
                const float *hrow = halo + ((size_t)(r * a.sh + ky) * HW + kx) * CHP;
                const float *wrow = Ws + (size_t)tap * CH * a.oc + g * OCG;
                for (int c = 0; c < cn; c++) {
                    float av[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) av[i] = hrow[(size_t)((lane + 32 * i) * a.sw) * CHP + c];
                    const float4 *wv = reinterpret_cast<const float4 *>(wrow + (size_t)c * a.oc);
#pragma unroll
                    for (int q = 0; q < OCG / 4; q++) {
                        float4 b = wv[q];
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            acc[i][4 * q + 0] = ffma(b.x, av[i], acc[i][4 * q + 0]);
                            acc[i][4 * q + 1] = ffma(b.y, av[i], acc[i][4 * q + 1]);
                            acc[i][4 * q + 2] = ffma(b.z, av[i], acc[i][4 * q + 2]);
                            acc[i][4 * q + 3] = ffma(b.w, av[i], acc[i][4 * q + 3]);
                        }
                    }
                }
            }
        }
    }
    if (oy >= oh) return;
    const long prow = __ldg(&L.pix0) + (long)oy * ow;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        int ox = ox0 + lane + 32 * i;
        if (ox >= ow) continue;
        long m = prow + ox;
        float *y = a.y + m * a.oc + g * OCG;
        const float *res = a.res ? a.res + m * a.oc + g * OCG : nullptr;
#pragma unroll
        for (int q = 0; q < OCG / 4; q++) {
            float v[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                int j = 4 * q + e;
                float x = acc[i][j];
                if (!first[i] && a.b) x = fadd(x, __ldg(a.b + g * OCG + j));
                x = activate(a.act, x);
                if (res) x = activate(a.act2, fadd(x, __ldg(res + j)));
                v[e] = x;
            }
            *reinterpret_cast<float4 *>(y + 4 * q) = make_float4(v[0], v[1], v[2], v[3]);
        }
    }
}

}  // namespace

bool conv_direct_supported(const ConvArgs &a) {
    // Only the RGB stems for now: their three channels fit one chunk, so the
    // order (and the bits) stay the reference's; wider inputs run faster as
    // the implicit GEMM of k_conv.cu.
    if (a.C > 4) return false;
    if (a.oc != 24 && a.oc != 48) return false;
    if (a.gate || a.kh * a.kw < 2 || a.kh > 7 || a.kw > 7 || a.sh > 2 || a.sw > 2) return false;
    return direct_smem(a.oc, a.C, a.kh, a.kw, a.sh, a.sw) <= 200 * 1024;
}

int conv_direct_rows(const ConvArgs &a) { return direct_shape(a.oc, a.C, a.sh).tr; }
int conv_direct_cols() { return TW; }

void configure_direct_kernels() {
    cudaFuncSetAttribute(conv_direct_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(conv_direct_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
}

int launch_conv_direct(const ConvArgs &a, long tiles, cudaStream_t s) {
    size_t smem = direct_smem(a.oc, a.C, a.kh, a.kw, a.sh, a.sw);
    if (a.oc == 24)
        conv_direct_kernel<1><<<(unsigned)tiles, 256, smem, s>>>(a);
    else
        conv_direct_kernel<2><<<(unsigned)tiles, 256, smem, s>>>(a);
    return 1;
}

}  // namespace ppocr
