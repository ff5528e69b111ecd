// Launch arguments and entry points of every CUDA kernel of the backend.
// Shared by the host runtime (model.cpp) and the kernels (*.cu).
//
// Tensors are NHWC f32. The lanes of one run (images of any sizes) are packed
// back to back pixel by pixel, so a pixelwise operation sees one array of
// M = sum of the lanes' pixels; an operation that needs a pixel's lane and
// coordinates finds them in its lane table (LaneInfo), one entry per lane
// with the prefix sums of the lanes' pixel counts.
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

namespace ppocr {

// Where a convolution adds its bias (the reference's tier-3 tiles decide it,
// see Model::bias_mode): before the taps, after them, or before them except
// on the last `ow % 4` pixels of each output row.
enum BiasMode : int { BIAS_FIRST = 0, BIAS_LAST = 1, BIAS_FIRST_BUT_ROW_TAIL = 2 };

// One input of a dense convolution: `c` channels of an image 2^shift times
// smaller than the convolution's input along both axes, read as if
// nearest-upsampled (the neck's upsample + concat, never written out;
// reference `src/engine/kernels/dense.rs:7-19`).
struct ConvSource {
    const float *p = nullptr;
    int c = 0;
    int shift = 0;
};

constexpr int MAX_SOURCES = 4;

// One lane of one operation: where its pixels start in the packed output,
// input and (per source, or the second input) tensors, and its sizes.
struct LaneInfo {
    long pix0;                // first output pixel
    long ipix0;               // first input pixel
    long spix0[MAX_SOURCES];  // first pixel in each conv source / the second input
    long tile0;               // first 128-pixel output tile when every lane is tiled on its own
    long run0;                // first DW_RUN-pixel run along an output row (depthwise threads)
    long ftile0;              // first FOLD_OUT-pixel tile of a tensor-core conv with folded taps
    long row0;                // first output row (rows of all lanes back to back)
    int ih, iw, oh, ow;
};

#ifdef __CUDACC__
// The lane holding packed pixel m: the last whose `pix0` (or `ipix0` when
// `input`) is at most m.
__device__ __forceinline__ int find_lane(const LaneInfo *L, int nl, long m, bool input = false) {
    int lo = 0, hi = nl - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        long start = input ? __ldg(&L[mid].ipix0) : __ldg(&L[mid].pix0);
        if (start <= m)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}

// The lane holding output row `r` (LaneInfo::row0).
__device__ __forceinline__ int find_row_lane(const LaneInfo *L, int nl, long r) {
    int lo = 0, hi = nl - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (__ldg(&L[mid].row0) <= r)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}

// The lane holding row run `r` (LaneInfo::run0).
__device__ __forceinline__ int find_run_lane(const LaneInfo *L, int nl, long r) {
    int lo = 0, hi = nl - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (__ldg(&L[mid].run0) <= r)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}
#endif

struct ConvArgs {
    ConvSource src[MAX_SOURCES];
    int nsrc = 1;
    int C = 0;                 // channels of all sources together
    const float *w = nullptr;  // [kh][kw][C][oc]
    const float *b = nullptr;  // [oc] or null
    float *y = nullptr;        // [M][oc]
    const LaneInfo *lanes = nullptr;
    int nl = 1;                // lanes
    long M = 0;                // output pixels of all lanes
    int oc = 0;
    int kh = 1, kw = 1, sh = 1, sw = 1, pt = 0, pl = 0;
    int act = 0;
    int bias_mode = BIAS_FIRST;
    const float *gate = nullptr;  // [lanes][C]: input channel c of lane n is x * gate[n][c]
    const float *res = nullptr;   // [M][oc]: y = act2(act(conv) + res)
    int act2 = 0;
    bool quick = false;           // stems: the activation's quick quotient (tensor-core mode)
    long out_rows = 0;            // output rows of all lanes (LaneInfo::row0)
    int max_ow = 0;               // the widest lane's output width
};

// Output pixels along one row that a depthwise thread computes together.
constexpr int DW_RUN = 4;

struct DwArgs {
    const float *x = nullptr;  // packed input, c channels
    const float *w = nullptr;  // [kh][kw][c]
    const float *b = nullptr;  // [c] or null
    float *y = nullptr;        // [M][c]
    const LaneInfo *lanes = nullptr;
    int nl = 1;
    long M = 0;
    int c = 0;
    int kh = 3, kw = 3, sh = 1, sw = 1, pt = 0, pl = 0;
    int act = 0;
    bool quick = false;        // the activation's quick quotient (tensor-core mode)
    long runs = 0;             // DW_RUN-pixel row runs over all lanes (LaneInfo::run0)
};

// Depthwise convolution whose output feeds a pointwise one straight from
// shared memory.
struct DwPwArgs {
    DwArgs dw;                  // dw.y unused
    const float *w2 = nullptr;  // [c][oc]
    const float *b2 = nullptr;  // [oc] or null
    float *y = nullptr;         // [M][oc]
    int oc = 0;
    int act2 = 0;
    int bias_mode2 = BIAS_FIRST;
    const float *res = nullptr;  // optional residual, y = act3(act2(pw) + res)
    int act3 = 0;
    // Row tiles of the fused tile kernel (dwpw_tile): output rows of all
    // lanes (LaneInfo::row0) times segments of each row.
    long rows = 0;
    int segs = 0;
};

enum EltMode : int {
    ELT_ADD = 0,        // y = act(x + x2)
    ELT_CHANNELMUL,     // y = x * g[n][c]
    ELT_GATE_ADD,       // y = act(x * g[n][c] + x)
    ELT_UPSAMPLE,       // y[r][c] = x[r/sh][c/sw]
    ELT_UPSAMPLE_ADD,   // y = x2 + upsample(x)
    ELT_CONCAT,         // y = [x | x2] per pixel
    ELT_GATE_UPSAMPLE_ADD,  // y = act(x2 * g[n][c] + x2) + upsample(x)
};

struct EltArgs {
    int mode = ELT_ADD;
    const float *x = nullptr, *x2 = nullptr;
    const float *g = nullptr;  // ELT_GATE_UPSAMPLE_ADD: the gate, [lanes][c]
    float *y = nullptr;
    const LaneInfo *lanes = nullptr;  // gates and upsampling
    int nl = 1;
    long M = 0;  // output pixels
    int c = 0, c2 = 0;
    int sh = 1, sw = 1;
    int act = 0;
};

struct PoolArgs {
    const float *x = nullptr;
    float *y = nullptr;
    const LaneInfo *lanes = nullptr;
    int nl = 1;
    long M = 0;
    int c = 0, kh = 1, kw = 1, sh = 1, sw = 1;
    bool average = false;
};

struct MeanArgs {
    const float *x = nullptr;  // packed input, c channels
    float *y = nullptr;        // [lanes][c]
    double *partial = nullptr; // [lanes][chunks][c] scratch
    const LaneInfo *lanes = nullptr;
    int nl = 1, c = 0, chunks = 1;
};

struct LayerNormArgs {
    const float *x = nullptr, *w = nullptr;  // w = [gamma | beta | eps]
    float *y = nullptr;
    int pixels = 0, c = 0;
    bool fast = false;  // tensor-core mode: the sums by warp-parallel reductions (another order)
};

struct AttentionArgs {
    const float *x = nullptr;  // packed [t][3c] per lane
    float *y = nullptr;        // packed [t][c] per lane
    const float *scale = nullptr;
    const LaneInfo *lanes = nullptr;  // t of lane n = lanes[n].iw
    int nl = 1, tmax = 0, c = 0, heads = 1;
    bool fast = false;  // tensor-core mode: eight threads per query, __expf, any order
};

// CTC head over `cols` = 16 * ceil(vocab / 16) panel columns: each block
// reduces a range of columns to a (max, sum of exp, best column) state per
// pixel in `partial`; the merge turns them into the output.
struct CtcArgs {
    const float *x = nullptr;  // [pixels][ci]
    const float *w = nullptr;  // [cols/16][ci][16]
    const float *b = nullptr;  // [cols]
    float *y = nullptr;        // argmax: [pixels][2]; probs: [pixels][vocab]
    float *partial = nullptr;  // [pixels][col_blocks][3]
    int pixels = 0, ci = 0, vocab = 0, cols = 0, col_blocks = 0;
    bool probs = false;
};

struct ConvTArgs {
    const float *x = nullptr;  // packed input, ic channels
    const float *w = nullptr;  // [ic][kh][kw][oc]
    const float *b = nullptr;  // [kh*kw*oc] or null
    float *y = nullptr;        // packed output, oc channels
    const LaneInfo *lanes = nullptr;
    int nl = 1;
    long Min = 0;              // input pixels of all lanes
    int ic = 0, oc = 0, kh = 2, kw = 2;
    int act = 0;
    bool bias_first = true;
};

// Pointwise convolution on the tensor cores (k_tc.cu), 3xTF32: weights
// pre-split and transposed to [n][kpad] (K-major, zero-padded to 32
// channels and to whole BN tiles of output channels).
// A convolution on the tensor cores (3xTF32), its input read with TMA.
// Pointwise layers (1x1, unit stride) take 128 packed pixels per tile.
// Windowed ones (`windowed`: unit stride, output the input's size, C % 32
// == 0) tile each lane on its own, so that a tap's 128 input pixels are 128
// consecutive packed pixels shifted by (ky - pt) * iw + kx - pl; the rows
// that fall outside the image read as zeros.
// Output pixels per tile of a tensor-core 3-wide conv with its horizontal
// taps folded into N: four 32-lane quadrants of 30 outputs, each quadrant's
// first and last lane holding the neighbours' sums.
constexpr int FOLD_OUT = 120;

struct TcArgs {
    bool windowed = false;
    // A windowed conv of kw = 3, pl = 1 with its three horizontal taps folded
    // into the columns: K = kh * C (k = ky * C + c), N = 48 per 16 output
    // channels (column 48 j + 16 kx + e is channel 16 j + e of tap kx), toc
    // the output channels; tiles of FOLD_OUT outputs (LaneInfo::ftile0).
    bool fold = false;
    bool stream_b = false;        // weights streamed with the A blocks even for a 1x1 layer
    const float *x = nullptr;     // [pixels][C], 16-byte aligned, C % 4 == 0
    long tiles = 0;               // windowed: 128-pixel tiles of all lanes, each lane on its own
    int C = 0;
    int kh = 1, kw = 1, pt = 0, pl = 0;
    const LaneInfo *lanes = nullptr;
    int nl = 1;
    const float *gate = nullptr;  // pointwise: [lanes][K], x of lane n scaled by gate[n] first
    const float *w_hi = nullptr;  // [N][kpad]: high tf32 halves, K-major
    const float *w_lo = nullptr;  // w_hi + N * kpad: the low halves
    const float *b = nullptr;     // [N] or null
    const float *res = nullptr;   // [M][N] or null
    float *y = nullptr;           // [M][N]
    long M = 0;
    int K = 0, N = 0, kpad = 0;   // K = kh * kw * C
    int act = 0, act2 = 0;
    int *err = nullptr;           // set to nonzero when a bounded wait gave up
    // Tiles each CTA takes at least: above 1 a small layer occupies few SMs
    // (other runs in flight use the rest) instead of spreading one tile per
    // SM, and slices are not narrowed for few tiles. Each output's sum is the
    // same whatever the grid and the slices.
    int min_tiles = 1;
    // A CTC argmax head (vocab > 0, 1x1, weights resident or streamed): no
    // y; per row and column block, (max, sum of exp(logit - max), 0) over
    // the block's columns below vocab, into partial [M][blocks][3]. Block
    // 2s + h holds columns s*bn + h*16 + 32j + e (e < 16) of slice s.
    int vocab = 0;
    float *partial = nullptr;
    int blocks = 0;               // filled: 2 * slices
    // A non-overlapping transposed conv (tkh > 0): rows are input pixels
    // (lanes by ipix0), column n = (ky * tkw + kx) * toc + o goes to output
    // pixel (iy * tkh + ky, ix * tkw + kx) of the lane (pix0, ow), channel o.
    // toc is also a folded conv's output channel count.
    int tkh = 0, tkw = 0, toc = 0;
    // filled by tc_prepare: output-channel slice width and count, K blocks,
    // ring stages, TMEM columns, grid, dynamic shared memory, and the tensor
    // maps (CUtensorMap, 128 bytes each) of the input and of the weights
    int bn = 0, slices = 0, nkb = 0, ns = 0, tmem_cols = 0, grid = 0, smem = 0;
    unsigned long long tmx[16] = {}, tmw[16] = {};
};
int launch_tc(const TcArgs &a, cudaStream_t s);
// Slices of the output channels a streamed-weight launch of N channels uses.
int tc_stream_slices(int N);
// Slices a 1x1 K x N layer takes on the tensor cores (resident or streamed
// weights, whichever takes fewer); 0 when neither fits.
int tc_pointwise_slices(int K, int N);

// The CTC argmax head's merge after its tensor-core logits: per row, the
// blocks' maxima and sums combine into 1 / sum exp(logit - max); every
// block whose maximum lies within `margin` of the row's (a bound on the
// tensor-core logits' error, twice over) has its logits recomputed in FP32
// in the reference's order (bias, then k increasing, one FMA each), so the
// class is the reference's first column of the maximum, bit for bit.
struct CtcMergeArgs {
    const float *partial = nullptr;  // [pixels][blocks][3]
    int blocks = 0, bn = 0;
    const float *x = nullptr;        // [pixels][ci]
    const float *w = nullptr;        // [cols/16][ci][16]
    const float *b = nullptr;        // [cols]
    float *y = nullptr;              // [pixels][2]
    int pixels = 0, ci = 0, vocab = 0;
    float wmax = 0.f, bmax = 0.f;    // largest |w| and |b| over the columns below vocab
};
int launch_ctc_tc_merge(const CtcMergeArgs &a, cudaStream_t s);

// The input a multi-source convolution reads, written out: per pixel of the
// conv's input size, the sources' channels side by side, each source read
// nearest-upsampled by 2^shift (a copy, so any layer reading it sees the
// same values the fused reads would).
struct GatherArgs {
    ConvSource src[MAX_SOURCES];
    int nsrc = 1, C = 0;
    const LaneInfo *lanes = nullptr;  // the conv's: ipix0, spix0, ih, iw
    int nl = 1;
    long M = 0;                       // input pixels of all lanes
    float *y = nullptr;               // [M][C]
};
int launch_gather(const GatherArgs &a, cudaStream_t s);
// Whether a K x N layer gets split tensor-core weights at load.
bool tc_weights_wanted(int K, int N);
// The padded K of the prepared weights (a multiple of 32).
int pw_tc_kpad(int K);
// Fills the launch shape and tensor maps; false when the layer cannot run
// there (alignment, sizes, no driver entry point).
bool tc_prepare(TcArgs &a);
void configure_tc_kernels();

// Each returns the number of kernels it launched.
int launch_conv(const ConvArgs &a, cudaStream_t s);
// A pointwise layer over per-lane vectors (one pixel per lane, one source),
// bit-identical to launch_conv; supported while its weights' 32-column slice
// and the vectors fit in shared memory.
int launch_conv_vector(const ConvArgs &a, cudaStream_t s);
bool conv_vector_supported(const ConvArgs &a);
int launch_dw(const DwArgs &a, cudaStream_t s);
int launch_dw_pw(const DwPwArgs &a, cudaStream_t s);
int launch_elt(const EltArgs &a, cudaStream_t s);
int launch_pool(const PoolArgs &a, cudaStream_t s);
int launch_mean(const MeanArgs &a, cudaStream_t s);
int launch_layernorm(const LayerNormArgs &a, cudaStream_t s);
int launch_attention(const AttentionArgs &a, cudaStream_t s);
int launch_ctc(const CtcArgs &a, cudaStream_t s);
int launch_convt(const ConvTArgs &a, cudaStream_t s);

// Per-device set-up (shared-memory ceilings); call with the device current.
void configure_dw_kernels();
void configure_conv_kernels();
void configure_misc_kernels();
bool ctc_supported(int ci);

// Output pixels under which a depthwise layer and the pointwise one it feeds
// run as two kernels (depthwise, then a small-tile pointwise GEMM over the
// map, which stays in L2) rather than fused: small maps give the fused
// kernel's 128-pixel tiles too few blocks for 148 SMs.
constexpr long DW_PW_MIN_PIXELS = 148L * 2 * 128;

// Scratch sizes (elements) the launches above need.
// Pixel runs a lane's channel mean is split into; a lane's result depends
// only on its own size, never on the other lanes of the run.
// Runs hold about 8192 values (a power of two of pixels, 16..2048), so a
// block has a few dozen loads per thread whatever the channel count.
__host__ __device__ inline int mean_chunks(long hw, int c) {
    int per = 16;
    while (per < 2048 && per * 2 * c <= 8192) per *= 2;
    long chunks = (hw + per - 1) / per;
    return int(chunks < 1 ? 1 : (chunks > 16384 ? 16384 : chunks));
}
int ctc_col_blocks(int cols);
// Largest shared-memory need of launch_dw_pw for `c` input channels; 0 when
// that kernel cannot take them.
bool dw_pw_supported(const DwPwArgs &a);
// The fused depthwise -> pointwise tile kernel for narrow layers (c of 24,
// 48 or 96 channels into oc of 24, 48, 96 or 192, 3x3 or 5x5, stride 1 or
// 2): whether it takes the layer, the pixels of one tile (segments of a
// row), and the launch (quick: the tensor-core mode's activation quotient).
bool dwpw_tile_supported(const DwPwArgs &a);
int dwpw_tile_pixels(const DwPwArgs &a);
int launch_dwpw_tile(const DwPwArgs &a, bool quick, cudaStream_t s);
bool attention_supported(int t, int c, int heads);

}  // namespace ppocr
