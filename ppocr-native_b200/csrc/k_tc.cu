// Convolutions on the 5th-generation tensor cores (sm_100a, tcgen05) in
// 3xTF32: y = act2(act(conv(x) + b) + res) over packed pixels, as an
// implicit GEMM with M = output pixels, N = output channels and
// K = kh*kw*C (k = (ky*kw + kx)*C + c, the weights' [kh][kw][C][oc] order).
//
// Each product is split into tf32 halves, x = xh + xl and w = wh + wl, and
// three MMAs accumulate xh wh + xh wl + xl wh in FP32 in tensor memory, which
// keeps the result within a few units of the FP32 one (the dropped xl wl
// term is 2^-22 of the product). The weights arrive already split, [n][kpad]
// (K-major), high halves then low halves; the pixels are split on chip.
//
// Both kernels are persistent and warp-specialised. Output channels are cut
// into S slices of BN (a multiple of 32, at most 256); CTA b owns slice
// b % S and walks the 128-pixel tiles q, q + Q, q + 2Q, ... with q = b / S,
// so the S CTAs working on one tile do so at about the same time and all but
// the first read it from L2. K advances 32 channels (one 128-byte swizzle
// row of f32) per stage through a ring of `ns` stages:
//   producer    one thread fills a stage's A block (128 pixels x 32 k,
//               16 KB) with one TMA copy: for pw_tc_kernel (1x1 layers) from
//               the packed input, whose pixels are the output's; for
//               conv_tc_kernel (stride-1 windowed layers whose output keeps
//               the input's size, C % 32 == 0) the block of tap (ky, kx) and
//               channels c0..c0+31 is the 128 packed input pixels starting
//               (ky - pt) * iw + kx - pl after the tile's first, each lane
//               tiled on its own;
//   converter   splits the block in place into its high half and a low-half
//               twin (multiplying by the lane's SE gate first, if any; for a
//               windowed layer, zeroing the rows whose tap falls outside the
//               image);
//   MMA         one thread issues the MMAs into one of two TMEM accumulators
//               and commits each stage back to the producer and each finished
//               tile to the epilogue;
//   epilogue    8 warps: warp w drains TMEM lanes 32(w%4)..+31, 16 columns at
//               a time (the two warps of a lane quadrant take alternate
//               chunks), adds the bias, applies the activation (one
//               instantiation per code, no branch per element), adds the
//               residual if any, and stores: rows of at most 48 channels
//               straight from each lane's registers (16-byte stores), wider
//               ones transposed through shared memory into coalesced rows.
// pw_tc_kernel keeps its slice's weights (all of K, both halves) resident in
// shared memory; conv_tc_kernel, whose K runs to kh*kw*C, streams them with
// the A blocks (one TMA copy per stage, from L2).
//
// Every wait on an mbarrier is bounded (globaltimer) and sleeps in the
// barrier rather than spinning. A wait that runs out records a code in `err`
// (page-locked host memory the runtime reads after the run) and raises an
// abort flag in shared memory that ends every role's loop; the producers then
// wait, bounded, for the copies they issued, the MMA thread for its last
// commit, and the tensor memory is freed before return.
#include <cuda.h>

#include <algorithm>
#include <cfloat>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "tc.cuh"

namespace ppocr {

namespace {

// Warp roles of both kernels: producer 0, MMA 1, converters 2-9, epilogue
// 10-17.
struct Roles {
    static constexpr int W_MMA = 1, W_CONV = 2, W_EPI = W_CONV + CONV_THREADS / 32;
    static constexpr int THREADS = (W_EPI + EPI_WARPS) * 32;
};


// The MMA thread. The weights of K block kb sit at b_base (resident) or in
// the stage beside the A block (streamed).
template <bool RESIDENT>
__device__ void role_mma(const TcArgs &a, const Ctx &x, uint64_t *bfull) {
    const uint32_t idesc = tf32_idesc(x.BN);
    long job = 0;
    int s = 0;        // ring stage
    uint32_t ph = 0;  // parity of this stage's current round
    uint32_t last_bar = 0, last_parity = 0;
    bool ok = !RESIDENT || wait_phase(smem_u32(bfull), 0, x.abort_flag, a.err);
    for (long t = x.first; t < x.tiles && ok; t += x.Q, job++) {
        const int buf = int(job & 1);
        const long use = job >> 1;
        if (use > 0 && !wait_phase(smem_u32(&x.acce[buf]), uint32_t(use - 1) & 1u, x.abort_flag, a.err)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = x.tmem + uint32_t(buf * x.BN);
        for (int kb = 0; kb < x.nkb; kb++) {
            if (!wait_phase(smem_u32(&x.conv[s]), ph, x.abort_flag, a.err)) {
                ok = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            // A: the converters' split halves in this slot's TMEM stage
            const uint32_t ah = x.tmem + uint32_t(a_col0(x.BN) + s * 64), al = ah + 32;
            uint32_t bh, bl;
            if (RESIDENT) {
                bh = x.b_base + uint32_t(kb) * x.b_bytes;
                bl = x.b_base + uint32_t(x.nkb + kb) * x.b_bytes;
            } else {
                bh = x.ring + uint32_t(s) * x.stage_bytes + SLOT_BYTES;
                bl = bh + x.b_bytes;
            }
            // K steps of 8 tf32: 8 TMEM columns of A, 32 bytes along B's
            // swizzled rows (+2 in the descriptor's address field, which stays
            // below 2^14 for any shared address); steps wholly past K hold
            // zeros and are skipped
            const int left = a.K - kb * TK;
            const int steps = left >= TK ? TK / 8 : (left + 7) / 8;
            const uint64_t dbh = sw128_desc(bh), dbl = sw128_desc(bl);
#pragma unroll
            for (int kk = 0; kk < TK / 8; kk++) {
                if (kk >= steps) break;
                const uint64_t step = uint64_t(2 * kk);
                const uint32_t col = uint32_t(8 * kk);
                mma_tf32_ta(d, ah + col, dbh + step, idesc, (kb | kk) ? 1u : 0u);
                mma_tf32_ta(d, ah + col, dbl + step, idesc, 1u);
                mma_tf32_ta(d, al + col, dbh + step, idesc, 1u);
            }
            commit(smem_u32(&x.empty[s]));
            last_bar = smem_u32(&x.empty[s]);
            last_parity = ph;
            if (++s == x.ns) {
                s = 0;
                ph ^= 1u;
            }
        }
        if (!ok) break;
        commit(smem_u32(&x.accf[buf]));
        last_bar = smem_u32(&x.accf[buf]);
        last_parity = uint32_t(use) & 1u;
    }
    // the tensor core is done with shared memory and TMEM before the CTA
    // frees them
    if (last_bar) drain(last_bar, last_parity, WAIT_LIMIT_NS);
}

// The converters (8 warps, ct = 0..255): split each landed A block into its
// high tf32 half and the remainder, after the SE gate when there is one, and
// store both into the slot's TMEM stage. Warp w owns TMEM lane quadrant w % 4
// (32 pixels, one per thread) and K columns 16 h .. 16 h + 15 of the block,
// h = (w - first converter warp) / 4: the thread reads those 16 values of its
// pixel's 128-byte swizzled row. For a windowed layer each row's taps that
// fall inside the image are found once per tile (a bit per tap) and the
// others zeroed.
__device__ void role_convert(const TcArgs &a, const Ctx &x, int ct, int warp, int lane) {
    const int qd = warp & 3, h = ct / 128;
    // this thread's row (pixel) of every tile, and the staged row it reads:
    // with folded taps, quadrant qd holds tile pixels 30 qd - 1 .. 30 qd + 30
    // (staged from pixel -1 on)
    const int r = a.fold ? qd * (32 - 2) + lane - 1 : qd * 32 + lane;
    const int srow = a.fold ? r + 1 : r;
    const int cblocks = a.C / TK;  // windowed: K blocks per tap
    const int taps = a.fold ? a.kh : a.kh * a.kw;
    const uint32_t tlane = uint32_t(qd * 32) << 16;
    int s = 0;         // ring stage
    uint32_t ph = 0;   // parity of this stage's current round
    int gi = 0;        // verdict slot
    bool ok = true;
    for (long t = x.first; t < x.tiles && ok; t += x.Q) {
        int gl = -1;           // the row's lane, for the gate
        uint32_t inside = 0;   // windowed: bit k set when tap k of the row reads the image
        if (a.gate) {
            const long m = t * TM + r;
            gl = m < a.M ? find_lane(a.lanes, a.nl, m) : -1;
        }
        if (a.windowed) {
            const TileInfo ti = tile_info(a, t);
            const LaneInfo &L = a.lanes[ti.n];
            const int ow = __ldg(&L.ow), ih = __ldg(&L.ih), iw = __ldg(&L.iw);
            const long q = ti.q0 + r;
            if (a.fold && q >= 0 && q < long(__ldg(&L.oh)) * ow) {
                // rows whose vertical tap falls inside the image
                const int oy = int(q / ow);
                for (int k = 0; k < taps && k < 32; k++)
                    if ((unsigned)(oy + k - a.pt) < (unsigned)ih) inside |= 1u << k;
            } else if (!a.fold && r < ti.rows) {
                const int oy = int(q / ow), ox = int(q - long(oy) * ow);
                for (int k = 0; k < taps && k < 32; k++) {
                    const int ky = k / a.kw, kx = k - ky * a.kw;
                    if ((unsigned)(oy + ky - a.pt) < (unsigned)ih && (unsigned)(ox + kx - a.pl) < (unsigned)iw)
                        inside |= 1u << k;
                }
            }
        }
        int tap = 0, cb = 0;  // windowed: the K block's tap and channel block
        for (int kb = 0; kb < x.nkb; kb++) {
            // one thread polls the stage, the others wait in the named
            // barrier (ordered after its acquire of the landed bytes)
            if (ct == 0) x.go_conv[gi] = wait_phase(smem_u32(&x.full[s]), ph, x.abort_flag, a.err);
            named_sync(BAR_CONV, CONV_THREADS);
            if (!x.go_conv[gi]) {
                ok = false;
                break;
            }
            gi ^= 1;
            const uint32_t row = x.ring + uint32_t(s) * x.stage_bytes + uint32_t(srow) * 128;
            const bool zero = a.windowed && !(inside & (1u << tap));
            float hv[16], lv[16];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int lc = 4 * h + q;  // logical 16-byte chunk: k = kb*32 + 4 lc .. + 3
                float4 v = lds4(row + uint32_t(((lc ^ (srow & 7)) << 4)));
                if (a.gate) {
                    const int k = kb * TK + 4 * lc;
                    float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (gl >= 0 && k < a.K) g = __ldg(reinterpret_cast<const float4 *>(a.gate + (long)gl * a.K + k));
                    v = make_float4(fmul(v.x, g.x), fmul(v.y, g.y), fmul(v.z, g.z), fmul(v.w, g.w));
                }
                if (zero) v = make_float4(0.f, 0.f, 0.f, 0.f);
                const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    hv[4 * q + u] = tf32_hi(e[u]);
                    lv[4 * q + u] = e[u] - hv[4 * q + u];
                }
            }
            const uint32_t col = uint32_t(a_col0(x.BN) + s * 64 + 16 * h);
            tmem_st16(x.tmem + tlane + col, hv);
            tmem_st16(x.tmem + tlane + col + 32, lv);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) arrive(smem_u32(&x.conv[s]));  // one arrival per warp
            if (++s == x.ns) {
                s = 0;
                ph ^= 1u;
            }
            if (++cb == cblocks) {
                cb = 0;
                tap++;
            }
        }
    }
}

// The epilogue of a conv with folded horizontal taps: lane i of quadrant qd
// holds tile pixel p = 30 qd + i - 1 and, per output channel, its products
// with the taps kx = 0, 1, 2 (columns 48 j + 16 kx + e). Output p sums its
// own kx = 1 column, its left neighbour's kx = 0 and its right neighbour's
// kx = 2 (adjacent lanes, by shuffles), skipping a neighbour outside the
// image row, then adds the bias and applies the activation; lanes 1..30 of
// each quadrant are the tile's outputs. Stores go through the same swizzled
// transpose as the plain epilogue.
template <int ACT>
__device__ void role_epilogue_fold(const TcArgs &a, const Ctx &x, int e, int warp, int lane, uint32_t staging,
                                   const float *bias_s) {
    const int qd = warp & 3;
    const int half = e / 4;
    const uint32_t stg = staging + uint32_t(e * STAGE_FLOATS * 4);
    const int q4 = lane & 3;
    const bool vec = (a.toc & 3) == 0;
    const int chunks = x.BN / 48;
    long job = 0;
    for (long t = x.first; t < x.tiles; t += x.Q, job++) {
        const int buf = int(job & 1);
        if (e == 0 && lane == 0)
            x.go_epi[job & 1] = wait_phase<true>(smem_u32(&x.accf[buf]), uint32_t(job >> 1) & 1u, x.abort_flag, a.err);
        named_sync(BAR_EPI, EPI_WARPS * 32);
        if (!x.go_epi[job & 1]) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const TileInfo ti = tile_info(a, t);
        const int ow = __ldg(&a.lanes[ti.n].ow);
        const int p = qd * 30 + lane - 1;  // this lane's tile pixel
        const long q = ti.q0 + p;
        const int ox = q >= 0 ? int(q % ow) : 0;
        const bool has_l = ox > 0, has_r = ox < ow - 1;
        const long mq = ti.m0 + qd * 30 - 1;  // packed pixel of lane 0
        const int last = ti.rows - qd * 30;  // lanes 1..last are outputs (at most 30)
        for (int ch = half; ch < chunks; ch += 2) {
            float z0[16], z1[16], z2[16];
            const uint32_t col = x.tmem + (uint32_t(qd * 32) << 16) + uint32_t(buf * x.BN + ch * 48);
            tmem_ld16(col, z0);
            tmem_ld16(col + 16, z1);
            tmem_ld16(col + 32, z2);
#pragma unroll
            for (int c = 0; c < 4; c++) {
                float o[4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int j = 4 * c + u;
                    const float l = __shfl_up_sync(0xffffffffu, z0[j], 1);
                    const float r = __shfl_down_sync(0xffffffffu, z2[j], 1);
                    float v = z1[j];
                    if (has_l) v = fadd(l, v);
                    if (has_r) v = fadd(v, r);
                    o[u] = activate_t<ACT, true>(fadd(v, bias_s[ch * 16 + j]));
                }
                sts4(stg + uint32_t(lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4)), make_float4(o[0], o[1], o[2], o[3]));
            }
            __syncwarp();
            const int n = x.n0 / 3 + ch * 16 + 4 * q4;  // output channel
#pragma unroll
            for (int pp = 0; pp < 4; pp++) {
                const int rr = 8 * pp + (lane >> 2);
                float4 o = lds4(stg + uint32_t(rr * 64 + ((q4 ^ ((rr >> 1) & 3)) << 4)));
                if (rr < 1 || rr > 30 || rr > last || n >= a.toc) continue;
                const long m = mq + rr;
                float *dst = a.y + m * a.toc + n;
                if (vec) {
                    if (a.res) {
                        const float4 rv = __ldg(reinterpret_cast<const float4 *>(a.res + m * a.toc + n));
                        o = make_float4(activate(a.act2, fadd(o.x, rv.x)), activate(a.act2, fadd(o.y, rv.y)),
                                        activate(a.act2, fadd(o.z, rv.z)), activate(a.act2, fadd(o.w, rv.w)));
                    }
                    *reinterpret_cast<float4 *>(dst) = o;
                } else {
                    const float ov[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        if (n + c >= a.toc) break;
                        float y = ov[c];
                        if (a.res) y = activate(a.act2, fadd(y, __ldg(a.res + m * a.toc + n + c)));
                        dst[c] = y;
                    }
                }
            }
            __syncwarp();
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) arrive(smem_u32(&x.acce[buf]));  // one arrival per warp
    }
}

template <int ACT, int MODE = EPI_PLAIN>
__global__ void __launch_bounds__(Roles::THREADS, 1)
    pw_tc_kernel(const TcArgs a, const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw) {
    using R = Roles;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    __shared__ __align__(8) uint64_t full[MAX_NS], conv[MAX_NS], empty[MAX_NS], accf[2], acce[2], bfull;
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s, go_conv_s[2], go_epi_s[2];

    Ctx x;
    x.go_conv = go_conv_s;
    x.go_epi = go_epi_s;
    x.ns = a.ns; x.nkb = a.nkb; x.BN = a.bn;
    x.Q = gridDim.x / a.slices;
    x.first = blockIdx.x / a.slices;
    x.n0 = int(blockIdx.x % a.slices) * a.bn;
    x.tiles = (a.M + TM - 1) / TM;
    x.ring = smem_u32(smem);
    x.stage_bytes = SLOT_BYTES;
    x.b_base = x.ring + uint32_t(x.ns) * SLOT_BYTES;
    x.b_bytes = uint32_t(a.bn) * 128;
    x.full = full; x.conv = conv; x.empty = empty; x.accf = accf; x.acce = acce;
    x.abort_flag = &abort_s;
    float *staging = reinterpret_cast<float *>(smem + size_t(x.ns) * SLOT_BYTES + size_t(2) * x.nkb * x.b_bytes);
    float *bias_s = staging + EPI_WARPS * STAGE_FLOATS;  // this slice's BN biases, zero past N
    setup<R>(a, x, 1, &bfull, bias_s, &tmem_base_s, &abort_s);

    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    if (warp == 0) {
        if (lane == 0) {
            // the weight slice: nkb blocks of BN rows, high halves then low
            const uint32_t bb = smem_u32(&bfull);
            arrive_expect(bb, uint32_t(2 * x.nkb) * x.b_bytes);
            for (int kb = 0; kb < x.nkb; kb++) {
                tma_load_3d(x.b_base + uint32_t(kb) * x.b_bytes, &tmw, kb * TK, x.n0, 0, bb);
                tma_load_3d(x.b_base + uint32_t(x.nkb + kb) * x.b_bytes, &tmw, kb * TK, x.n0, 1, bb);
            }
            long it = 0;  // K blocks issued
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (long t = x.first; t < x.tiles && ok; t += x.Q)
                for (int kb = 0; kb < x.nkb; kb++, it++) {
                    // the stage's previous round was read by the MMAs
                    if (it >= x.ns && !wait_phase(smem_u32(&empty[s]), ph ^ 1u, x.abort_flag, a.err)) {
                        ok = false;
                        break;
                    }
                    arrive_expect(smem_u32(&full[s]), A_BYTES);
                    tma_load_2d(x.ring + uint32_t(s) * SLOT_BYTES, &tmx, kb * TK, int(t * TM), smem_u32(&full[s]));
                    if (++s == x.ns) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            if (*x.abort_flag) {
                // the copies still in flight land before the CTA leaves
                drain(bb, 0, WAIT_LIMIT_NS);
                for (int q = 0; q < x.ns && q < it; q++)
                    drain(smem_u32(&full[q]), uint32_t((it - 1 - q) / x.ns) & 1u, WAIT_LIMIT_NS);
            }
        }
    } else if (warp == R::W_MMA) {
        if (lane == 0) role_mma<true>(a, x, &bfull);
    } else if (warp < R::W_EPI) {
        role_convert(a, x, tid - R::W_CONV * 32, warp, lane);
    } else {
        role_epilogue<ACT, MODE>(a, x, warp - R::W_EPI, warp, lane, smem_u32(staging), bias_s);
    }
    teardown<R>(a, x);
}

template <int ACT, int MODE = EPI_PLAIN>
__global__ void __launch_bounds__(Roles::THREADS, 1)
    conv_tc_kernel(const TcArgs a, const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw) {
    using R = Roles;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    __shared__ __align__(8) uint64_t full[MAX_NS], conv[MAX_NS], empty[MAX_NS], accf[2], acce[2], bfull;
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s, go_conv_s[2], go_epi_s[2];

    Ctx x;
    x.go_conv = go_conv_s;
    x.go_epi = go_epi_s;
    x.ns = a.ns; x.nkb = a.nkb; x.BN = a.bn;
    x.Q = gridDim.x / a.slices;
    x.first = blockIdx.x / a.slices;
    x.n0 = int(blockIdx.x % a.slices) * a.bn;
    x.tiles = a.windowed ? a.tiles : (a.M + TM - 1) / TM;
    x.ring = smem_u32(smem);
    x.b_bytes = uint32_t(a.bn) * 128;
    x.stage_bytes = SLOT_BYTES + 2 * x.b_bytes;
    x.b_base = 0;
    x.full = full; x.conv = conv; x.empty = empty; x.accf = accf; x.acce = acce;
    x.abort_flag = &abort_s;
    float *staging = reinterpret_cast<float *>(smem + size_t(x.ns) * x.stage_bytes);
    float *bias_s = staging + EPI_WARPS * STAGE_FLOATS;
    setup<R>(a, x, 1, &bfull, bias_s, &tmem_base_s, &abort_s);

    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    if (warp == 0) {
        if (lane == 0) {
            const int cblocks = a.windowed ? a.C / TK : x.nkb;  // K blocks per tap
            long it = 0;
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (long t = x.first; t < x.tiles && ok; t += x.Q) {
                const TileInfo ti = tile_info(a, t);
                long base = ti.m0;  // a 1x1 layer's packed input is its output's
                int iw = 0;
                if (a.windowed) {
                    const LaneInfo &L = a.lanes[ti.n];
                    base = __ldg(&L.ipix0) + ti.q0;
                    iw = __ldg(&L.iw);
                }
                int cb = 0, ky = 0, kx = 0;  // the K block's channel block and tap
                for (int kb = 0; kb < x.nkb; kb++, it++) {
                    if (it >= x.ns && !wait_phase(smem_u32(&empty[s]), ph ^ 1u, x.abort_flag, a.err)) {
                        ok = false;
                        break;
                    }
                    const int c0 = cb * TK;
                    // rows before the first pixel or past the last read as
                    // zeros; rows of another lane are zeroed by the converters
                    const long y = base + long(ky - a.pt) * iw + (kx - a.pl);
                    const uint32_t stage = x.ring + uint32_t(s) * x.stage_bytes;
                    const uint32_t bar = smem_u32(&full[s]);
                    arrive_expect(bar, A_BYTES + 2 * x.b_bytes);
                    tma_load_2d(stage, &tmx, c0, int(y), bar);
                    tma_load_3d(stage + SLOT_BYTES, &tmw, kb * TK, x.n0, 0, bar);
                    tma_load_3d(stage + SLOT_BYTES + x.b_bytes, &tmw, kb * TK, x.n0, 1, bar);
                    if (++s == x.ns) {
                        s = 0;
                        ph ^= 1u;
                    }
                    if (++cb == cblocks) {
                        cb = 0;
                        // folded taps: the K blocks walk the vertical taps
                        // only, each staged from the tile's pixel -1 on
                        if (a.fold || ++kx == a.kw) {
                            kx = 0;
                            ky++;
                        }
                    }
                }
            }
            if (*x.abort_flag)
                // the copies still in flight land before the CTA leaves
                for (int q = 0; q < x.ns && q < it; q++)
                    drain(smem_u32(&full[q]), uint32_t((it - 1 - q) / x.ns) & 1u, WAIT_LIMIT_NS);
        }
    } else if (warp == R::W_MMA) {
        if (lane == 0) role_mma<false>(a, x, &bfull);
    } else if (warp < R::W_EPI) {
        role_convert(a, x, tid - R::W_CONV * 32, warp, lane);
    } else if constexpr (MODE == EPI_FOLD) {
        role_epilogue_fold<ACT>(a, x, warp - R::W_EPI, warp, lane, smem_u32(staging), bias_s);
    } else {
        role_epilogue<ACT, MODE>(a, x, warp - R::W_EPI, warp, lane, smem_u32(staging), bias_s);
    }
    teardown<R>(a, x);
}

// One warp per row: the blocks' (max, sum, first column) merge in a fixed
// order; then every block within the margin of the row's maximum has its 16
// x (bn / 32) columns recomputed exactly, lanes two columns each.
__global__ void __launch_bounds__(256) ctc_tc_merge_kernel(const CtcMergeArgs a) {
    extern __shared__ float xrow[];  // [8 warps][ci]: each warp's input row
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const long t = (long)blockIdx.x * 8 + warp;
    if (t >= a.pixels) return;
    float *xs = xrow + warp * a.ci;
    for (int k = lane; k < a.ci; k += 32) xs[k] = __ldg(a.x + t * a.ci + k);
    __syncwarp();
    const float *st = a.partial + t * a.blocks * 3;
    float m = -FLT_MAX;
    for (int b = lane; b < a.blocks; b += 32) m = fmaxf(m, st[b * 3]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    float sum = 0.0f;
    for (int b = lane; b < a.blocks; b += 32)
        if (st[b * 3] > -FLT_MAX) sum = fadd(sum, fmul(st[b * 3 + 1], __expf(fsub(st[b * 3], m))));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float o = __shfl_xor_sync(0xffffffffu, sum, off);
        sum = (lane & off) ? fadd(o, sum) : fadd(sum, o);  // the same order in both lanes
    }
    // The margin: twice a bound on |tensor-core logit - FP32 logit|. Each
    // sum of k products, |w_k x_k| <= wmax |x_k|, carries at most 3k + 8
    // roundings of 2^-23 relative in either form (three products per k on
    // the tensor core, the dropped low-low term, the bias), so
    // 2 * 2 * (3k + 8) * 2^-23 * (wmax * sum|x| + bmax) covers both errors.
    float ax = 0.0f;
    for (int k = lane; k < a.ci; k += 32) ax += fabsf(xs[k]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ax += __shfl_xor_sync(0xffffffffu, ax, off);
    const float margin = 4.0f * float(3 * a.ci + 8) * 1.1920929e-7f * (ax * a.wmax + a.bmax) * 1.01f;
    float best_v = -FLT_MAX;
    int best = 0x7fffffff;
    for (int b0 = 0; b0 < a.blocks; b0 += 32) {
        const int b = b0 + lane;
        unsigned cand = __ballot_sync(0xffffffffu, b < a.blocks && st[b * 3] >= m - margin);
        while (cand) {
            const int bb = b0 + __ffs(cand) - 1;
            cand &= cand - 1;
            const int slice = bb / 2, half = bb % 2;
            for (int q = lane; q < a.bn / 2; q += 32) {
                const int col = slice * a.bn + half * 16 + (q / 16) * 32 + (q % 16);
                if (col >= a.vocab) continue;
                float acc = __ldg(a.b + col);
                const float *wc = a.w + (long)(col >> 4) * a.ci * 16 + (col & 15);
                // eight weights in flight, then their terms in k order
                for (int k0 = 0; k0 < a.ci; k0 += 8) {
                    float wv[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) wv[j] = k0 + j < a.ci ? __ldg(wc + (k0 + j) * 16) : 0.0f;
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        if (k0 + j < a.ci) acc = ffma(wv[j], xs[k0 + j], acc);
                }
                if (acc > best_v || (acc == best_v && col < best)) {
                    best_v = acc;
                    best = col;
                }
            }
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, best_v, off);
        const int c2 = __shfl_xor_sync(0xffffffffu, best, off);
        if (v2 > best_v || (v2 == best_v && c2 < best)) {
            best_v = v2;
            best = c2;
        }
    }
    if (lane == 0) {
        a.y[2 * t] = float(best);
        a.y[2 * t + 1] = fdiv(1.0f, sum);
    }
}

size_t pw_smem(int kpad, int bn, int ns) { return 1024 + size_t(ns) * SLOT_BYTES + size_t(8) * kpad * bn + EPI_BYTES; }

size_t conv_smem(int bn, int ns) { return 1024 + size_t(ns) * (SLOT_BYTES + size_t(256) * bn) + EPI_BYTES; }

// Ring stages: as many as shared memory and the TMEM A stages allow.
int max_stages(int bn) { return tmem_stages(bn) < MAX_NS ? tmem_stages(bn) : MAX_NS; }

// The weight slice width for a pointwise K x N: the fewest slices of at
// most 256 channels (a multiple of 32) whose weights, both halves, fit in
// shared memory beside a three-stage ring (else a two-stage one). 0 when
// none does.
int pw_slice_width(int K, int N) {
    const int kpad = (K + TK - 1) / TK * TK;
    for (int stages = 3; stages >= 2; stages--)
        for (int S = 1; S <= (N + 31) / 32; S++) {
            const int bn = ((N + S - 1) / S + 31) / 32 * 32;
            if (bn <= 128 && pw_smem(kpad, bn, stages) <= size_t(DYN_CEILING)) return bn;
        }
    return 0;
}

// The streaming kernel's slice: as wide as a three-stage ring allows (at
// most 128).
int conv_slice_width(int N) {
    for (int S = 1; S <= (N + 31) / 32; S++) {
        const int bn = ((N + S - 1) / S + 31) / 32 * 32;
        if (bn <= 128 && conv_smem(bn, 3) <= size_t(DYN_CEILING)) return bn;
    }
    return 0;
}

bool set_grid(TcArgs &a) {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
        return false;
    const long tiles = a.windowed ? a.tiles : (a.M + TM - 1) / TM;
    const long per = std::max(1, a.min_tiles);
    const long q = std::max(1L, std::min(long(sms / a.slices), (tiles + per - 1) / per));
    a.grid = int(q) * a.slices;
    a.tmem_cols = TMEM_COLS;
    return true;
}

}  // namespace

int pw_tc_kpad(int K) { return (K + TK - 1) / TK * TK; }

bool tc_weights_wanted(int K, int N) { return K >= 1 && N >= 1 && N <= 512; }

bool tc_prepare(TcArgs &a) {
    if (a.M < 1 || a.N < 1 || a.K < 1 || a.kpad != pw_tc_kpad(a.K)) return false;
    const auto aligned = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!aligned(a.w_hi) || a.w_lo != a.w_hi + size_t(a.N) * a.kpad) return false;
    EncodeTiled enc = encode_tiled();
    if (!enc) return false;
    a.nkb = a.kpad / TK;
    if (a.C % 4 || !aligned(a.x) || (a.gate && !aligned(a.gate))) return false;
    if (a.vocab > 0 && (a.windowed || a.act || a.res || a.gate || !a.partial)) return false;
    if (a.tkh) {
        // the scattering epilogue lives in the streaming kernel; its stores
        // are 16-byte runs of one tap's channels
        if (a.windowed || a.res || a.gate || a.vocab || a.N != a.tkh * a.tkw * a.toc || a.toc % 4) return false;
        a.stream_b = true;
    }
    if (a.fold) {
        // three horizontal taps (pl = 1) in 48-column groups of 16 outputs
        if (!a.windowed || a.kw != 3 || a.pl != 1 || a.K != a.kh * a.C || a.N % 48 || a.toc < 1 ||
            a.toc > a.N / 3)
            return false;
    }
    if (a.windowed) {
        // a tap's K blocks never straddle taps; the output keeps the input's
        // size, so the packed input has M pixels too
        if (a.gate || a.C % TK || a.tiles < 1 || (!a.fold && a.K != a.kh * a.kw * a.C) || a.kh * a.kw > 32)
            return false;
    } else {
        // 1x1: the packed input is [M][K]; its weights stay resident unless
        // streaming them takes fewer slices
        if (a.K != a.C || a.kh * a.kw != 1) return false;
        if (!a.stream_b) {
            const int bn = pw_slice_width(a.K, a.N);
            const int streamed = tc_stream_slices(a.N);
            if (streamed > 0 && (!bn || streamed < (a.N + bn - 1) / bn)) a.stream_b = true;
            if (!bn && !a.stream_b) return false;
        }
    }
    if (!a.windowed && !a.stream_b) {
        a.bn = pw_slice_width(a.K, a.N);
        a.slices = (a.N + a.bn - 1) / a.bn;
        a.ns = 2;
        while (a.ns < max_stages(a.bn) && pw_smem(a.kpad, a.bn, a.ns + 1) <= size_t(DYN_CEILING)) a.ns++;
        a.smem = int(pw_smem(a.kpad, a.bn, a.ns));
    } else if (a.fold) {
        // two 16-channel groups per slice, one when few tiles
        a.bn = a.N >= 96 && (a.min_tiles > 1 || a.tiles * ((a.N + 95) / 96) >= 74) ? 96 : 48;
        a.slices = a.N / a.bn + (a.N % a.bn ? 1 : 0);
        a.ns = 2;
        while (a.ns < max_stages(a.bn) && conv_smem(a.bn, a.ns + 1) <= size_t(DYN_CEILING)) a.ns++;
        a.smem = int(conv_smem(a.bn, a.ns));
    } else {
        a.bn = conv_slice_width(a.N);
        if (!a.bn) return false;
        // few tiles: narrower slices, so that more SMs share the layer (each
        // output's sum is the same whatever the slice). Not for the CTC
        // head: its per-block softmax sums group the columns by slice, so the
        // slice width must depend on the head alone, never on how many time
        // steps the run holds (a lane then reads the same alone as beside
        // others).
        const long tiles = a.windowed ? a.tiles : (a.M + TM - 1) / TM;
        while (a.vocab == 0 && a.min_tiles <= 1 && a.bn > 32 && tiles * ((a.N + a.bn - 1) / a.bn) < 74) a.bn -= 32;
        a.slices = (a.N + a.bn - 1) / a.bn;
        a.ns = 2;
        while (a.ns < max_stages(a.bn) && conv_smem(a.bn, a.ns + 1) <= size_t(DYN_CEILING)) a.ns++;
        a.smem = int(conv_smem(a.bn, a.ns));
    }
    // pixels: [M][C], boxes of 32 channels x 128 pixels; channels past C and
    // pixels outside the buffer read as zeros
    CUtensorMap mx;
    cuuint64_t dims[2] = {cuuint64_t(a.C), cuuint64_t(a.M)};
    cuuint64_t strides[1] = {cuuint64_t(a.C) * 4};
    cuuint32_t box[2] = {TK, TM}, estr[2] = {1, 1};
    if (enc(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(a.x), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    std::memcpy(a.tmx, &mx, sizeof mx);
    a.blocks = 2 * a.slices;
    return encode_weights(a, enc) && set_grid(a);
}

int launch_ctc_tc_merge(const CtcMergeArgs &a, cudaStream_t s) {
    ctc_tc_merge_kernel<<<unsigned((a.pixels + 7) / 8), 256, sizeof(float) * 8 * a.ci, s>>>(a);
    return 1;
}

int tc_stream_slices(int N) {
    const int bn = conv_slice_width(N);
    return bn ? (N + bn - 1) / bn : 0;
}

int tc_pointwise_slices(int K, int N) {
    // set_grid's choice for a 1x1 layer: resident weights unless streaming
    // them takes fewer slices
    const int bn = pw_slice_width(K, N);
    const int streamed = tc_stream_slices(N);
    if (streamed > 0 && (!bn || streamed < (N + bn - 1) / bn)) return streamed;
    return bn ? (N + bn - 1) / bn : 0;
}

template <int ACT>
void configure_act() {
    cudaFuncSetAttribute(pw_tc_kernel<ACT>, cudaFuncAttributeMaxDynamicSharedMemorySize, DYN_CEILING);
    cudaFuncSetAttribute(conv_tc_kernel<ACT>, cudaFuncAttributeMaxDynamicSharedMemorySize, DYN_CEILING);
    cudaFuncSetAttribute(conv_tc_kernel<ACT, EPI_CONVT>, cudaFuncAttributeMaxDynamicSharedMemorySize, DYN_CEILING);
    cudaFuncSetAttribute(conv_tc_kernel<ACT, EPI_FOLD>, cudaFuncAttributeMaxDynamicSharedMemorySize, DYN_CEILING);
}

void configure_tc_kernels() {
    cudaFuncSetAttribute(conv_tc_kernel<0, EPI_CTC>, cudaFuncAttributeMaxDynamicSharedMemorySize, DYN_CEILING);
    cudaFuncSetAttribute(pw_tc_kernel<0, EPI_CTC>, cudaFuncAttributeMaxDynamicSharedMemorySize, DYN_CEILING);
    configure_act<0>(); configure_act<1>(); configure_act<2>(); configure_act<3>();
    configure_act<4>(); configure_act<5>(); configure_act<6>(); configure_act<7>();
}

template <int ACT>
void launch_act(const TcArgs &a, const CUtensorMap &mx, const CUtensorMap &mw, cudaStream_t s) {
    if (a.vocab > 0 && a.stream_b)
        conv_tc_kernel<0, EPI_CTC><<<a.grid, Roles::THREADS, a.smem, s>>>(a, mx, mw);
    else if (a.vocab > 0)
        pw_tc_kernel<0, EPI_CTC><<<a.grid, Roles::THREADS, a.smem, s>>>(a, mx, mw);
    else if (a.tkh)
        conv_tc_kernel<ACT, EPI_CONVT><<<a.grid, Roles::THREADS, a.smem, s>>>(a, mx, mw);
    else if (a.fold)
        conv_tc_kernel<ACT, EPI_FOLD><<<a.grid, Roles::THREADS, a.smem, s>>>(a, mx, mw);
    else if (a.windowed || a.stream_b)
        conv_tc_kernel<ACT><<<a.grid, Roles::THREADS, a.smem, s>>>(a, mx, mw);
    else
        pw_tc_kernel<ACT><<<a.grid, Roles::THREADS, a.smem, s>>>(a, mx, mw);
}

int launch_tc(const TcArgs &a, cudaStream_t s) {
    CUtensorMap mx, mw;
    std::memcpy(&mx, a.tmx, sizeof mx);
    std::memcpy(&mw, a.tmw, sizeof mw);
    switch (a.act) {
    case 1: launch_act<1>(a, mx, mw, s); break;
    case 2: launch_act<2>(a, mx, mw, s); break;
    case 3: launch_act<3>(a, mx, mw, s); break;
    case 4: launch_act<4>(a, mx, mw, s); break;
    case 5: launch_act<5>(a, mx, mw, s); break;
    case 6: launch_act<6>(a, mx, mw, s); break;
    case 7: launch_act<7>(a, mx, mw, s); break;
    default: launch_act<0>(a, mx, mw, s); break;
    }
    return 1;
}

}  // namespace ppocr
