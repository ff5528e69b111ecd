// Shared pieces of the tensor-core kernels (sm_100a, tcgen05, 3xTF32): tile
// and ring constants, descriptors, bounded mbarrier waits, TMEM access, the
// epilogue role, the CTA set-up and tear-down, and the host's tensor-map
// encoding. Every kernel that includes this keeps its own copy (an unnamed
// namespace per translation unit).
#pragma once

#include <cuda.h>

#include <cfloat>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "async.cuh"
#include "devmath.cuh"
#include "kernels.hpp"

namespace ppocr {

namespace {

constexpr int TM = 128;                   // pixels per tile (MMA M, one TMEM lane each)
constexpr int TK = 32;                    // k per block: one 128-byte swizzle row of f32
constexpr int A_BYTES = TM * 128;         // one half of an A block
constexpr int SLOT_BYTES = A_BYTES;       // the staged A block (its split halves go to TMEM)
constexpr int EPI_WARPS = 8;
constexpr int STAGE_FLOATS = 32 * 16;     // one epilogue warp's 32 x 16 transpose tile (swizzled)
constexpr int EPI_BYTES = EPI_WARPS * STAGE_FLOATS * 4 + 256 * 4;  // + the bias slice
constexpr int MAX_NS = 8;
// Tensor memory: all 512 columns; the two accumulators (BN columns each)
// first, then one 64-column stage per ring slot for the split A block (high
// half in its first 32 columns, low half in the next 32), one lane per pixel.
constexpr int TMEM_COLS = 512;
__host__ __device__ constexpr int a_col0(int bn) { return (2 * bn + 63) / 64 * 64; }
__host__ __device__ constexpr int tmem_stages(int bn) { return (TMEM_COLS - a_col0(bn)) / 64; }
// Dynamic shared memory per CTA: the block's limit (227 KB) less room for the
// kernels' static shared memory.
constexpr int DYN_CEILING = 226 * 1024;
// How long one wait on an mbarrier may take before the kernel gives up: a
// K block's copy or MMAs take microseconds.
constexpr unsigned long long WAIT_LIMIT_NS = 200ull * 1000 * 1000;
// How long a waiting thread may stay suspended in an mbarrier before it
// looks at the abort flag and the time limit again.
constexpr uint32_t WAIT_SLEEP_NS = 20000;
// Threads of the converter role (arrivals on a stage's `conv` barrier: one
// per warp).
constexpr int CONV_THREADS = 256;

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SM100 layout: start >> 4 in [0,14), leading offset
// [16,30) unused for swizzled K-major (1), stride offset >> 4 in [32,46),
// version 1 in [46,48), layout type 2 in [61,64)).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    uint64_t d = 0;
    d |= uint64_t((addr >> 4) & 0x3FFF);
    d |= uint64_t(1) << 16;
    d |= uint64_t(1024 >> 4) << 32;
    d |= uint64_t(1) << 46;
    d |= uint64_t(2) << 61;
    return d;
}

// Instruction descriptor of kind::tf32: D f32, A and B tf32, both K-major,
// M = 128, N = n.
__host__ __device__ constexpr uint32_t tf32_idesc(int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(TM >> 4) << 24);
}

// One MMA with A in tensor memory (lanes = rows, one tf32 per column) and B
// in shared memory; acc 0 overwrites D.
__device__ __forceinline__ void mma_tf32_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}\n"
        :
        : "r"(d_tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}


// Waits for the phase of `bar` with this parity to complete. Gives up when
// another role raised the abort flag, or after the time limit (then raises
// it and records the error). The waiting thread stays suspended in the
// barrier between looks (longer with BACKOFF: a wait expected to be long, a
// tile's accumulator).
template <bool BACKOFF = false>
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile int *abort_flag, int *err) {
    if (try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
        // suspended in the barrier (at most WAIT_SLEEP_NS a round) rather
        // than polling: the roles on the critical path keep the issue slots
        if (try_wait_sleep(bar, parity, BACKOFF ? WAIT_SLEEP_NS : WAIT_SLEEP_NS / 4)) return true;
        if (*abort_flag) return false;
        if (global_ns() - t0 > WAIT_LIMIT_NS) {
            *abort_flag = 1;
            if (err) atomicExch(err, 1);
            return false;
        }
    }
}


// A named barrier among `count` threads (a multiple of 32): the threads
// that wait there issue nothing.
__device__ __forceinline__ void named_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
constexpr int BAR_CONV = 1, BAR_EPI = 2;

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float v[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float4 lds4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

__device__ __forceinline__ void sts4(uint32_t addr, float4 v) {
    asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float v[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
        : "memory");
}

__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

// Where tile t's 128 rows land: output pixels m0..m0+rows-1 of lane n,
// from the lane's own pixel q0 on.
struct TileInfo {
    long m0, q0;
    int rows, n;
};

__device__ __forceinline__ TileInfo tile_info(const TcArgs &a, long t) {
    TileInfo ti;
    if (!a.windowed) {
        ti.m0 = ti.q0 = t * TM;
        ti.rows = int(a.M - ti.m0 < TM ? a.M - ti.m0 : TM);
        ti.n = 0;
        return ti;
    }
    int lo = 0, hi = a.nl - 1;  // the last lane whose first tile is at most t
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if ((a.fold ? __ldg(&a.lanes[mid].ftile0) : __ldg(&a.lanes[mid].tile0)) <= t)
            lo = mid;
        else
            hi = mid - 1;
    }
    const LaneInfo &L = a.lanes[lo];
    const int per = a.fold ? FOLD_OUT : TM;
    ti.n = lo;
    ti.q0 = (t - (a.fold ? __ldg(&L.ftile0) : __ldg(&L.tile0))) * per;
    ti.m0 = __ldg(&L.pix0) + ti.q0;
    const long left = long(__ldg(&L.oh)) * __ldg(&L.ow) - ti.q0;
    ti.rows = int(left < per ? left : per);
    return ti;
}

// What every role of one CTA shares.
struct Ctx {
    uint32_t ring;         // shared address of stage 0
    uint32_t stage_bytes;  // one stage: the A block's two halves (+ the B block's when streamed)
    uint32_t b_base;       // resident weights (pw_tc_kernel)
    uint32_t b_bytes;      // one K block of one half of the weight slice: BN x 128 bytes
    uint64_t *full, *conv, *empty, *accf, *acce;
    volatile int *abort_flag;
    // the converters' and the epilogue's polling thread's verdicts, two
    // slots each (alternate rounds), read by the others after the named
    // barrier: 1 go on, 0 stop
    volatile int *go_conv, *go_epi;
    int ns, nkb, BN, n0, Q;
    long first, tiles;
    uint32_t tmem;
};

// Epilogue modes: the plain store, the CTC argmax partials, a transposed
// conv's scattered store, a folded conv's sum of its three horizontal taps.
enum EpiMode : int { EPI_PLAIN = 0, EPI_CTC = 1, EPI_CONVT = 2, EPI_FOLD = 3 };

template <int ACT, int MODE>
__device__ void role_epilogue(const TcArgs &a, const Ctx &x, int e, int warp, int lane, uint32_t staging,
                              const float *bias_s) {
    const int qd = warp & 3;  // the TMEM lane quadrant this warp may read
    const int half = e / 4;   // which alternate 16-column chunks it takes
    const uint32_t stg = staging + uint32_t(e * STAGE_FLOATS * 4);
    const int q = lane & 3;   // read-back chunk of this lane
    const bool vec = (a.N & 3) == 0 && (MODE != EPI_CONVT || (a.toc & 3) == 0);
    long job = 0;
    for (long t = x.first; t < x.tiles; t += x.Q, job++) {
        const int buf = int(job & 1);
        // one thread polls the accumulator (sleeping between polls), the
        // other epilogue threads wait in the named barrier
        if (e == 0 && lane == 0)
            x.go_epi[job & 1] = wait_phase<true>(smem_u32(&x.accf[buf]), uint32_t(job >> 1) & 1u, x.abort_flag, a.err);
        named_sync(BAR_EPI, EPI_WARPS * 32);
        if (!x.go_epi[job & 1]) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const TileInfo ti = tile_info(a, t);
        const long mrow = ti.m0 + qd * 32;
        const int nrows = ti.rows - qd * 32;  // rows of this warp's quadrant that exist
        // a transposed conv: this lane's row (an input pixel) and where its
        // kh x kw output block starts
        long tbase = 0;
        int tow = 0;
        if (MODE == EPI_CONVT && lane < nrows) {
            const long m = mrow + lane;
            const LaneInfo &L = a.lanes[find_lane(a.lanes, a.nl, m, true)];
            const int iw = __ldg(&L.iw);
            const int qq = int(m - __ldg(&L.ipix0));
            const int iy = qq / iw, ix = qq - iy * iw;
            tow = __ldg(&L.ow);
            tbase = __ldg(&L.pix0) + (long)iy * a.tkh * tow + (long)ix * a.tkw;
        }
        if (MODE == EPI_CTC) {
            // this thread's row over the columns of its block, 16 at a
            // time in increasing column order: the chunk's maximum raises
            // the running one (rescaling the sum), then the chunk's
            // exponentials (__expf; columns past vocab count as -FLT_MAX,
            // so as zeros) join the running sum. Only the block's maximum
            // and sum are kept: the merge finds the class by recomputing
            // every block near the row's maximum exactly.
            float m = -FLT_MAX, sum = 0.0f;
            for (int c0 = half * 16; c0 < x.BN; c0 += 32) {
                float v[16];
                tmem_ld16(x.tmem + (uint32_t(qd * 32) << 16) + uint32_t(buf * x.BN + c0), v);
                float cm = -FLT_MAX;
                if (x.n0 + c0 + 16 <= a.vocab) {
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        v[j] += bias_s[c0 + j];
                        cm = fmaxf(cm, v[j]);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        v[j] = x.n0 + c0 + j < a.vocab ? v[j] + bias_s[c0 + j] : -FLT_MAX;
                        cm = fmaxf(cm, v[j]);
                    }
                }
                if (cm > m) {
                    sum = m > -FLT_MAX ? sum * __expf(m - cm) : 0.0f;
                    m = cm;
                }
                if (m > -FLT_MAX) {
                    float cs = 0.0f;
#pragma unroll
                    for (int j = 0; j < 16; j++) cs += __expf(v[j] - m);
                    sum += cs;
                }
            }
            if (lane < nrows) {
                float *st = a.partial + ((mrow + lane) * a.blocks + 2 * (x.n0 / x.BN) + half) * 3;
                st[0] = m;
                st[1] = sum;
                st[2] = 0.0f;  // (unused)
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) arrive(smem_u32(&x.acce[buf]));  // one arrival per warp
            continue;
        }
        if (MODE == EPI_PLAIN && vec && a.N <= 48) {
            // narrow rows (at most 192 bytes) straight to memory: each lane
            // stores its own four-channel groups, 16 bytes each (a row's
            // pieces merge in L2), with no transpose through shared memory
            // on the epilogue's critical path; wider rows are stored
            // coalesced below, fewer L2 transactions per byte
            const long m = mrow + lane;
            for (int c0 = half * 16; c0 < x.BN; c0 += 32) {
                float v[16];
                tmem_ld16(x.tmem + (uint32_t(qd * 32) << 16) + uint32_t(buf * x.BN + c0), v);
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const int n = x.n0 + c0 + 4 * c;
                    const float *bb = bias_s + c0 + 4 * c;
                    float4 o = make_float4(activate_t<ACT, true>(fadd(v[4 * c], bb[0])),
                                           activate_t<ACT, true>(fadd(v[4 * c + 1], bb[1])),
                                           activate_t<ACT, true>(fadd(v[4 * c + 2], bb[2])),
                                           activate_t<ACT, true>(fadd(v[4 * c + 3], bb[3])));
                    if (lane >= nrows || n >= a.N) continue;
                    if (a.res) {
                        const float4 rr = __ldg(reinterpret_cast<const float4 *>(a.res + m * a.N + n));
                        o = make_float4(activate(a.act2, fadd(o.x, rr.x)), activate(a.act2, fadd(o.y, rr.y)),
                                        activate(a.act2, fadd(o.z, rr.z)), activate(a.act2, fadd(o.w, rr.w)));
                    }
                    *reinterpret_cast<float4 *>(a.y + m * a.N + n) = o;
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) arrive(smem_u32(&x.acce[buf]));  // one arrival per warp
            continue;
        }
        for (int c0 = half * 16; c0 < x.BN; c0 += 32) {
            float v[16];
            tmem_ld16(x.tmem + (uint32_t(qd * 32) << 16) + uint32_t(buf * x.BN + c0), v);
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const float *bb = bias_s + c0 + 4 * c;
                const float4 o = make_float4(activate_t<ACT, true>(fadd(v[4 * c], bb[0])),
                                             activate_t<ACT, true>(fadd(v[4 * c + 1], bb[1])),
                                             activate_t<ACT, true>(fadd(v[4 * c + 2], bb[2])),
                                             activate_t<ACT, true>(fadd(v[4 * c + 3], bb[3])));
                sts4(stg + uint32_t(lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4)), o);
            }
            __syncwarp();
            const int n = x.n0 + c0 + 4 * q;
            // a transposed conv's column n is tap (ky, kx), channel o
            int tap_off = 0, o_ch = 0;
            if (MODE == EPI_CONVT) {
                const int tap = n / a.toc, ky = tap / a.tkw;
                o_ch = n - tap * a.toc;
                tap_off = ky * 0x10000 + (tap - ky * a.tkw);
            }
#pragma unroll
            for (int p = 0; p < 4; p++) {
                const int r = 8 * p + (lane >> 2);
                float4 o = lds4(stg + uint32_t(r * 64 + ((q ^ ((r >> 1) & 3)) << 4)));
                long ob = 0;
                int ow2 = 0;
                if (MODE == EPI_CONVT) {
                    ob = __shfl_sync(0xffffffffu, tbase, r);
                    ow2 = __shfl_sync(0xffffffffu, tow, r);
                }
                if (r >= nrows || n >= a.N) continue;
                const long m = mrow + r;
                float *dst = MODE == EPI_CONVT
                                 ? a.y + (ob + (long)(tap_off >> 16) * ow2 + (tap_off & 0xffff)) * a.toc + o_ch
                                 : a.y + m * a.N + n;
                if (vec) {
                    if (a.res) {
                        const float4 rr = __ldg(reinterpret_cast<const float4 *>(a.res + m * a.N + n));
                        o = make_float4(activate(a.act2, fadd(o.x, rr.x)), activate(a.act2, fadd(o.y, rr.y)),
                                        activate(a.act2, fadd(o.z, rr.z)), activate(a.act2, fadd(o.w, rr.w)));
                    }
                    *reinterpret_cast<float4 *>(dst) = o;
                } else {
                    const float ov[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        if (n + c >= a.N) break;
                        float y = ov[c];
                        if (a.res) y = activate(a.act2, fadd(y, __ldg(a.res + m * a.N + n + c)));
                        if (MODE == EPI_CONVT) {
                            // column n + c: its own tap when the channels end
                            const int tap = (n + c) / a.toc, ky = tap / a.tkw;
                            a.y[(ob + (long)ky * ow2 + (tap - ky * a.tkw)) * a.toc + (n + c - tap * a.toc)] = y;
                        } else {
                            dst[c] = y;
                        }
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

// Shared set-up of both kernels: barriers, bias slice, TMEM.
template <class R>
__device__ __forceinline__ void setup(const TcArgs &a, Ctx &x, int full_count, uint64_t *bfull, float *bias_s,
                                      uint32_t *tmem_base_s, int *abort_s) {
    const int tid = threadIdx.x, warp = tid / 32;
    if (tid == 0) {
        for (int s = 0; s < x.ns; s++) {
            bar_init(smem_u32(&x.full[s]), full_count);
            bar_init(smem_u32(&x.conv[s]), CONV_THREADS / 32);
            bar_init(smem_u32(&x.empty[s]), 1);
        }
        for (int b = 0; b < 2; b++) {
            bar_init(smem_u32(&x.accf[b]), 1);
            bar_init(smem_u32(&x.acce[b]), EPI_WARPS);
        }
        bar_init(smem_u32(bfull), 1);
        *abort_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (a.fold) {
        // a folded slice's BN / 3 output channels start at channel n0 / 3
        for (int j = tid; j < x.BN / 3; j += R::THREADS)
            bias_s[j] = (a.b && x.n0 / 3 + j < a.toc) ? a.b[x.n0 / 3 + j] : 0.0f;
    } else {
        for (int j = tid; j < x.BN; j += R::THREADS) bias_s[j] = (a.b && x.n0 + j < a.N) ? a.b[x.n0 + j] : 0.0f;
    }
    if (warp == R::W_MMA) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_base_s)),
                     "r"(a.tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    x.tmem = *tmem_base_s;
}

template <class R>
__device__ __forceinline__ void teardown(const TcArgs &a, const Ctx &x) {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (threadIdx.x / 32 == R::W_MMA) {
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(x.tmem), "r"(a.tmem_cols));
    }
}

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_tiled() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

bool encode_weights(TcArgs &a, EncodeTiled enc) {
    // weights: [half][N][kpad], boxes of 32 k x BN outputs; outputs past N
    // read as zeros
    CUtensorMap mw;
    cuuint64_t dims[3] = {cuuint64_t(a.kpad), cuuint64_t(a.N), 2};
    cuuint64_t strides[2] = {cuuint64_t(a.kpad) * 4, cuuint64_t(a.N) * a.kpad * 4};
    cuuint32_t box[3] = {TK, cuuint32_t(a.bn), 1}, estr[3] = {1, 1, 1};
    if (enc(&mw, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(a.w_hi), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    static_assert(sizeof(CUtensorMap) == sizeof(a.tmw), "tensor map size");
    std::memcpy(a.tmw, &mw, sizeof mw);
    return true;
}

}  // namespace

}  // namespace ppocr
