// Pointwise (1x1) convolution on the 5th-generation tensor cores (sm_100a,
// tcgen05) in 3xTF32: y = act2(act(x W + b) + res) over packed pixels.
//
// Each product is split into tf32 halves, x = xh + xl and w = wh + wl, and
// three MMAs accumulate xh wh + xh wl + xl wh in FP32 in tensor memory, which
// keeps the result within a few units of the FP32 one (the dropped xl wl
// term is 2^-22 of the product). The weights arrive already split, [n][kpad]
// (K-major), high halves then low halves; the pixels are split on chip.
//
// The kernel is persistent and warp-specialised. Output channels are cut
// into S slices of BN (a multiple of 32, at most 256); CTA b owns slice
// b % S, keeps that slice's weights (all of K, both halves) resident in
// shared memory, and walks the 128-pixel tiles q, q + Q, q + 2Q, ... with
// q = b / S, so the S CTAs working on one tile do so at about the same time
// and all but the first read it from L2. Per CTA:
//   warp 0      TMA producer: the weight slice once, then each tile's K
//               blocks (128 pixels x 32 channels, 16 KB, 128-byte swizzle)
//               into a ring of `ns` stages;
//   warp 1      allocates tensor memory (two accumulators of BN columns) and
//               one thread issues the MMAs, committing each stage back to the
//               producer and each finished tile to the epilogue;
//   warps 2-5   split each staged block in place into its high half and a
//               low-half twin, then release it to the MMA thread;
//   warps 6-13  epilogue: warp w drains TMEM lanes 32(w%4)..+31 of a finished
//               accumulator, 16 columns at a time (the two warps of a lane
//               quadrant take alternate chunks), adds the bias, applies the
//               activation (one instantiation per code, no branch per
//               element), transposes through shared memory and stores rows
//               (coalesced), adding the residual if any.
// The epilogue of one tile overlaps the MMAs of the next (two accumulators)
// and the producer runs up to `ns` K blocks ahead.
//
// Every wait on an mbarrier is bounded (globaltimer). A wait that runs out
// records a code in `err` (page-locked host memory the runtime reads after
// the run) and raises an abort flag in shared memory that ends every role's
// loop; the producer then waits, bounded, for the copies it issued, the MMA
// thread for its last commit, and the tensor memory is freed before return.
#include <cuda.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "devmath.cuh"
#include "kernels.hpp"

namespace ppocr {

namespace {

constexpr int TM = 128;                   // pixels per tile (MMA M, one TMEM lane each)
constexpr int TK = 32;                    // channels per K block: one 128-byte swizzle row of f32
constexpr int THREADS = 448;              // 14 warps
constexpr int W_MMA = 1, W_CONV = 2, W_EPI = 6, EPI_WARPS = 8;
constexpr int SLOT_BYTES = 2 * TM * 128;  // high half (TMA lands here) + low half
constexpr int STAGE_FLOATS = 32 * 17;     // one epilogue warp's 32 x 16 transpose tile, padded
constexpr int EPI_BYTES = EPI_WARPS * STAGE_FLOATS * 4 + 256 * 4;  // + the bias slice
constexpr int MAX_NS = 6;
// Dynamic shared memory per CTA: the block's limit (227 KB) less room for the
// kernel's static shared memory.
constexpr int DYN_CEILING = 226 * 1024;
// How long one wait on an mbarrier may take before the kernel gives up: a
// K block's copy or MMAs take microseconds.
constexpr unsigned long long WAIT_LIMIT_NS = 200ull * 1000 * 1000;
// A waiting thread sleeps in the mbarrier until the phase completes or this
// many nanoseconds pass, instead of spinning on it.
constexpr uint32_t SUSPEND_HINT_NS = 100000;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

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

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n"
        :
        : "r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void bar_init(uint32_t bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void arrive_expect(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity), "r"(SUSPEND_HINT_NS)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits for the phase of `bar` with this parity to complete. Gives up when
// another role raised the abort flag, or after the time limit (then raises
// it and records the error).
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile int *abort_flag, int *err) {
    if (try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
        if (try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_ns() - t0 > WAIT_LIMIT_NS) {
            *abort_flag = 1;
            if (err) atomicExch(err, 1);
            return false;
        }
    }
}

// The same wait for the clean-up after an abort: bounded, flag ignored.
__device__ __forceinline__ void drain(uint32_t bar, uint32_t parity) {
    const unsigned long long t0 = global_ns();
    while (!try_wait(bar, parity))
        if (global_ns() - t0 > WAIT_LIMIT_NS) return;
}

// Tiled TMA loads (no multicast) completing on an mbarrier.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, int x, int y, int z, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float v[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

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

// Bias and activation over one thread's 16 accumulators, staged for the
// transpose; the activation code is a template argument so the loop holds
// no branch.
template <int ACT>
__device__ __forceinline__ void bias_act_stage(const float v[16], const float *bias, float *row) {
#pragma unroll
    for (int j = 0; j < 16; j++) row[j] = activate_t<ACT>(fadd(v[j], bias[j]));
}

__device__ __forceinline__ void bias_act_stage(int act, const float v[16], const float *bias, float *row) {
    switch (act) {
    case 1: bias_act_stage<1>(v, bias, row); break;
    case 2: bias_act_stage<2>(v, bias, row); break;
    case 3: bias_act_stage<3>(v, bias, row); break;
    case 4: bias_act_stage<4>(v, bias, row); break;
    case 5: bias_act_stage<5>(v, bias, row); break;
    case 6: bias_act_stage<6>(v, bias, row); break;
    case 7: bias_act_stage<7>(v, bias, row); break;
    default: bias_act_stage<0>(v, bias, row); break;
    }
}

__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

__global__ void __launch_bounds__(THREADS, 1)
    pw_tc_kernel(const PwTcArgs a, const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte alignment for the swizzled tiles
    unsigned char *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    __shared__ __align__(8) uint64_t full[MAX_NS], conv[MAX_NS], empty[MAX_NS], accf[2], acce[2], bfull;
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s;

    const int BN = a.bn, ns = a.ns, nkb = a.nkb, S = a.slices;
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const int Q = gridDim.x / S;
    const long first = blockIdx.x / S;
    const int n0 = int(blockIdx.x % S) * BN;
    const long tiles = (a.M + TM - 1) / TM;
    volatile int *abort_flag = &abort_s;

    const uint32_t ring = smem_u32(smem);
    const uint32_t b_base = ring + uint32_t(ns) * SLOT_BYTES;
    const uint32_t b_bytes = uint32_t(BN) * 128;  // one K block of one half
    float *staging = reinterpret_cast<float *>(smem + size_t(ns) * SLOT_BYTES + size_t(2) * nkb * b_bytes);
    float *bias_s = staging + EPI_WARPS * STAGE_FLOATS;  // this slice's BN biases, zero past N

    if (tid == 0) {
        for (int s = 0; s < ns; s++) {
            bar_init(smem_u32(&full[s]), 1);
            bar_init(smem_u32(&conv[s]), 128);
            bar_init(smem_u32(&empty[s]), 1);
        }
        for (int b = 0; b < 2; b++) {
            bar_init(smem_u32(&accf[b]), 1);
            bar_init(smem_u32(&acce[b]), EPI_WARPS * 32);
        }
        bar_init(smem_u32(&bfull), 1);
        abort_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int j = tid; j < BN; j += THREADS) bias_s[j] = (a.b && n0 + j < a.N) ? a.b[n0 + j] : 0.0f;
    if (warp == W_MMA) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                     "r"(a.tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_s;

    if (warp == 0) {
        if (lane == 0) {
            // the weight slice: nkb blocks of BN rows, high halves then low
            const uint32_t bb = smem_u32(&bfull);
            arrive_expect(bb, uint32_t(2 * nkb) * b_bytes);
            for (int kb = 0; kb < nkb; kb++) {
                tma_load_3d(b_base + uint32_t(kb) * b_bytes, &tmw, kb * TK, n0, 0, bb);
                tma_load_3d(b_base + uint32_t(nkb + kb) * b_bytes, &tmw, kb * TK, n0, 1, bb);
            }
            long it = 0;  // K blocks issued
            bool ok = true;
            for (long t = first; t < tiles && ok; t += Q)
                for (int kb = 0; kb < nkb; kb++, it++) {
                    const int s = int(it % ns);
                    const long round = it / ns;
                    if (round > 0 && !wait_phase(smem_u32(&empty[s]), uint32_t(round - 1) & 1u, abort_flag, a.err)) {
                        ok = false;
                        break;
                    }
                    arrive_expect(smem_u32(&full[s]), TM * 128);
                    tma_load_2d(ring + uint32_t(s) * SLOT_BYTES, &tmx, kb * TK, int(t * TM), smem_u32(&full[s]));
                }
            if (*abort_flag) {
                // the copies still in flight land before the CTA leaves
                drain(bb, 0);
                for (int s = 0; s < ns && s < it; s++) drain(smem_u32(&full[s]), uint32_t((it - 1 - s) / ns) & 1u);
            }
        }
    } else if (warp == W_MMA) {
        if (lane == 0) {
            const uint32_t idesc = tf32_idesc(BN);
            long it = 0, job = 0;
            uint32_t last_bar = 0, last_parity = 0;
            bool ok = wait_phase(smem_u32(&bfull), 0, abort_flag, a.err);
            for (long t = first; t < tiles && ok; t += Q, job++) {
                const int buf = int(job & 1);
                const long use = job >> 1;
                if (use > 0 && !wait_phase(smem_u32(&acce[buf]), uint32_t(use - 1) & 1u, abort_flag, a.err)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t d = tmem + uint32_t(buf * BN);
                for (int kb = 0; kb < nkb; kb++, it++) {
                    const int s = int(it % ns);
                    const long round = it / ns;
                    if (!wait_phase(smem_u32(&conv[s]), uint32_t(round) & 1u, abort_flag, a.err)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t ah = ring + uint32_t(s) * SLOT_BYTES, al = ah + TM * 128;
                    const uint32_t bh = b_base + uint32_t(kb) * b_bytes, bl = b_base + uint32_t(nkb + kb) * b_bytes;
                    // K steps of 8 tf32 (32 bytes along the swizzled rows);
                    // steps wholly past K hold zeros and are skipped
                    const int left = a.K - kb * TK;
                    const int steps = left >= TK ? TK / 8 : (left + 7) / 8;
                    for (int kk = 0; kk < steps; kk++) {
                        const uint32_t acc = (kb == 0 && kk == 0) ? 0u : 1u;
                        const uint64_t dah = sw128_desc(ah + kk * 32), dal = sw128_desc(al + kk * 32);
                        const uint64_t dbh = sw128_desc(bh + kk * 32), dbl = sw128_desc(bl + kk * 32);
                        mma_tf32(d, dah, dbh, idesc, acc);
                        mma_tf32(d, dah, dbl, idesc, 1u);
                        mma_tf32(d, dal, dbh, idesc, 1u);
                    }
                    commit(smem_u32(&empty[s]));
                    last_bar = smem_u32(&empty[s]);
                    last_parity = uint32_t(round) & 1u;
                }
                if (!ok) break;
                commit(smem_u32(&accf[buf]));
                last_bar = smem_u32(&accf[buf]);
                last_parity = uint32_t(use) & 1u;
            }
            // the tensor core is done with shared memory and TMEM before the
            // CTA frees them
            if (last_bar) drain(last_bar, last_parity);
        }
    } else if (warp < W_EPI) {
        // split in place: the staged block becomes the high half, its twin
        // the low half (same swizzled layout, so element for element)
        const int ct = tid - W_CONV * 32;
        long it = 0;
        bool ok = true;
        for (long t = first; t < tiles && ok; t += Q)
            for (int kb = 0; kb < nkb; kb++, it++) {
                const int s = int(it % ns);
                const long round = it / ns;
                if (!wait_phase(smem_u32(&full[s]), uint32_t(round) & 1u, abort_flag, a.err)) {
                    ok = false;
                    break;
                }
                float4 *hi = reinterpret_cast<float4 *>(smem + size_t(s) * SLOT_BYTES);
                float4 *lo = hi + TM * 128 / 16;
#pragma unroll
                for (int i = ct; i < TM * 128 / 16; i += 128) {
                    const float4 v = hi[i];
                    const float4 h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
                    hi[i] = h;
                    lo[i] = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
                }
                // make the generic-proxy stores visible to the tensor core
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                arrive(smem_u32(&conv[s]));
            }
    } else {
        const int qd = warp & 3;                 // the TMEM lane quadrant this warp may read
        const int half = (warp - W_EPI) / 4;     // which alternate 16-column chunks it takes
        float *stg = staging + (warp - W_EPI) * STAGE_FLOATS;
        const int col = lane & 15, sub = lane >> 4;
        long job = 0;
        for (long t = first; t < tiles; t += Q, job++) {
            const int buf = int(job & 1);
            const bool ok = wait_phase(smem_u32(&accf[buf]), uint32_t(job >> 1) & 1u, abort_flag, a.err);
            __syncwarp();
            if (!__all_sync(0xffffffffu, ok)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const long mrow = t * TM + qd * 32;
            for (int c0 = half * 16; c0 < BN; c0 += 32) {
                float v[16];
                tmem_ld16(tmem + (uint32_t(qd * 32) << 16) + uint32_t(buf * BN + c0), v);
                bias_act_stage(a.act, v, bias_s + c0, stg + lane * 17);
                __syncwarp();
                // two rows of 16 channels per pass
                const int n = n0 + c0 + col;
                if (n < a.N) {
#pragma unroll 4
                    for (int i = sub; i < 32; i += 2) {
                        const long m = mrow + i;
                        if (m >= a.M) break;
                        float x = stg[i * 17 + col];
                        if (a.res) x = activate(a.act2, fadd(x, __ldg(a.res + m * a.N + n)));
                        a.y[m * a.N + n] = x;
                    }
                }
                __syncwarp();
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            arrive(smem_u32(&acce[buf]));
        }
    }

    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == W_MMA) {
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_cols));
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

size_t smem_for(int kpad, int bn, int ns) {
    return 1024 + size_t(ns) * SLOT_BYTES + size_t(8) * kpad * bn + EPI_BYTES;
}

// The weight slice width for K x N: the fewest slices of at most 256
// channels (a multiple of 32) whose weights, both halves, fit in shared
// memory beside a three-stage ring (else a two-stage one). 0 when none does.
int slice_width(int K, int N) {
    const int kpad = (K + TK - 1) / TK * TK;
    for (int stages = 3; stages >= 2; stages--)
        for (int S = 1; S <= (N + 31) / 32; S++) {
            const int bn = ((N + S - 1) / S + 31) / 32 * 32;
            if (bn <= 256 && smem_for(kpad, bn, stages) <= size_t(DYN_CEILING)) return bn;
        }
    return 0;
}

}  // namespace

bool pw_tc_supported(int K, int N) { return K >= 1 && K % 4 == 0 && N >= 1 && slice_width(K, N) > 0; }

int pw_tc_kpad(int K) { return (K + TK - 1) / TK * TK; }

bool pw_tc_prepare(PwTcArgs &a) {
    if (!pw_tc_supported(a.K, a.N) || a.M < 1 || a.kpad != pw_tc_kpad(a.K)) return false;
    const auto aligned = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!aligned(a.x) || !aligned(a.w_hi) || a.w_lo != a.w_hi + size_t(a.N) * a.kpad) return false;
    EncodeTiled enc = encode_tiled();
    if (!enc) return false;
    a.bn = slice_width(a.K, a.N);
    a.slices = (a.N + a.bn - 1) / a.bn;
    a.nkb = a.kpad / TK;
    a.ns = 2;
    while (a.ns < MAX_NS && smem_for(a.kpad, a.bn, a.ns + 1) <= size_t(DYN_CEILING)) a.ns++;
    a.smem = int(smem_for(a.kpad, a.bn, a.ns));
    a.tmem_cols = 32;
    while (a.tmem_cols < 2 * a.bn) a.tmem_cols *= 2;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
        return false;
    const long tiles = (a.M + TM - 1) / TM;
    const long q = std::max(1L, std::min(long(sms / a.slices), tiles));
    a.grid = int(q) * a.slices;

    CUtensorMap mx, mw;
    {
        // pixels: [M][K], boxes of 32 channels x 128 pixels; channels past K
        // and pixels past M read as zeros
        cuuint64_t dims[2] = {cuuint64_t(a.K), cuuint64_t(a.M)};
        cuuint64_t strides[1] = {cuuint64_t(a.K) * 4};
        cuuint32_t box[2] = {TK, TM}, estr[2] = {1, 1};
        if (enc(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(a.x), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    {
        // weights: [half][N][kpad], boxes of 32 channels x BN outputs; outputs
        // past N read as zeros
        cuuint64_t dims[3] = {cuuint64_t(a.kpad), cuuint64_t(a.N), 2};
        cuuint64_t strides[2] = {cuuint64_t(a.kpad) * 4, cuuint64_t(a.N) * a.kpad * 4};
        cuuint32_t box[3] = {TK, cuuint32_t(a.bn), 1}, estr[3] = {1, 1, 1};
        if (enc(&mw, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(a.w_hi), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    static_assert(sizeof(CUtensorMap) == sizeof(a.tmx), "tensor map size");
    std::memcpy(a.tmx, &mx, sizeof mx);
    std::memcpy(a.tmw, &mw, sizeof mw);
    return true;
}

void configure_tc_kernels() {
    cudaFuncSetAttribute(pw_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, DYN_CEILING);
}

int launch_pw_tc(const PwTcArgs &a, cudaStream_t s) {
    CUtensorMap mx, mw;
    std::memcpy(&mx, a.tmx, sizeof mx);
    std::memcpy(&mw, a.tmw, sizeof mw);
    pw_tc_kernel<<<a.grid, THREADS, a.smem, s>>>(a, mx, mw);
    return 1;
}

}  // namespace ppocr
