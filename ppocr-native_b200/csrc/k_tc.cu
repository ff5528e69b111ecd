// Pointwise (1x1) convolution on the 5th-generation tensor cores (sm_100a,
// tcgen05) in 3xTF32: y = act2(act(x W + b) + res) over packed pixels.
//
// Each product is split into tf32 halves, x = xh + xl and w = wh + wl, and
// three MMAs accumulate xh wh + xh wl + xl wh in FP32 in tensor memory, which
// keeps the result within a few units of the FP32 one (the dropped xl wl
// term is 2^-22 of the product). The weights arrive already split and
// transposed ([n][k], K-major) from the host; the pixels are split as they
// are staged.
//
// A CTA owns 128 pixels (the MMA's M, one TMEM lane each) and BN output
// channels (one TMEM column each, 16 <= BN <= 256). K advances 32 channels at
// a time through two shared-memory stages in the 128-byte-swizzled K-major
// layout the MMA reads: while the tensor core works on one stage, the
// threads load and split the next. One thread issues the MMAs and commits
// them to the stage's mbarrier; the loaders wait on that mbarrier before
// overwriting the stage. The epilogue reads the accumulators back with
// tcgen05.ld, adds the bias, applies the activations and the residual, and
// stores.
//
// Every wait on an mbarrier is bounded: past the limit the kernel records a
// code in `err` (page-locked host memory the runtime reads after the run),
// waits once more, bounded, for its own MMAs, frees its tensor memory and
// returns.
#include <cstdint>

#include "devmath.cuh"
#include "kernels.hpp"

namespace ppocr {

namespace {

constexpr int TM = 128;         // pixels per CTA (MMA M)
constexpr int TK = 32;          // channels per stage: one 128-byte swizzle row of f32
constexpr int THREADS = 128;    // warp w owns TMEM lanes 32w..32w+31
// How long one wait on an mbarrier may take before the kernel gives up: a
// stage's MMAs take microseconds.
constexpr unsigned long long WAIT_LIMIT_NS = 200ull * 1000 * 1000;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Byte offset of 16-byte chunk `c` (0..7) of row `r` in a 128B-swizzled,
// K-major tile whose rows are 128 bytes and whose base is 1024-aligned.
__device__ __forceinline__ uint32_t swz(int r, int c) { return uint32_t(r * 128 + ((c ^ (r & 7)) << 4)); }

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

__device__ __forceinline__ bool try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity) {
    const unsigned long long t0 = global_ns();
    while (!try_wait(bar, parity))
        if (global_ns() - t0 > WAIT_LIMIT_NS) return false;
    return true;
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

__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

struct Stage {
    uint32_t a_hi, a_lo, b_hi, b_lo;  // shared addresses of the four tiles
};

__global__ void __launch_bounds__(THREADS, 1) pw_tc_kernel(const PwTcArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte alignment for the swizzled tiles
    unsigned char *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const int BN = a.bn;
    const uint32_t a_bytes = TM * 128, b_bytes = uint32_t(BN) * 128;
    const uint32_t stage_bytes = 2 * a_bytes + 2 * b_bytes;
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ uint32_t tmem_base_s;

    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const long m0 = (long)blockIdx.x * TM;
    const int n0 = blockIdx.y * BN;
    const int nkb = (a.K + TK - 1) / TK;

    Stage st[2];
    for (int s = 0; s < 2; s++) {
        uint32_t base = smem_u32(smem) + s * stage_bytes;
        st[s] = {base, base + a_bytes, base + 2 * a_bytes, base + 2 * a_bytes + b_bytes};
    }
    const uint32_t bar0 = smem_u32(&bars[0]), bar1 = smem_u32(&bars[1]);
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar1));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                     "r"(a.tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_s;

    // Stage loader: rows of the A tile (pixels) and of the B tiles (output
    // channels), 8 chunks of 4 channels each, split into tf32 halves.
    auto load = [&](int kb, const Stage &s) {
        const int k0 = kb * TK;
        for (int e = tid; e < TM * 8; e += THREADS) {
            int r = e / 8, c = e % 8;
            long m = m0 + r;
            int k = k0 + c * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (m < a.M) {
                const float *src = a.x + m * a.K + k;
                if (a.kvec4 && k + 3 < a.K) {
                    v = __ldg(reinterpret_cast<const float4 *>(src));
                } else {
                    if (k < a.K) v.x = __ldg(src);
                    if (k + 1 < a.K) v.y = __ldg(src + 1);
                    if (k + 2 < a.K) v.z = __ldg(src + 2);
                    if (k + 3 < a.K) v.w = __ldg(src + 3);
                }
            }
            float4 h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
            float4 l = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
            uint32_t off = swz(r, c);
            asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(s.a_hi + off), "f"(h.x), "f"(h.y), "f"(h.z),
                         "f"(h.w));
            asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(s.a_lo + off), "f"(l.x), "f"(l.y), "f"(l.z),
                         "f"(l.w));
        }
        // weights: [n][kpad] hi and lo, already zero-padded
        for (int e = tid; e < BN * 8; e += THREADS) {
            int r = e / 8, c = e % 8;
            long row = (long)(n0 + r) * a.kpad + k0 + c * 4;
            float4 h = __ldg(reinterpret_cast<const float4 *>(a.w_hi + row));
            float4 l = __ldg(reinterpret_cast<const float4 *>(a.w_lo + row));
            uint32_t off = swz(r, c);
            asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(s.b_hi + off), "f"(h.x), "f"(h.y), "f"(h.z),
                         "f"(h.w));
            asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(s.b_lo + off), "f"(l.x), "f"(l.y), "f"(l.z),
                         "f"(l.w));
        }
        // make the generic-proxy stores visible to the tensor core
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    };

    const uint32_t idesc = tf32_idesc(BN);
    bool ok = true;
    int last = -1;  // the last K block whose MMAs were committed
    load(0, st[0]);
    __syncthreads();
    for (int kb = 0; kb < nkb; kb++) {
        const Stage &s = st[kb & 1];
        last = kb;
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
            for (int kk = 0; kk < TK / 8; kk++) {
                // K steps of 8 tf32 = 32 bytes along the swizzled rows
                uint64_t ah = sw128_desc(s.a_hi + kk * 32), al = sw128_desc(s.a_lo + kk * 32);
                uint64_t bh = sw128_desc(s.b_hi + kk * 32), bl = sw128_desc(s.b_lo + kk * 32);
                uint32_t first = (kb == 0 && kk == 0) ? 0u : 1u;
                mma_tf32(tmem, ah, bh, idesc, first);
                mma_tf32(tmem, ah, bl, idesc, 1u);
                mma_tf32(tmem, al, bh, idesc, 1u);
            }
            commit((kb & 1) ? bar1 : bar0);
        }
        if (kb + 1 < nkb) {
            // the stage being refilled was last read by the MMAs of kb - 1
            if (kb >= 1) {
                uint32_t bar = ((kb + 1) & 1) ? bar1 : bar0;
                if (!wait_bounded(bar, uint32_t((kb - 1) >> 1) & 1u)) ok = false;
            }
            if (ok) load(kb + 1, st[(kb + 1) & 1]);
        }
        // every thread agrees on whether to go on
        ok = __syncthreads_and(ok) != 0;
        if (!ok) break;
    }
    // all MMAs done: the last commit's completion (waited for once more,
    // bounded, after a wait that gave up)
    {
        uint32_t bar = (last & 1) ? bar1 : bar0;
        uint32_t parity = uint32_t(last >> 1) & 1u;
        if (!wait_bounded(bar, parity)) {
            ok = false;
            wait_bounded(bar, parity);
        }
    }
    if (!ok && a.err && lane == 0) atomicExch(a.err, 1);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

    // Epilogue: warp w reads TMEM lanes 32w..32w+31, 16 columns at a time.
    const long m = m0 + warp * 32 + lane;
    for (int c0 = 0; c0 < BN; c0 += 16) {
        float v[16];
        tmem_ld16(tmem + (uint32_t(warp * 32) << 16) + uint32_t(c0), v);
        if (m >= a.M || !ok) continue;
#pragma unroll
        for (int j = 0; j < 16; j++) {
            int n = n0 + c0 + j;
            if (n >= a.N) continue;
            float x = v[j];
            if (a.b) x = fadd(x, __ldg(a.b + n));
            x = activate(a.act, x);
            if (a.res) x = activate(a.act2, fadd(x, __ldg(a.res + m * a.N + n)));
            a.y[m * a.N + n] = x;
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_cols));
    }
}

}  // namespace

size_t pw_tc_smem(int bn) { return 1024 + 2 * (2 * TM * 128 + 2 * size_t(bn) * 128); }

bool pw_tc_supported(int K, int N) {
    (void)K;
    if (N < 1) return false;
    int bn = pw_tc_bn(N);
    return bn >= 16 && bn <= 256 && pw_tc_smem(bn) <= 227 * 1024;
}

// Output channels per CTA: all of them up to 256 (rounded up to 16), else
// the fewest equal tiles of at most 256.
int pw_tc_bn(int N) {
    int tiles = (N + 255) / 256;
    int per = (N + tiles - 1) / tiles;
    return (per + 15) / 16 * 16;
}

void configure_tc_kernels() {
    cudaFuncSetAttribute(pw_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
}

int launch_pw_tc(const PwTcArgs &a, cudaStream_t s) {
    dim3 grid((unsigned)((a.M + TM - 1) / TM), (unsigned)((a.N + a.bn - 1) / a.bn));
    pw_tc_kernel<<<grid, THREADS, pw_tc_smem(a.bn), s>>>(a);
    return 1;
}

}  // namespace ppocr
