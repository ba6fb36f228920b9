// Shared device helpers for the sm_100a token sampler: order-preserving float
// keys, mbarrier + bulk-copy (TMA, non-tensor) PTX wrappers, bounded waits.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace mxs {

// ---------------------------------------------------------------------------
// Sizes of the fused sampling kernel. One CTA streams row chunks through a ring
// of STAGES bulk-copy buffers of TILE floats and keeps a candidate buffer of
// CAP (key, index) pairs in shared memory.
// ---------------------------------------------------------------------------
constexpr int NT = 256;                 // threads per CTA (8 warps)
constexpr int NWARPS = NT / 32;
constexpr int TILE = 4096;              // floats per ring stage (16 KB)
constexpr int SUB = NT * 4;             // floats consumed per sync step (one float4 per thread)
constexpr int STAGES = 4;               // ring depth (64 KB in flight per CTA)
constexpr int CAP = 4096;               // candidate buffer entries
constexpr int KFAST = 2048;             // largest k the streaming path selects
constexpr int SORTMAX = 2048;           // largest candidate set the final sort takes
constexpr int HEAP_SMEM_MAX = 2048;     // exact path keeps its heap in shared memory up to here
constexpr int XTILE = 2048;             // exact path: largest replay step (logits)

// Row flag bits (optional per-row output).
constexpr uint32_t FLAG_EXACT = 1u;     // row resolved by the exact heap replay
constexpr uint32_t FLAG_NAN = 2u;       // row holds a NaN logit
constexpr uint32_t FLAG_OVERFLOW = 4u;  // candidate buffer overflowed (massive ties)
constexpr uint32_t FLAG_TIMEOUT = 8u;   // a bounded wait gave up; outputs of the row are invalid
constexpr uint32_t FLAG_UNSCANNED = 1u << 16;  // internal: row not streamed (k > KFAST), NaN state unknown
constexpr uint32_t FLAG_DONE = 1u << 17;       // internal: row finished by the streaming kernel's idle warps

// Order-preserving 32-bit key of a float: a > b (as floats, not NaN) iff
// key(a) > key(b). -0.0 is folded into +0.0 first, since the reference compares
// widened doubles and -0.0 == +0.0 there.
__device__ __forceinline__ uint32_t fkey(float x) {
    uint32_t u = __float_as_uint(x + 0.0f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(u);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------------------
// mbarrier and bulk copy (cp.async.bulk, global -> shared, completion counted
// in bytes on the mbarrier). No cluster multicast anywhere in this library.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_inval(uint64_t* bar) {
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// Bulk copy of `bytes` (multiple of 16) from 16-byte aligned global memory into
// 16-byte aligned shared memory, with an L2 cache policy. (An evict-first hint
// measured ~5% slower than evict-normal for this streaming read on B200.)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}" : "=r"(done) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return done != 0;
}
// Wait for the phase with the given parity to complete, for at most ~1 s.
// Returns false when the limit ran out; the caller flags the row and stops.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > 1000000000ull) return false;
    }
}

// Phase timers of the profiling build (-DMXS_PROFILE): thread 0 of each CTA
// accumulates clock64 deltas per phase into g_mxs_prof[blockIdx.x][phase].
#ifdef MXS_PROFILE
constexpr int PROF_CTAS = 1024, PROF_PHASES = 8;
__device__ unsigned long long g_mxs_prof[PROF_CTAS][PROF_PHASES];
__shared__ unsigned long long s_mxs_prof[PROF_PHASES];  // per CTA, flushed once at kernel end
#define MXS_PROF_T0(v) long long v = (threadIdx.x == 0) ? clock64() : 0
#define MXS_PROF_ADD(ph, v)                                                          \
    do {                                                                             \
        if (threadIdx.x == 0) mxs::s_mxs_prof[ph] += (unsigned long long)(clock64() - (v)); \
    } while (0)
#define MXS_PROF_BEGIN()                                                             \
    do {                                                                             \
        if (threadIdx.x == 0)                                                        \
            for (int i_ = 0; i_ < mxs::PROF_PHASES; ++i_) mxs::s_mxs_prof[i_] = 0;   \
    } while (0)
#define MXS_PROF_FLUSH()                                                             \
    do {                                                                             \
        if (threadIdx.x == 0 && blockIdx.x < mxs::PROF_CTAS)                         \
            for (int i_ = 0; i_ < mxs::PROF_PHASES; ++i_)                            \
                mxs::g_mxs_prof[blockIdx.x][i_] += mxs::s_mxs_prof[i_];              \
    } while (0)
#define MXS_PROF_COUNT(ph, n)                                                        \
    do {                                                                             \
        if (threadIdx.x == 0) mxs::s_mxs_prof[ph] += (unsigned long long)(n);        \
    } while (0)
#else
#define MXS_PROF_COUNT(ph, n) (void)0
#define MXS_PROF_T0(v) (void)0
#define MXS_PROF_ADD(ph, v) (void)0
#define MXS_PROF_BEGIN() (void)0
#define MXS_PROF_FLUSH() (void)0
#endif

// Barrier over the CTA's NT sampling threads only (named barrier 1). A
// warp-specialised CTA adds a producer warp that never joins it.
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory"); }
__device__ __forceinline__ int csync_or(int pred) {
    int r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.s32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.s32 %0, 1, 0, q;\n}"
        : "=r"(r) : "r"(pred), "n"(NT) : "memory");
    return r;
}

// max that returns NaN when either input is NaN (PTX max.NaN, sm_80+): one
// reduction both screens 16 logits against the threshold and detects a NaN.
__device__ __forceinline__ float fmax_nan(float a, float b) {
    float d;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}
__device__ __forceinline__ float max16_nan(const float4 (&f)[4]) {
    const float a = fmax_nan(fmax_nan(f[0].x, f[0].y), fmax_nan(f[0].z, f[0].w));
    const float b = fmax_nan(fmax_nan(f[1].x, f[1].y), fmax_nan(f[1].z, f[1].w));
    const float c = fmax_nan(fmax_nan(f[2].x, f[2].y), fmax_nan(f[2].z, f[2].w));
    const float d = fmax_nan(fmax_nan(f[3].x, f[3].y), fmax_nan(f[3].z, f[3].w));
    return fmax_nan(fmax_nan(a, b), fmax_nan(c, d));
}

// Warp-inclusive prefix sum.
__device__ __forceinline__ int warp_incl_scan(int v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

}  // namespace mxs
