// Two-kernel sampling path for k <= KSPLIT on 16-byte aligned rows.
//
//  1. stream_select_kernel: a producer warp streams every tile of the CTA's
//     (row, chunk) units through a bulk-copy ring; 8 consumer warps each filter
//     a 512-logit slice of every tile against a shared lower bound of the
//     unit's k-th largest value, with no CTA-wide barrier at all: per-unit
//     state lives in an 8-slot ring recycled by the last warp to leave a unit,
//     and each warp appends its surviving candidates to the row's list in
//     global memory when it leaves the unit.
//  2. finish_rows_kernel: one warp per row selects the k-th largest candidate,
//     sorts the k survivors in registers, checks for ties and draws.
//  3. then the finish kernel's CTA (8 warps = one replay CTA) replays each of
//     its rows that needs it (a tie, a NaN, an overflow): the reference's heap
//     process over the row.
#include <cmath>
#include <cstdint>
#include <cuda_runtime.h>

#ifdef MXS_PROFILE
// Phase clocks of the streaming kernel's consumer warp 0 (profiling build),
// summed over CTAs: units, full-barrier waits, first-tile work, later-tile
// work, unit-end flush, slot recycling, whole kernel, tiles.
namespace mxs {
__device__ unsigned long long g_str_clk[8];
}
extern "C" __attribute__((visibility("default"))) int mxs_prof_read_stream(unsigned long long* host, int clear) {
    if (cudaMemcpyFromSymbol(host, mxs::g_str_clk, sizeof(mxs::g_str_clk)) != cudaSuccess) return -3;
    if (clear) {
        static unsigned long long zeros[8];
        if (cudaMemcpyToSymbol(mxs::g_str_clk, zeros, sizeof(zeros)) != cudaSuccess) return -3;
    }
    return 0;
}
// Phase clocks of the finish warps' draws, summed over rows (profiling build):
// sort + tie check, entry
// writes, exps + sum, normalise, truncate + second sum, divide, cumulative
// pick, calls.
namespace mxs {
__device__ unsigned long long g_draw_prof[8];
}
extern "C" __attribute__((visibility("default"))) int mxs_prof_read_draw(unsigned long long* host, int clear) {
    if (cudaMemcpyFromSymbol(host, mxs::g_draw_prof, sizeof(mxs::g_draw_prof)) != cudaSuccess) return -3;
    if (clear) {
        static unsigned long long zeros[8];
        if (cudaMemcpyToSymbol(mxs::g_draw_prof, zeros, sizeof(zeros)) != cudaSuccess) return -3;
    }
    return 0;
}
#define MXS_DRAW_T(v) long long v = clock64()
#define MXS_DRAW_ADD(i, dt) do { if ((threadIdx.x & 31) == 0) atomicAdd(&g_draw_prof[i], (unsigned long long)(dt)); } while (0)
#define MXS_SCLK(v) long long v = clock64()
#define MXS_SADD(i, x) do { if (warp == 0) sclk[i] += (unsigned long long)(x); } while (0)
#else
#define MXS_DRAW_T(v) (void)0
#define MXS_DRAW_ADD(i, x) (void)0
#define MXS_SCLK(v) (void)0
#define MXS_SADD(i, x) (void)0
#endif
#ifdef MXS_PROFILE
// Counters of the per-warp replays (profiling build): replays, heap build,
// first-tile reads, list windows, final sort, draw (cycles summed over
// replays).
namespace mxs {
__device__ unsigned long long g_rep_prof[8];
}
#endif
#include "mxs_rowfinish.cuh"
#include "mxs_stream.h"

namespace mxs {

constexpr int KSPLIT_K = 128;       // largest k of this path (register sort of 128)
constexpr int SW_CAP = 128;         // candidates per consumer warp
constexpr int SLOTS = 8;            // per-unit state ring (> the STAGES a warp can run ahead)
constexpr int FCAP = 256;           // candidate buffer of a finish warp (longer lists stream through it)
static_assert(KSPLIT_K == KSPLIT, "KSPLIT must match the register sort");


struct UnitState {
    // per warp: its m-th largest key (m = ceil(k / NWARPS)) after each of its
    // last four tiles of the unit, as (tile << 32) | key; only grows
    uint64_t pubh[NWARPS][4];
    uint32_t done;           // warps that have left the unit
};

struct StreamSmem {
    uint64_t full[S_STAGES];
    uint64_t empty[S_STAGES];
    UnitState us[SLOTS];
    uint32_t dead;  // a bounded wait ran out: the producer issues no more copies
};

constexpr size_t S_RING = size_t(S_STAGES) * S_TILE * 4;
constexpr size_t S_WBUF = size_t(NWARPS) * SW_CAP * 8;
constexpr size_t S_SMEM = S_RING + S_WBUF + sizeof(StreamSmem);

// Counters of the profiling build: lane 0 of each warp adds to the CTA's totals.
#ifdef MXS_PROFILE
#define MXS_WCOUNT(ph, n)                                                                   \
    do {                                                                                    \
        if ((threadIdx.x & 31) == 0) atomicAdd(&mxs::s_mxs_prof[ph], (unsigned long long)(n)); \
    } while (0)
#else
#define MXS_WCOUNT(ph, n) (void)0
#endif

// The bound a key word stands for: 0 means "no bound yet" (-inf), not the
// NaN that key 0 would decode to.
__device__ __forceinline__ float bound_of(uint32_t key) { return key ? fkey_inv(key) : -INFINITY; }

// Warp-wide bitonic sort of one key per lane, descending.
__device__ __forceinline__ uint32_t warp_sort32_desc(uint32_t v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            const uint32_t o = __shfl_xor_sync(0xffffffffu, v, stride);
            const bool desc = ((lane & size) == 0) || size == 32;
            const bool keep_max = (desc == ((lane & stride) == 0));
            v = keep_max ? max(v, o) : min(v, o);
        }
    }
    return v;
}

#ifndef MXS_EARLY_FINISH
#define MXS_EARLY_FINISH 1
#endif
__device__ void finish_rows_early(const Params& p, unsigned char* smem, int64_t nj);

__global__ void __launch_bounds__(NT_WS, 2) stream_select_kernel(Params p) {
    extern __shared__ __align__(128) unsigned char smem[];
    float* ring = reinterpret_cast<float*>(smem);
    uint32_t* wkeys = reinterpret_cast<uint32_t*>(smem + S_RING);
    int32_t* widx = reinterpret_cast<int32_t*>(smem + S_RING + S_WBUF / 2);
    StreamSmem& sm = *reinterpret_cast<StreamSmem*>(smem + S_RING + S_WBUF);
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int k = p.k_use;
    const int64_t V = p.vocab;
    const int64_t G = gridDim.x;
    const int64_t nj = (p.units > (int64_t)blockIdx.x) ? (p.units - blockIdx.x + G - 1) / G : 0;
    const int S = p.S, TPC = p.tiles_per_chunk;
    const int64_t NTL = (V + S_TILE - 1) / S_TILE;
    auto unit_tiles = [&](int64_t u) -> int {
        const int64_t t0 = (int64_t)(u % S) * TPC;
        return (int)min((int64_t)TPC, NTL - t0);
    };

    if (tid == 0) {
        for (int s = 0; s < S_STAGES; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], NWARPS);
        }
        sm.dead = 0u;
        for (int i = 0; i < SLOTS; ++i) {
            sm.us[i].done = 0u;
            for (int w = 0; w < NWARPS; ++w)
                for (int q = 0; q < 4; ++q) sm.us[i].pubh[w][q] = 0ull;
        }
        fence_mbar_init();
    }
    MXS_PROF_BEGIN();
    __syncthreads();
    // The finish kernel (launched with programmatic stream serialization) may
    // be scheduled as SMs free up; it waits for this grid's completion before
    // reading anything this grid writes.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == NWARPS) {  // producer
        if (lane == 0) {
            const uint64_t pol = policy_evict_normal();
            volatile uint32_t* dead = &sm.dead;
            uint32_t seq = 0;  // copies issued (tiles)
            bool stop = false;
            for (int64_t j = 0; j < nj && !stop; ++j) {
                const int64_t u = blockIdx.x + j * G;
                const int64_t row = u / S;
                const int nt = unit_tiles(u);
                for (int t = 0; t < nt; ++t) {
                    const int s = seq % S_STAGES;
                    // A consumer's wait ran out, or (test hook) CTA 0 stops
                    // before this tile: issue nothing more.
                    if (*dead || (blockIdx.x == 0 && (int64_t)seq == p.debug_drop_tile)) {
                        stop = true;
                        break;
                    }
                    if (seq >= S_STAGES && !mbar_wait_bounded(&sm.empty[s], ((seq / S_STAGES) - 1) & 1)) {
                        atomicOr(&p.row_flag[row], FLAG_TIMEOUT);
                        *dead = 1u;
                        stop = true;
                        break;  // consumers time out on the stages that never come
                    }
                    const int64_t a = ((int64_t)(u % S) * TPC + t) * S_TILE;
                    const int64_t b = min(a + S_TILE, V);
                    const uint32_t bytes = (uint32_t)(((b - a) & ~int64_t(3)) * 4);
                    if (bytes) {
                        mbar_arrive_expect_tx(&sm.full[s], bytes);
                        bulk_g2s(ring + s * S_TILE, p.logits + row * p.ld + a, bytes, &sm.full[s], pol);
                    } else {
                        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&sm.full[s])) : "memory");
                    }
                    ++seq;
                }
            }
            // Before the CTA can retire, every copy this thread issued must have
            // landed: consumers that gave up no longer wait for them. Only the
            // last S_STAGES copies can still be in flight (each stage's earlier
            // phases were waited for through `empty`); each wait is bounded.
            for (uint32_t q = seq > S_STAGES ? seq - S_STAGES : 0; q < seq; ++q)
                (void)mbar_wait_bounded(&sm.full[q % S_STAGES], (q / S_STAGES) & 1);
        }
        return;
    }

    uint32_t* wk = wkeys + warp * SW_CAP;
#ifdef MXS_PROFILE
    unsigned long long sclk[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const long long k0 = clock64();
#endif
    int32_t* wi = widx + warp * SW_CAP;
    const int m = (k + NWARPS - 1) / NWARPS;  // <= 16
    int s = 0;             // ring stage of the next tile
    uint32_t parity = 0;   // its phase parity
    bool dead = false;  // a wait ran out: stop waiting, flag every later row
    for (int64_t j = 0; j < nj; ++j) {
        const int64_t u = blockIdx.x + j * G;
        const int64_t row = u / S;
        const int c = (int)(u % S);
        const int nt = unit_tiles(u);
        const float* xr = p.logits + row * p.ld;
        UnitState& us = sm.us[j % SLOTS];
        int wcnt = 0, nan = 0;
        uint32_t fl = dead ? FLAG_TIMEOUT : 0u;
        // Lanes 0..m-1: keys of m distinct logits of this warp's slices, the
        // largest it has seen (0 = none yet); the m-th is what it publishes.
        uint32_t lkey = 0u;
        uint64_t* rlist = p.row_cand + row * (int64_t)p.row_cap;
        // Append the warp buffer to the row's list (a row over capacity is
        // flagged; its count keeps growing, so the finish kernel sees it too).
        auto flush = [&]() {
            uint32_t base = 0;
            if (lane == 0 && wcnt) base = atomicAdd(&p.row_cnt[row], (uint32_t)wcnt);
            base = __shfl_sync(0xffffffffu, base, 0);
            if (base + (uint32_t)wcnt > (uint32_t)p.row_cap) {
                fl |= FLAG_OVERFLOW;
            } else {
                for (int i = lane; i < wcnt; i += 32) rlist[base + i] = ((uint64_t)wk[i] << 32) | (uint32_t)wi[i];
            }
            MXS_WCOUNT(5, wcnt);
            __syncwarp();
            wcnt = 0;
        };
        // After tile t: this warp's m-th key, tagged with t.
        auto publish = [&](int t) {
            const uint32_t km = __shfl_sync(0xffffffffu, lkey, m - 1);
            if (lane == 0)
                *reinterpret_cast<volatile uint64_t*>(&us.pubh[warp][t & 3]) = ((uint64_t)(uint32_t)t << 32) | km;
        };
        // Fold keys wk[from, from + n) into the top-m list.
        auto fold = [&](int from, int n) {
            for (int r0 = 0; r0 < n; r0 += 32 - m) {
                const int ii = r0 + lane - m;
                uint32_t v = lkey;
                if (lane >= m) v = (ii < n) ? wk[from + ii] : 0u;
                v = warp_sort32_desc(v);
                lkey = (lane < m) ? v : 0u;
            }
        };
        const int a0 = c * TPC * S_TILE;  // the unit's first column (V < 2^31)
        const int last_len = (int)(V - (int64_t)(a0 + (nt - 1) * S_TILE));
        float th_c = -INFINITY;  // cached prefix bound of the later tiles
        for (int t = 0; t < nt; ++t) {
            const int a = a0 + t * S_TILE;
            const int len = (t == nt - 1) ? last_len : S_TILE;
            const int bulk_n = len & ~3;
            if (!dead && *reinterpret_cast<volatile uint32_t*>(&sm.dead)) {
                fl |= FLAG_TIMEOUT;  // another warp's wait ran out: no more copies come
                dead = true;
            }
            MXS_SCLK(w0);
            if (!dead && !mbar_wait_bounded(&sm.full[s], parity)) {
                fl |= FLAG_TIMEOUT;
                dead = true;
                *reinterpret_cast<volatile uint32_t*>(&sm.dead) = 1u;
            }
            MXS_SCLK(w1);
            MXS_SADD(1, w1 - w0);
            MXS_SADD(7, 1);
            const float* st = ring + s * S_TILE;
            float vv[32];
            uint32_t valid = 0xFFFFFFFFu;
            if (len >= (warp + 1) * 1024) {  // this warp's slice is whole (in the bulk copy)
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float4 f = *reinterpret_cast<const float4*>(st + 4 * (warp * 256 + lane + 32 * q));
                    vv[4 * q] = f.x; vv[4 * q + 1] = f.y; vv[4 * q + 2] = f.z; vv[4 * q + 3] = f.w;
                }
            } else {
                valid = 0;
#pragma unroll
                for (int b = 0; b < 32; ++b) {
                    const int e = 4 * (warp * 256 + lane + 32 * (b >> 2)) + (b & 3);
                    vv[b] = -INFINITY;
                    if (e < len) {
                        vv[b] = (e < bulk_n) ? st[e] : xr[a + e];
                        valid |= 1u << b;
                    }
                }
            }
            // max.NaN tree; oct[o] = max of values 8o..8o+7 (kept to screen octets)
            float mx16[16], oct[4];
#pragma unroll
            for (int b = 0; b < 16; ++b) mx16[b] = fmax_nan(vv[2 * b], vv[2 * b + 1]);
#pragma unroll
            for (int b = 0; b < 8; ++b) mx16[b] = fmax_nan(mx16[2 * b], mx16[2 * b + 1]);
#pragma unroll
            for (int b = 0; b < 4; ++b) oct[b] = fmax_nan(mx16[2 * b], mx16[2 * b + 1]);
            const float mxn = fmax_nan(fmax_nan(oct[0], oct[1]), fmax_nan(oct[2], oct[3]));
            nan |= (mxn != mxn);
            float th;  // logits strictly above it pass
            if (t == 0) {
                // The unit's first tile: the fast path's candidates, every logit
                // >= a lower bound of the tile's k-th largest value, seeded from
                // each lane's largest logit (the max tree's top). Its
                // would-enter logits are not listed: a replay reads the first
                // tile again.
                const int nv = __popc(valid);
                // lane maxima sorted: lanes 0..m-1 seed the top-m list; for
                // k <= 32 the k-th is also this warp's own bound (k distinct
                // logits are >= it).
                const uint32_t sorted1 = warp_sort32_desc(nv >= 1 ? fkey(mxn) : 0u);
                float seed = (k <= 32) ? bound_of(__shfl_sync(0xffffffffu, sorted1, k - 1)) : -INFINITY;
                lkey = (lane < m) ? sorted1 : 0u;
                publish(0);
                // Once every consumer warp has published its first-tile m-th
                // key, their minimum bounds the tile's k-th largest: 8m >= k
                // distinct logits are at or above it.
                csync();
                uint32_t mn = 0xFFFFFFFFu;
                if (lane < NWARPS) mn = (uint32_t)*reinterpret_cast<volatile uint64_t*>(&us.pubh[lane][0]);
                mn = __reduce_min_sync(0xffffffffu, mn);
                if (mn) {
                    seed = fmaxf(seed, bound_of(mn));
                } else if (k > 32) {
                    // Some warp holds fewer than m logits of this tile (a short
                    // row): this warp's own bound, the ceil(k/2)-th largest lane
                    // second maximum (k <= 64) or the ceil(k/4)-th largest lane
                    // fourth maximum (each such lane holds 2 or 4 logits >= it).
                    float m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY, m4 = -INFINITY;
                    for (int b = 0; b < 32; ++b) {
                        if ((valid >> b) & 1u) {
                            const float x = vv[b];
                            if (x > m1) {
                                m4 = m3; m3 = m2; m2 = m1; m1 = x;
                            } else if (x > m2) {
                                m4 = m3; m3 = m2; m2 = x;
                            } else if (x > m3) {
                                m4 = m3; m3 = x;
                            } else if (x > m4) {
                                m4 = x;
                            }
                        }
                    }
                    uint32_t own;
                    if (k <= 64) {
                        const uint32_t sorted2 = warp_sort32_desc(nv >= 2 ? fkey(m2) : 0u);
                        own = __shfl_sync(0xffffffffu, sorted2, (k + 1) / 2 - 1);
                    } else {
                        const uint32_t sorted4 = warp_sort32_desc(nv >= 4 ? fkey(m4) : 0u);
                        own = __shfl_sync(0xffffffffu, sorted4, (k + 3) / 4 - 1);
                    }
                    seed = bound_of(own);
                }
                // x >= seed as a strict test (a seed of -inf lets -inf through
                // as "not above": a row whose k-th largest is -inf then has too
                // few candidates and is replayed from its full logits)
                th = (seed == -INFINITY) ? -INFINITY : nextafterf(seed, -INFINITY);
            } else {
                // Later tiles: the would-enter superset. A logit can enter the
                // reference's heap only if it is strictly above the k-th largest
                // logit before it; the smallest m-th key published by the eight
                // warps for tiles before this one stands for 8m >= k distinct
                // earlier logits, so it bounds that from below. Each warp's
                // latest publication from an earlier tile is used (the slots
                // hold the last four, tagged; no warp runs more than two tiles
                // ahead of another, so the one wanted is never overwritten).
                // Bounds only grow, so an older one is valid too: a tile is
                // first screened against the cached bound, and the current one
                // is read only when something passes (or every fourth tile).
                auto prefix_bound = [&]() -> float {
                    uint32_t b = 0xFFFFFFFFu;
                    if (lane < NWARPS) {
                        b = 0u;
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const uint64_t e = *reinterpret_cast<volatile uint64_t*>(&us.pubh[lane][q]);
                            if ((int)(e >> 32) < t) b = max(b, (uint32_t)e);
                        }
                    }
                    return bound_of(__reduce_min_sync(0xffffffffu, b));
                };
                if (t == 1 || (t & 3) == 0) th_c = prefix_bound();
                th = th_c;
                if (__any_sync(0xffffffffu, mxn > th)) {
                    th_c = prefix_bound();
                    th = th_c;
                }
            }
            if (__any_sync(0xffffffffu, mxn > th)) {
                uint32_t mm = 0;
                if (mxn > th) {
#pragma unroll
                    for (int o = 0; o < 4; ++o) {
                        if (oct[o] > th) {  // only octets whose maximum passes
#pragma unroll
                            for (int b = 8 * o; b < 8 * o + 8; ++b)
                                if (vv[b] > th) mm |= 1u << b;
                        }
                    }
                }
                mm &= valid;
                const int cc = __popc(mm);
                int incl, tot;
                MXS_WCOUNT(2, 1);
                if (!__any_sync(0xffffffffu, cc > 1)) {  // usual case: at most one per lane
                    const uint32_t one = __ballot_sync(0xffffffffu, cc != 0);
                    incl = __popc(one & ((2u << lane) - 1u));
                    tot = __popc(one);
                } else {
                    incl = warp_incl_scan(cc);
                    tot = __shfl_sync(0xffffffffu, incl, 31);
                }
                MXS_WCOUNT(t == 0 ? 0 : 1, tot);
                if (wcnt + tot > SW_CAP) flush();
                if (tot <= SW_CAP) {
                    int pos = wcnt + incl - cc;
                    // a new key at or below the warp's own m-th cannot change the top-m list
                    const uint32_t own_mth = __shfl_sync(0xffffffffu, lkey, m - 1);
                    bool grows = false;
                    while (mm) {
                        const int b = __ffs(mm) - 1;
                        mm &= mm - 1;
                        const int e = 4 * (warp * 256 + lane + 32 * (b >> 2)) + (b & 3);
                        const uint32_t key = fkey((e < bulk_n) ? st[e] : xr[a + e]);
                        grows |= key > own_mth;
                        wk[pos] = key;
                        wi[pos] = (int32_t)(a + e);
                        ++pos;
                    }
                    __syncwarp();
                    grows = __any_sync(0xffffffffu, grows);
                    // Fold the new keys into the top-m list. Not on the first
                    // tile: its logits seeded the list already, and counting a
                    // logit twice would break the bound's guarantee.
                    if (grows && t > 0) {
                        MXS_WCOUNT(4, 1);
                        if (tot <= 4) {
                            // a few keys: insert each one by rank (ballot) and a shift
                            for (int ii = 0; ii < tot; ++ii) {
                                const uint32_t v = wk[wcnt + ii];
                                const uint32_t above = __ballot_sync(0xffffffffu, lane < m && lkey >= v);
                                const int r = __popc(above);  // lanes 0..r-1 keep their keys
                                const uint32_t up = __shfl_up_sync(0xffffffffu, lkey, 1);
                                if (r < m && lane >= r && lane < m) lkey = (lane == r) ? v : up;
                            }
                        } else {
                            fold(wcnt, tot);
                        }
                    }
                    wcnt += tot;
                } else {
                    // More than the buffer holds in one slice (a weak bound on an
                    // early tile, or rising runs): append in rounds of at most
                    // two logits per lane, flushing between rounds.
                    MXS_WCOUNT(3, 1);
                    uint32_t rest = mm;
                    while (__any_sync(0xffffffffu, rest != 0u)) {
                        if (wcnt > SW_CAP - 64) flush();
                        uint32_t part = 0u;
                        if (rest) {
                            part = rest & (0u - rest);
                            const uint32_t r1 = rest & ~part;
                            if (r1) part |= r1 & (0u - r1);
                        }
                        rest &= ~part;
                        const int cq = __popc(part);
                        const int iq = warp_incl_scan(cq);
                        const int tq = __shfl_sync(0xffffffffu, iq, 31);
                        int pq = wcnt + iq - cq;
                        for (; part; part &= part - 1) {
                            const int b = __ffs(part) - 1;
                            const int e = 4 * (warp * 256 + lane + 32 * (b >> 2)) + (b & 3);
                            wk[pq] = fkey((e < bulk_n) ? st[e] : xr[a + e]);
                            wi[pq] = (int32_t)(a + e);
                            ++pq;
                        }
                        __syncwarp();
                        if (t > 0) fold(wcnt, tq);
                        wcnt += tq;
                    }
                }
            }
            if (t > 0) publish(t);
            MXS_SCLK(te);
            MXS_SADD(t == 0 ? 2 : 3, te - w1);
            // every lane of the warp is done with the stage: hand it back
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&sm.empty[s])) : "memory");
            if (++s == S_STAGES) {
                s = 0;
                parity ^= 1u;
            }
        }
        // Leave the unit: the rest of the buffer goes to the row's list.
        MXS_SCLK(f0);
        MXS_SADD(0, 1);
        flush();
        if (warp == 0) MXS_WCOUNT(6, 1);
        if (__any_sync(0xffffffffu, nan)) fl |= FLAG_NAN;
        if (lane == 0 && fl) atomicOr(&p.row_flag[row], fl);
        MXS_SCLK(f1);
        MXS_SADD(4, f1 - f0);
        // The last warp out recycles the slot for unit j + SLOTS (no warp can be
        // that far ahead: the ring keeps them within S_STAGES tiles of each other).
        __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            if (atomicAdd(&us.done, 1u) == NWARPS - 1) {
                // Every warp's final m-th key is published: their minimum bounds
                // the unit's k-th largest logit, so the row's (a chunk's k-th
                // largest is at most the row's). The finish kernel starts its
                // selection from it.
                uint32_t mn = 0xFFFFFFFFu;
                for (int w = 0; w < NWARPS; ++w) {
                    uint32_t b = 0u;
                    for (int q = 0; q < 4; ++q) {
                        b = max(b, (uint32_t)us.pubh[w][q]);
                        us.pubh[w][q] = 0ull;
                    }
                    mn = min(mn, b);
                }
                if (mn) atomicMax(&p.row_bound[row], mn);
                __threadfence_block();
                us.done = 0u;
            }
        }
        __syncwarp();
        MXS_SCLK(f2);
        MXS_SADD(5, f2 - f1);
    }
    // A CTA with one unit fewer than the busiest ones would idle for about a
    // unit's streaming time until the grid completes: its consumer warps
    // finish its own rows meanwhile (whole-row units only), so fewer are left
    // to the finish kernel. Every tile this CTA loaded has been consumed, so
    // the ring is free.
    if (MXS_EARLY_FINISH && S == 1 && p.mode == MODE_SAMPLE && !p.edit_cnt && nj > 0 && nj < (p.units + G - 1) / G) {
        csync();  // the CTA's rows are complete: lists, counts, flags, bounds
        if (!*reinterpret_cast<volatile uint32_t*>(&sm.dead)) finish_rows_early(p, smem, nj);
    }
#ifdef MXS_PROFILE
    if (warp == 0 && lane == 0) {
        sclk[6] = (unsigned long long)(clock64() - k0);
        for (int i = 0; i < 8; ++i) atomicAdd(&g_str_clk[i], sclk[i]);
    }
#endif
#ifdef MXS_PROFILE
    csync();  // consumers only: the counters are complete
    MXS_PROF_FLUSH();
#endif
}

// One warp per row: select, register sort, tie check, draw; rows that need the
// exact replay are replayed by the same kernel afterwards.
constexpr int F_WARPS = 8;
struct FinishWarpSmem {
    uint32_t keys[FCAP];
    int32_t idx[FCAP];
    double pbuf[KSPLIT_K];
    Ent e[KSPLIT_K];
    // the replay's heap, 1-based (pair_* in mxs_heap.cuh)
    alignas(16) Ent hp[KSPLIT_K + 2];
    // the replay's heap over double values, for edited rows (dpair_*)
    alignas(16) DEnt dh[KSPLIT_K + 2];
};

// The exact value of edited column `col` of row `row` (binary search of the
// row's edit list, sorted by column).
__device__ __forceinline__ double edit_value(const Params& p, int64_t row, int32_t col) {
    const int32_t* c = p.edit_col + row * (int64_t)p.edit_cap;
    int lo = 0, hi = (int)p.edit_cnt[row];
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (c[mid] < col) lo = mid + 1;
        else hi = mid;
    }
    return p.edit_val[row * (int64_t)p.edit_cap + lo];
}

// An edited value as the float it is rounded down to, and whether that
// float is inexact (then the value lies strictly between it and the next
// float up, and bit 31 of the entry's column marks it).
__device__ __forceinline__ float edit_float(double d, bool* inexact) {
    const float f = __double2float_rd(d);
    *inexact = (double)f != d;
    return f;
}

// Draws for row `row` from e[0, k) and writes next (and the optional outputs);
// returns the drawn position (in every lane).
// Column bits of an Ent index: bit 31 marks a penalised logit whose double
// value fp32 cannot hold (the entry's float is the value rounded down).
constexpr int32_t COL_MASK = 0x7FFFFFFF;

// dv (nullable): the entries' exact values, where penalised logits make the
// floats inexact.
__device__ int warp_draw(const Params& p, int64_t row, const Ent* e, int k, double* pbuf,
                         const double* dv = nullptr) {
    const int lane = threadIdx.x & 31;
    if (p.topk_idx)
        for (int i = lane; i < k; i += 32) p.topk_idx[row * k + i] = e[i].i & COL_MASK;
    const double T = p.temperature;
    bool greedy = (T <= 0.0);
    double sum = 0.0;
    MXS_DRAW_T(d0);
    if (!greedy) {
        const double maxs = dv ? dv[0] : (double)e[0].v;
        for (int i = lane; i < k; i += 32) pbuf[i] = exp(((dv ? dv[i] : (double)e[i].v) - maxs) / T);
        __syncwarp();
        if (lane == 0) sum = seq_sum(pbuf, k);
        sum = __shfl_sync(0xffffffffu, sum, 0);
        greedy = (sum <= 0.0);
    }
    MXS_DRAW_T(d1);
    MXS_DRAW_ADD(2, d1 - d0);
    if (greedy) {
        if (p.topk_prob)
            for (int i = lane; i < k; i += 32) p.topk_prob[row * k + i] = (i == 0) ? 1.0 : 0.0;
        if (lane == 0) p.next[row] = e[0].i & COL_MASK;
        return 0;
    }
    for (int i = lane; i < k; i += 32) {
        const double q = pbuf[i] / sum;
        pbuf[i] = q;
        if (p.topk_prob) p.topk_prob[row * k + i] = q;
    }
    __syncwarp();
    MXS_DRAW_T(d2);
    MXS_DRAW_ADD(3, d2 - d1);
    int n = 0;
    double s2 = 0.0;
    if (lane == 0) {
        n = truncate_p(pbuf, k, p.top_p, p.min_p);
        s2 = (n >= 2) ? seq_sum(pbuf, n) : 0.0;
    }
    n = __shfl_sync(0xffffffffu, n, 0);
    s2 = __shfl_sync(0xffffffffu, s2, 0);
    __syncwarp();
    MXS_DRAW_T(d3);
    MXS_DRAW_ADD(4, d3 - d2);
    if (n < 2) {  // discrete_distribution with fewer than two weights returns 0
        if (lane == 0) p.next[row] = e[0].i & COL_MASK;
        return 0;
    }
    for (int i = lane; i < n; i += 32) pbuf[i] = pbuf[i] / s2;
    __syncwarp();
    MXS_DRAW_T(d4);
    MXS_DRAW_ADD(5, d4 - d3);
    int pick = 0;
    if (lane == 0) {
        pick = cdf_pick(pbuf, n, p.u[row]);
        p.next[row] = e[pick].i & COL_MASK;
    }
    MXS_DRAW_T(d5);
    MXS_DRAW_ADD(6, d5 - d4);
    MXS_DRAW_ADD(7, 1);
    return __shfl_sync(0xffffffffu, pick, 0);
}

// Sort the cnt (<= 32*NS) survivors, find ties, draw. Returns true when the
// row still needs the replay (a tie and a requested top-k list, or a draw that
// lands on a tied position).
template <int NS>
__device__ __forceinline__ bool finish_sorted(const Params& p, int64_t row, FinishWarpSmem& w, int cnt, int k,
                                              bool tie, int lane) {
    MXS_DRAW_T(s0);
    uint64_t b[NS];
#pragma unroll
    for (int s2 = 0; s2 < NS; ++s2) {
        const int i = lane + 32 * s2;
        b[s2] = i < cnt ? ((uint64_t)w.keys[i] << 32) | (uint32_t)w.idx[i] : 0ull;
    }
    warp_sort_desc<NS>(b);
    // tied[i]: position i < k holds a value equal to a neighbour among the cnt sorted
    uint32_t tm[NS];
#pragma unroll
    for (int s2 = 0; s2 < NS; ++s2) {
        const uint64_t up = __shfl_up_sync(0xffffffffu, b[s2], 1);
        const uint64_t dn = __shfl_down_sync(0xffffffffu, b[s2], 1);
        const uint64_t prev_last = __shfl_sync(0xffffffffu, b[s2 > 0 ? s2 - 1 : 0], 31);
        const uint64_t next_first = __shfl_sync(0xffffffffu, b[s2 + 1 < NS ? s2 + 1 : s2], 0);
        const int i = lane + 32 * s2;
        const uint64_t pv = (lane == 0) ? prev_last : up;   // position i - 1 (valid when i > 0)
        const uint64_t nx = (lane == 31) ? next_first : dn;  // position i + 1 (valid when i + 1 < 32 NS)
        const bool t = i < k && ((i > 0 && (b[s2] >> 32) == (pv >> 32)) ||
                                 (i + 1 < cnt && (b[s2] >> 32) == (nx >> 32)));
        tm[s2] = __ballot_sync(0xffffffffu, t);
    }
    uint32_t any = 0u;
#pragma unroll
    for (int s2 = 0; s2 < NS; ++s2) any |= tm[s2];
    tie = tie || any != 0u;
    MXS_DRAW_T(s1);
    MXS_DRAW_ADD(0, s1 - s0);
    // With edited rows a key tie may hide an inexact double (bit 31): the
    // double replay resolves every tie there.
    if (tie && (p.topk_idx || p.edit_cnt)) return true;
#pragma unroll
    for (int s2 = 0; s2 < NS; ++s2) {
        const int i = lane + 32 * s2;
        if (i < k) w.e[i] = Ent{fkey_inv((uint32_t)(b[s2] >> 32)), (int32_t)(uint32_t)b[s2]};
    }
    __syncwarp();
    double* dv = nullptr;
    if (p.edit_cnt) {  // exact values of the k entries (the candidate buffer is free now)
        dv = reinterpret_cast<double*>(w.keys);
        for (int i = lane; i < k; i += 32)
            dv[i] = (w.e[i].i < 0) ? edit_value(p, row, w.e[i].i & COL_MASK) : (double)w.e[i].v;
        __syncwarp();
    }
    MXS_DRAW_T(s2);
    MXS_DRAW_ADD(1, s2 - s1);
    const int pick = warp_draw(p, row, w.e, k, w.pbuf, dv);
    uint32_t tp = 0u;
#pragma unroll
    for (int s2 = 0; s2 < NS; ++s2)
        if ((pick >> 5) == s2) tp = tm[s2];
    return tie && ((tp >> (pick & 31)) & 1u);
}

// The replay list of a finish warp.
constexpr int XSLOT = FCAP;  // Ent entries in w.keys + w.idx
static_assert(sizeof(uint32_t) * FCAP * 2 == sizeof(Ent) * XSLOT, "replay list overlays keys and idx");

__device__ __forceinline__ void xload4(const float* x, int64_t j, int64_t V, float4& v) {
    if (j + 3 < V) {
        v = __ldg(reinterpret_cast<const float4*>(x + j));
    } else {
        v.x = j < V ? x[j] : 0.f;
        v.y = j + 1 < V ? x[j + 1] : 0.f;
        v.z = j + 2 < V ? x[j + 2] : 0.f;
        v.w = 0.f;
    }
}

#ifdef MXS_PROFILE
#define MXS_REP_T(v) long long v = clock64()
#define MXS_REP_ADD(i, x) do { if (lane == 0) atomicAdd(&g_rep_prof[i], (unsigned long long)(x)); } while (0)
extern "C" __attribute__((visibility("default"))) int mxs_prof_read_rep(unsigned long long* host, int clear) {
    if (cudaMemcpyFromSymbol(host, g_rep_prof, sizeof(g_rep_prof)) != cudaSuccess) return -3;
    if (clear) {
        static unsigned long long zeros[8];
        if (cudaMemcpyToSymbol(g_rep_prof, zeros, sizeof(zeros)) != cudaSuccess) return -3;
    }
    return 0;
}
#else
#define MXS_REP_T(v) (void)0
#define MXS_REP_ADD(i, x) (void)0
#endif

// Offer the logits x[lo, hi) to the heap in index order (one warp; lane 0 runs
// the heap). The range is read once, 512 logits per step with the next step's
// loads in flight; every logit above the root seen at the last offer goes to
// the ordered list `slot`, which lane 0 offers whenever it could not take
// another quarter step. The root only rises (no NaN), so a stale root lets
// through a superset of the logits that enter, and each offer makes the exact
// comparison itself. Returns the root (in every lane).
__device__ __noinline__ float warp_replay_range(const float* x, int64_t V, int64_t lo, int64_t hi, PairHeap h,
                                                int k, Ent* slot, float r0) {
    const int lane = threadIdx.x & 31;
    if (lo >= hi) return r0;
    int c = 0;
    const int64_t g0 = lo & ~(int64_t)3;  // rows start 16-byte aligned on this path
    float4 nx[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int64_t j = g0 + 128 * q + 4 * lane;
        if (j < hi) xload4(x, j, V, nx[q]);
    }
    for (int64_t g = g0; g < hi; g += 512) {
        float4 cur[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) cur[q] = nx[q];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int64_t j = g + 512 + 128 * q + 4 * lane;
            if (j < hi) xload4(x, j, V, nx[q]);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (c > XSLOT - 128) {
                __syncwarp();
                MXS_REP_T(o0);
                if (lane == 0) r0 = pair_offer_list(h, k, slot, c, r0);
                MXS_REP_T(o1);
                MXS_REP_ADD(6, o1 - o0);
                MXS_REP_ADD(7, c);
                r0 = __shfl_sync(0xffffffffu, r0, 0);
                c = 0;
            }
            const int64_t j = g + 128 * q + 4 * lane;
            const float e4[4] = {cur[q].x, cur[q].y, cur[q].z, cur[q].w};
            uint32_t m = 0u;
#pragma unroll
            for (int t = 0; t < 4; ++t)
                if (j + t >= lo && j + t < hi && e4[t] > r0) m |= 1u << t;
            const int n = __popc(m);
            const int incl = warp_incl_scan(n);
            int at = c + incl - n;
#pragma unroll
            for (int t = 0; t < 4; ++t)
                if (m & (1u << t)) slot[at++] = Ent{e4[t], (int32_t)(j + t)};
            c += __shfl_sync(0xffffffffu, incl, 31);
        }
    }
    __syncwarp();
    MXS_REP_T(o0);
    if (lane == 0) r0 = pair_offer_list(h, k, slot, c, r0);
    MXS_REP_T(o1);
    MXS_REP_ADD(6, o1 - o0);
    MXS_REP_ADD(7, c);
    return __shfl_sync(0xffffffffu, r0, 0);
}

// Offer the row list's entries with column in [lo, hi) and a value above the
// root, in column order: windows of at most LWIN entries (halved until they
// fit), each gathered into `slot`, sorted by column in registers and offered.
constexpr int LWIN = 128;
__device__ __noinline__ float warp_replay_list(const uint64_t* list, int n, int64_t lo, int64_t hi, PairHeap h,
                                               int k, Ent* slot, float r0) {
    const int lane = threadIdx.x & 31;
    const uint32_t lt = (1u << lane) - 1u;
    while (lo < hi) {
        int64_t whi = hi;
        int c;
        for (;;) {  // gather the window's entries above the root; halve it while they overflow
            const uint32_t rk = fkey(r0);
            c = 0;
            for (int i0 = 0; i0 < n && c <= LWIN; i0 += 32) {
                const int i = i0 + lane;
                const uint64_t v = i < n ? list[i] : 0ull;
                const int64_t col = (int64_t)(uint32_t)v;
                const bool take = i < n && col >= lo && col < whi && (uint32_t)(v >> 32) > rk;
                const uint32_t bal = __ballot_sync(0xffffffffu, take);
                const int pos = c + __popc(bal & lt);
                if (take && pos < LWIN) slot[pos] = Ent{fkey_inv((uint32_t)(v >> 32)), (int32_t)col};
                c += __popc(bal);
            }
            // a window of <= LWIN columns always fits (the list's columns are
            // distinct); the one-column stop only guarantees progress
            if (c <= LWIN || whi - lo == 1) {
                c = min(c, LWIN);
                break;
            }
            whi = lo + (whi - lo) / 2;
        }
        __syncwarp();
        if (c > 0) {
            // sort the window's entries by column: keys (~column << 32 | value
            // bits) sorted descending put the smallest column first
            constexpr int NS = LWIN / 32;
            uint64_t b[NS];
#pragma unroll
            for (int q = 0; q < NS; ++q) {
                const int i = lane + 32 * q;
                b[q] = i < c ? ((uint64_t)(~(uint32_t)slot[i].i) << 32) | __float_as_uint(slot[i].v) : 0ull;
            }
            warp_sort_desc<NS>(b);
            __syncwarp();
#pragma unroll
            for (int q = 0; q < NS; ++q) {
                const int i = lane + 32 * q;
                if (i < c) slot[i] = Ent{__uint_as_float((uint32_t)b[q]), (int32_t)~(uint32_t)(b[q] >> 32)};
            }
            __syncwarp();
            if (lane == 0) r0 = pair_offer_list(h, k, slot, c, r0);
            r0 = __shfl_sync(0xffffffffu, r0, 0);
        }
        lo = whi;
    }
    return r0;
}

// One warp replays the reference's partial_sort heap process over row `row`
// without reading the whole row again, and draws. Rows without NaN, k <=
// KSPLIT_K, whose list did not overflow. The heap lives in w.hp; w.keys
// / w.idx hold the replay list. A row is streamed as S chunks of TPC tiles; in
// each chunk the logits of the first tile are read again from memory, and
// those of the later tiles come from the row's list, which holds every one of
// them that is strictly above a lower bound of the k-th largest logit before
// it within the chunk -- so every logit that can enter the heap (the
// reference enters logit i only if it is strictly above the k-th largest of
// x[0, i)), in the chunk's order.
__device__ void exact_row_warp_log(const Params& p, int64_t row, FinishWarpSmem& w, uint32_t cnt_all) {
    const int lane = threadIdx.x & 31;
    const int k = p.k_use;
    const int64_t V = p.vocab;
    const float* x = p.logits + row * p.ld;
    const uint64_t* list = p.row_cand + row * (int64_t)p.row_cap;
    const PairHeap h{w.hp};
    Ent* slot = reinterpret_cast<Ent*>(w.keys);
    MXS_REP_T(q0);
    for (int i = lane; i < k; i += 32) w.hp[i + 1] = Ent{x[i], i};
    __syncwarp();
    if (lane == 0) pair_build(h, k);
    __syncwarp();
    MXS_REP_T(q1);
    MXS_REP_ADD(0, 1);
    MXS_REP_ADD(1, q1 - q0);
    float r0 = w.hp[1].v;
    const int64_t chunk = (int64_t)p.tiles_per_chunk * S_TILE;
    for (int c = 0; c < p.S; ++c) {
        const int64_t c0 = c * chunk;
        if (c0 >= V) break;
        const int64_t t1 = min(V, c0 + S_TILE), ce = min(V, c0 + chunk);
        MXS_REP_T(q2);
        r0 = warp_replay_range(x, V, max(c0, (int64_t)k), t1, h, k, slot, r0);
        __syncwarp();
        MXS_REP_T(q3);
        r0 = warp_replay_list(list, (int)cnt_all, t1, ce, h, k, slot, r0);
        __syncwarp();
        MXS_REP_T(q4);
        MXS_REP_ADD(2, q3 - q2);
        MXS_REP_ADD(3, q4 - q3);
    }
    MXS_REP_T(q5);
    if (lane == 0) pair_sort(h, k);
    __syncwarp();
    for (int i = lane; i < k; i += 32) w.e[i] = w.hp[i + 1];
    __syncwarp();
    MXS_REP_T(q6);
    warp_draw(p, row, w.e, k, w.pbuf);
    __syncwarp();
    MXS_REP_T(q7);
    MXS_REP_ADD(4, q6 - q5);
    MXS_REP_ADD(5, q7 - q6);
}

// One warp replays the reference's heap process over an edited row in double,
// reading the whole row once (512 logits per step) and merging the row's edit
// list (sorted by column; those columns read -inf in memory) at its columns,
// then draws. Rows without NaN; k <= KSPLIT_K. The heap lives in w.dh; w.keys /
// w.idx hold the ordered list of logits above the root seen at the last offer.
__device__ __forceinline__ void exact_row_warp_edits(const Params& p, int64_t row, FinishWarpSmem& w) {
    const int lane = threadIdx.x & 31;
    const int k = p.k_use;
    const int64_t V = p.vocab;
    const float* x = p.logits + row * p.ld;
    const int32_t* ec = p.edit_col + row * (int64_t)p.edit_cap;
    const double* ev = p.edit_val + row * (int64_t)p.edit_cap;
    const int ne = (int)p.edit_cnt[row];
    DEnt* h = w.dh;
    Ent* slot = reinterpret_cast<Ent*>(w.keys);
    int ecur = 0;  // the next edit to offer (lane 0's cursor)
    for (int i = lane; i < k; i += 32) h[i + 1] = DEnt{(double)x[i], i, 0};
    __syncwarp();
    if (lane == 0) {
        // edited columns inside the first k (node c + 1 holds column c before the build)
        for (; ecur < ne && ec[ecur] < k; ++ecur) h[ec[ecur] + 1].v = ev[ecur];
        dpair_build(h, k);
    }
    ecur = __shfl_sync(0xffffffffu, ecur, 0);
    __syncwarp();
    double r0 = h[1].v;
    // lane 0: offer slot[0, c) in column order, each preceded by the edits of
    // smaller columns; then the edits below `upto`
    auto offer = [&](int c, int64_t upto) {
        __syncwarp();
        if (lane == 0) {
            for (int j = 0; j <= c; ++j) {
                const int64_t col = j < c ? (int64_t)slot[j].i : upto;
                for (; ecur < ne && ec[ecur] < col; ++ecur)
                    if (ev[ecur] > r0) r0 = dpair_place(h, 1, k, DEnt{ev[ecur], ec[ecur], 0});
                if (j < c && (double)slot[j].v > r0) r0 = dpair_place(h, 1, k, DEnt{(double)slot[j].v, slot[j].i, 0});
            }
        }
        r0 = __shfl_sync(0xffffffffu, r0, 0);
        ecur = __shfl_sync(0xffffffffu, ecur, 0);
    };
    int c = 0;
    const int64_t g0 = (int64_t)k & ~(int64_t)3;  // rows start 16-byte aligned on this path
    for (int64_t g = g0; g < V; g += 512) {
        float4 cur[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int64_t j = g + 128 * q + 4 * lane;
            if (j < V) xload4(x, j, V, cur[q]);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (c > XSLOT - 128) {
                offer(c, g + 128 * q);
                c = 0;
            }
            const int64_t j = g + 128 * q + 4 * lane;
            const float e4[4] = {cur[q].x, cur[q].y, cur[q].z, cur[q].w};
            uint32_t m = 0u;
#pragma unroll
            for (int t = 0; t < 4; ++t)
                if (j + t >= k && j + t < V && (double)e4[t] > r0) m |= 1u << t;
            const int n = __popc(m);
            const int incl = warp_incl_scan(n);
            int at = c + incl - n;
#pragma unroll
            for (int t = 0; t < 4; ++t)
                if (m & (1u << t)) slot[at++] = Ent{e4[t], (int32_t)(j + t)};
            c += __shfl_sync(0xffffffffu, incl, 31);
        }
    }
    offer(c, V);
    if (lane == 0) dpair_sort(h, k);
    __syncwarp();
    double* dv = reinterpret_cast<double*>(w.keys);  // the list is offered: free
    for (int i = lane; i < k; i += 32) {
        w.e[i] = Ent{(float)h[i + 1].v, h[i + 1].i};
        dv[i] = h[i + 1].v;
    }
    __syncwarp();
    warp_draw(p, row, w.e, k, w.pbuf, dv);
    __syncwarp();
}

// One warp finishes row `row`; returns true (in every lane) when the row needs
// the replay. The row's counters are cleared for the next call.
// The k-th largest of keys[0, n), n <= FCAP, for one warp: the keys stay in
// registers (FCAP / 32 per lane) and the answer is built from the top bit
// down, two bits per step, counting with warp reductions. Same result as
// warp_select_kth, without its shared-memory histogram passes.
__device__ __forceinline__ uint32_t warp_select_kth_small(const uint32_t* keys, int n, int k) {
    constexpr int PER = FCAP / 32;
    const int lane = threadIdx.x & 31;
    uint32_t kv[PER];
    uint32_t a = ~0u, o = 0u;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int i = lane + 32 * j;
        kv[j] = i < n ? keys[i] : 0u;
        if (i < n) {
            a &= kv[j];
            o |= kv[j];
        }
    }
    a = __reduce_and_sync(0xffffffffu, a);
    o = __reduce_or_sync(0xffffffffu, o);
    if (a == o) return a;
    const int hi = 31 - __clz(a ^ o);
    uint32_t mask = ~((2u << hi) - 1u);  // bits above hi: the same in every key
    uint32_t prefix = a & mask;
    unsigned krem = (unsigned)k;
    int b = hi;
    // two bits per step: the counts of the digits 3, 2 and 1 among the keys
    // that match the prefix (three independent reductions)
#pragma unroll 1
    for (; b >= 1; b -= 2) {
        const uint32_t tm = mask | (3u << (b - 1));
        unsigned c3 = 0, c2 = 0, c1 = 0;
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const bool in = lane + 32 * j < n && (kv[j] & mask) == prefix;
            const uint32_t d = (kv[j] >> (b - 1)) & 3u;
            c3 += (in && d == 3u) ? 1u : 0u;
            c2 += (in && d == 2u) ? 1u : 0u;
            c1 += (in && d == 1u) ? 1u : 0u;
        }
        c3 = __reduce_add_sync(0xffffffffu, c3);
        c2 = __reduce_add_sync(0xffffffffu, c2);
        c1 = __reduce_add_sync(0xffffffffu, c1);
        uint32_t d;
        if (c3 >= krem) {
            d = 3u;
        } else if (c3 + c2 >= krem) {
            d = 2u;
            krem -= c3;
        } else if (c3 + c2 + c1 >= krem) {
            d = 1u;
            krem -= c3 + c2;
        } else {
            d = 0u;
            krem -= c3 + c2 + c1;
        }
        prefix |= d << (b - 1);
        mask = tm;
    }
    if (b == 0) {  // one bit left
        unsigned c = 0;
#pragma unroll
        for (int j = 0; j < PER; ++j) c += (lane + 32 * j < n && (kv[j] & (mask | 1u)) == (prefix | 1u)) ? 1u : 0u;
        c = __reduce_add_sync(0xffffffffu, c);
        if (c >= krem) prefix |= 1u;
    }
    return prefix;
}

#ifdef MXS_PROFILE
// Phase clocks of the finish warps (profiling build), summed over rows: list,
// select, sort + draw, wait for the streaming grid, whole row, rows, list
// length; and a timeline in globaltimer ns: first CTA start, first and last
// end of the wait, last CTA end.
__device__ unsigned long long g_fin_prof[8];
__device__ unsigned long long g_fin_tl[4];
#define MXS_FIN_T(v) long long v = clock64()
#define MXS_FIN_ADD(i, x) do { if (lane == 0) atomicAdd(&g_fin_prof[i], (unsigned long long)(x)); } while (0)
#else
#define MXS_FIN_T(v) (void)0
#define MXS_FIN_ADD(i, x) (void)0
#endif

// Gather the entries of src[0, n) whose key is >= `bound` into w.keys / w.idx
// (after the cnt entries already there), raising the bound to the k-th largest
// key held whenever the buffer fills, so lists longer than the buffer still
// fit. Sets massive when ties keep the buffer full. seg_min (nullable) gets the
// smallest key of the segment.
__device__ __forceinline__ void gather_segment(const uint64_t* src, int n, FinishWarpSmem& w, int k, int& cnt,
                                               uint32_t& bound, bool& massive, uint32_t* seg_min = nullptr) {
    const int lane = threadIdx.x & 31;
    const uint32_t lt = (1u << lane) - 1u;
    uint32_t mn = 0xFFFFFFFFu;
    // 256 entries per load round trip (8 per lane in flight).
    for (int i0 = 0; i0 < n && !massive; i0 += 256) {
        uint64_t vv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = i0 + 32 * j + lane;
            vv[j] = i < n ? src[i] : 0ull;
            if (i < n) mn = min(mn, (uint32_t)(vv[j] >> 32));
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (massive || i0 + 32 * j >= n) break;
            const int i = i0 + 32 * j + lane;
            const uint64_t v = vv[j];
            const bool take = i < n && (uint32_t)(v >> 32) >= bound;
            const uint32_t bal = __ballot_sync(0xffffffffu, take);
            if (take) {
                const int pos = cnt + __popc(bal & lt);
                w.keys[pos] = (uint32_t)(v >> 32);
                w.idx[pos] = (int32_t)(uint32_t)v;
            }
            cnt += __popc(bal);
            __syncwarp();
            if (cnt > FCAP - 32) {
                bound = warp_select_kth_small(w.keys, cnt, k);
                cnt = warp_compact_ge(w.keys, w.idx, cnt, bound);
                if (cnt > FCAP - 32) massive = true;  // massive ties
            }
        }
    }
    if (seg_min) *seg_min = __reduce_min_sync(0xffffffffu, mn);
}

// Row `row`'s candidate list into w.keys / w.idx, starting from the streaming
// warps' lower bound of the row's k-th largest. Returns the count; sets
// *massive when ties keep the buffer full.
__device__ __forceinline__ int gather_row_list(const Params& p, int64_t row, FinishWarpSmem& w, uint32_t cnt_all,
                                           int k, bool* massive) {
    int cnt = 0;
    uint32_t bound = p.row_bound[row];
    bool m = false;
    gather_segment(p.row_cand + row * (int64_t)p.row_cap, (int)cnt_all, w, k, cnt, bound, m);
    *massive = m;
    return cnt;
}

// MODE_EMIT (vocab-sharded step 1 on this path): publish row `row`'s candidate
// list -- every logit of the shard >= the shard's k-th largest value -- with
// global column indices: first every logit above the k-th largest (fewer than
// k), then those equal to it. When more tie at the k-th largest than out_cap
// holds, the list keeps as many as fit and gets FLAG_EXACT ("truncated": every
// logit left out equals the list's smallest value). A row the list cannot
// represent (NaN, overflow, massive ties) gets a count of 0 and a flag, and
// the merge hands it back. The row's streaming-list length is kept in
// log_count (when given) for a later replay; the list itself stays in the
// workspace until the next call.
__device__ void emit_row_warp(const Params& p, int64_t row, FinishWarpSmem& w) {
    const int lane = threadIdx.x & 31;
    const uint32_t lt = (1u << lane) - 1u;
    const int k = p.k_use;
    uint32_t flags = p.row_flag[row] & (FLAG_NAN | FLAG_OVERFLOW | FLAG_TIMEOUT);
    const uint32_t cnt_all = p.row_cnt[row];
    if (!flags && (cnt_all > (uint32_t)p.row_cap || cnt_all < (uint32_t)k)) flags |= FLAG_OVERFLOW;
    int n_out = 0;
    uint64_t* dst = p.out_cand + row * p.out_cap;
    if (!flags) {
        bool massive = false;
        int cnt = gather_row_list(p, row, w, cnt_all, k, &massive);
        if (massive || cnt < k) {
            flags |= FLAG_OVERFLOW;
        } else {
            const uint32_t kth = warp_select_kth_small(w.keys, cnt, k);
            cnt = warp_compact_ge(w.keys, w.idx, cnt, kth);
            int pos = 0;
            for (int pass = 0; pass < 2; ++pass) {  // above the k-th largest, then equal to it
                for (int i0 = 0; i0 < cnt; i0 += 32) {
                    const int i = i0 + lane;
                    const bool take = i < cnt && (pass == 0 ? w.keys[i] > kth : w.keys[i] == kth);
                    const uint32_t bal = __ballot_sync(0xffffffffu, take);
                    const int at = pos + __popc(bal & lt);
                    if (take && at < p.out_cap)
                        dst[at] = ((uint64_t)w.keys[i] << 32) | (uint32_t)(w.idx[i] + (int32_t)p.col_offset);
                    pos += __popc(bal);
                }
            }
            n_out = min(pos, p.out_cap);
            if (pos > p.out_cap) flags |= FLAG_EXACT;
        }
    }
    if (lane == 0) {
        p.out_count[row] = (uint32_t)n_out;
        p.out_flags[row] = flags;
        if (p.log_count) p.log_count[row] = cnt_all;
        if (flags & FLAG_TIMEOUT) atomicOr(p.status, flags);
        p.row_cnt[row] = 0u;  // left clear for the next call on this workspace
        p.row_flag[row] = 0u;
        p.row_bound[row] = 0u;
    }
}

// MODE_MERGE on this path (k <= KSPLIT_K): one warp merges row `row`'s shard
// lists (nshards blocks of [rows x in_cap] words), selects the k largest,
// checks for ties and draws. Handed back (next = -1, MXS_ROW_EXACT plus the
// shard flags) are rows with a flagged shard list (NaN, overflow, timeout), a
// truncated list whose left-out logits could be among the k largest, and tie
// rows whose order matters (a requested top-k list, or a draw that lands on a
// tied position): their tie order depends on logits no list holds.
__device__ void merge_row_warp(const Params& p, int64_t row, FinishWarpSmem& w) {
    const int lane = threadIdx.x & 31;
    const int k = p.k_use;
    uint32_t bad = 0u, trunc_min = 0u;
    int cnt = 0;
    uint32_t bound = 0u;
    bool massive = false;
    for (int s = 0; s < p.nshards; ++s) {
        const int64_t at = (int64_t)s * p.rows + row;
        const uint32_t fl = p.in_flags ? p.in_flags[at] : 0u;
        if (fl & (FLAG_NAN | FLAG_OVERFLOW | FLAG_TIMEOUT)) {
            bad |= fl & (FLAG_NAN | FLAG_OVERFLOW | FLAG_TIMEOUT);
            continue;
        }
        const int n = (int)min(p.in_count[at], (uint32_t)p.in_cap);
        uint32_t mn = 0u;
        gather_segment(p.in_cand + at * p.in_cap, n, w, k, cnt, bound, massive, &mn);
        if ((fl & FLAG_EXACT) && n > 0) trunc_min = max(trunc_min, mn);
    }
    bool back = bad != 0u || massive || cnt < k;
    if (!back) {
        bool tie = false;
        if (cnt > k) {
            const uint32_t kth = warp_select_kth_small(w.keys, cnt, k);
            cnt = warp_compact_ge(w.keys, w.idx, cnt, kth);
            tie = cnt != k;
            back = trunc_min >= kth;  // left-out logits would be among the k largest
        } else {
            back = trunc_min >= warp_select_kth_small(w.keys, cnt, k);
        }
        if (!back && cnt > KSPLIT_K) back = true;
        if (!back) back = (cnt <= 64) ? finish_sorted<2>(p, row, w, cnt, k, tie, lane)
                                      : finish_sorted<4>(p, row, w, cnt, k, tie, lane);
    }
    if (lane == 0) {
        if (back) p.next[row] = -1;
        if (p.row_flags) p.row_flags[row] = back ? (FLAG_EXACT | bad) : 0u;
    }
}

__global__ void __launch_bounds__(F_WARPS * 32) merge_rows_kernel(Params p) {
    extern __shared__ __align__(128) unsigned char msmem[];
    FinishWarpSmem& w = reinterpret_cast<FinishWarpSmem*>(msmem)[threadIdx.x >> 5];
    const int64_t row = (int64_t)blockIdx.x * F_WARPS + (threadIdx.x >> 5);
    if (row < p.rows) merge_row_warp(p, row, w);
}

// *out_full: the row's list cannot stand for it (NaN, overflow, fewer than k
// candidates), so a replay must read the whole row.
// EARLY (the streaming kernel's idle warps, finish_rows_early): a row that
// needs a replay or timed out is left untouched for the finish kernel (its
// outputs are rewritten there); any other row is finished and marked
// FLAG_DONE, which the finish kernel clears and skips.
template <bool EARLY>
__device__ bool finish_row_warp(const Params& p, int64_t row, FinishWarpSmem& w, uint32_t* out_flags,
                                uint32_t* out_cnt, bool* out_full) {
    const int lane = threadIdx.x & 31;
    MXS_FIN_T(f0);
    const int k = p.k_use;
    uint32_t flags = p.row_flag[row];
    if (EARLY && (flags & FLAG_TIMEOUT)) return true;
    if (!EARLY && (flags & FLAG_DONE)) {
        __syncwarp();
        if (lane == 0) p.row_flag[row] = 0u;  // left clear for the next call
        *out_flags = 0u;
        *out_cnt = 0u;
        *out_full = false;
        return false;
    }
    const uint32_t cnt_all = p.row_cnt[row];
    bool exact = (flags & (FLAG_NAN | FLAG_OVERFLOW)) != 0 || cnt_all > (uint32_t)p.row_cap ||
                 cnt_all < (uint32_t)k;
    bool full = exact;
    if (!(flags & FLAG_TIMEOUT) && !exact) {
        bool massive = false;
        int cnt = gather_row_list(p, row, w, cnt_all, k, &massive);
        if (p.edit_cnt && !massive) {
            // the edited (penalised) logits, which the streaming pass never
            // saw: their floats rounded down, inexact ones marked in bit 31
            const int ne = (int)p.edit_cnt[row];
            const uint32_t lt = (1u << lane) - 1u;
            uint32_t bound = 0u;
            for (int j0 = 0; j0 < ne && !massive; j0 += 32) {
                const int j = j0 + lane;
                bool take = false;
                uint32_t key = 0u;
                int32_t col = 0;
                if (j < ne) {
                    bool inexact;
                    key = fkey(edit_float(p.edit_val[row * (int64_t)p.edit_cap + j], &inexact));
                    col = p.edit_col[row * (int64_t)p.edit_cap + j] | (inexact ? (int32_t)0x80000000 : 0);
                    take = key >= bound;
                }
                const uint32_t bal = __ballot_sync(0xffffffffu, take);
                if (take) {
                    w.keys[cnt + __popc(bal & lt)] = key;
                    w.idx[cnt + __popc(bal & lt)] = col;
                }
                cnt += __popc(bal);
                __syncwarp();
                if (cnt > FCAP - 32) {
                    bound = warp_select_kth_small(w.keys, cnt, k);
                    cnt = warp_compact_ge(w.keys, w.idx, cnt, bound);
                    if (cnt > FCAP - 32) massive = true;
                }
            }
        }
        exact = massive;
        // Ties among the survivors, or across the cut, make the reference's
        // order of the equal values a product of its heap process. The
        // probabilities and their running sums depend only on the values by
        // position, so without a requested top-k list the draw is exact unless
        // it lands on a tied position; only then does the row need the replay.
        MXS_FIN_T(f1);
        MXS_FIN_ADD(0, f1 - f0);
        MXS_FIN_ADD(6, cnt_all);
        bool tie = false;
        if (!exact && cnt > (k <= 64 ? 64 : KSPLIT_K)) {
            // more candidates than the smallest register sort for k takes:
            // keep those >= the k-th
            const uint32_t kth = warp_select_kth_small(w.keys, cnt, k);
            cnt = warp_compact_ge(w.keys, w.idx, cnt, kth);
            if (cnt != k) {  // a tie straddles the cut
                tie = true;
                exact = (cnt > KSPLIT_K) || (p.topk_idx != nullptr) || (p.edit_cnt != nullptr);
            }
        } else if (!exact && cnt < k) {
            exact = true;
            full = true;
        }
        MXS_FIN_T(f2);
        MXS_FIN_ADD(1, f2 - f1);
        if (!exact) {
            if (cnt <= 64)
                exact = finish_sorted<2>(p, row, w, cnt, k, tie, lane);
            else
                exact = finish_sorted<4>(p, row, w, cnt, k, tie, lane);
        }
        MXS_FIN_T(f3);
        MXS_FIN_ADD(2, f3 - f2);
    }
    if (EARLY) {
        if (exact) return true;
        __syncwarp();
        if (lane == 0) {
            if (p.row_flags) p.row_flags[row] = flags;
            p.row_cnt[row] = 0u;
            p.row_bound[row] = 0u;
            p.row_flag[row] = FLAG_DONE;
        }
        return false;
    }
    if (lane == 0) {
        if (flags & FLAG_TIMEOUT) {
            p.next[row] = -1;
            atomicOr(p.status, flags);
        }
        if (p.row_flags) p.row_flags[row] = flags | ((exact && !(flags & FLAG_TIMEOUT)) ? FLAG_EXACT : 0u);
        p.row_cnt[row] = 0u;  // left clear for the next call on this workspace
        p.row_flag[row] = 0u;
        p.row_bound[row] = 0u;
    }
    *out_flags = flags;
    *out_cnt = cnt_all;
    *out_full = full;
    return exact && !(flags & FLAG_TIMEOUT);
}

// The idle consumer warps of a streaming CTA (stream_select_kernel) finish up
// to two rows each of the CTA's own rows, the last ones first; the ring holds
// their FinishWarpSmem. Rows that need a replay are left to the finish kernel.
constexpr int EARLY_ROWS_PER_WARP = 2;
static_assert(sizeof(FinishWarpSmem) * NWARPS <= S_RING, "finish areas overlay the streaming ring");
__device__ void finish_rows_early(const Params& p, unsigned char* smem, int64_t nj) {
    const int warp = threadIdx.x >> 5;
    FinishWarpSmem& w = reinterpret_cast<FinishWarpSmem*>(smem)[warp];
    const int64_t lo = max((int64_t)0, nj - (int64_t)NWARPS * EARLY_ROWS_PER_WARP);
    for (int64_t j = nj - 1 - warp; j >= lo; j -= NWARPS) {
        const int64_t row = blockIdx.x + j * (int64_t)gridDim.x;
        uint32_t flags, cnt_all;
        bool full;
        (void)finish_row_warp<true>(p, row, w, &flags, &cnt_all, &full);
        __syncwarp();
    }
}

// Rows of the exact replay need a whole CTA; the finish kernel's CTAs are
// exactly NT threads (F_WARPS warps) and replay their own handed-over rows.
constexpr size_t F_WARP_AREA = sizeof(FinishWarpSmem) * F_WARPS;
constexpr size_t F_REGION = F_WARP_AREA > REGION_BYTES ? F_WARP_AREA : REGION_BYTES;
constexpr size_t F_SMEM = (F_REGION + 15) / 16 * 16 + sizeof(Misc);
static_assert(F_WARPS * 32 == NT, "the replay needs a CTA of NT threads");

// Three CTAs per SM (80 registers): the per-warp replays are latency-bound, so
// more resident warps replay more rows at once.
// Batches of at most this many rows (148 SMs x 3 resident CTAs) get one CTA
// per row: the GPU has room for them, and a tie row then always has a whole
// CTA to replay it, which is faster for a lone row than a warp.
constexpr int64_t FINISH_ONE_ROW_PER_CTA = 444;

__device__ __forceinline__ int finish_rows_per_cta(int64_t rows) {
    return rows <= FINISH_ONE_ROW_PER_CTA ? 1 : F_WARPS;
}

__global__ void __launch_bounds__(F_WARPS * 32, 3) finish_rows_kernel(Params p) {
    extern __shared__ __align__(128) unsigned char fsmem[];
    __shared__ __align__(16) Ent s_heap[HEAP_SMEM_MAX];
    __shared__ int64_t s_xrow[F_WARPS];
    __shared__ uint32_t s_xflag[F_WARPS];
    __shared__ int s_xn, s_wn;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    FinishWarpSmem& w = reinterpret_cast<FinishWarpSmem*>(fsmem)[warp];
    const int rpc = finish_rows_per_cta(p.rows);
    const int64_t row = warp < rpc ? (int64_t)blockIdx.x * rpc + warp : p.rows;  // p.rows: no row
    if (threadIdx.x == 0) s_xn = s_wn = 0;
#ifdef MXS_PROFILE
    const unsigned long long tl0 = (unsigned long long)globaltimer_ns();
    const long long fw0 = clock64();
#endif
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the streaming grid's lists are complete
#ifdef MXS_PROFILE
    const unsigned long long tl1 = (unsigned long long)globaltimer_ns();
    if (threadIdx.x == 0) {
        atomicMin(&g_fin_tl[0], tl0);
        atomicMin(&g_fin_tl[1], tl1);
        atomicMax(&g_fin_tl[2], tl1);
    }
    if (lane == 0 && row < p.rows) atomicAdd(&g_fin_prof[3], (unsigned long long)(clock64() - fw0));
#endif
    MXS_PROF_BEGIN();
    csync();
    uint32_t flags = 0u, cnt_all = 0u;
    bool full = false;
    const bool need = row < p.rows && finish_row_warp<false>(p, row, w, &flags, &cnt_all, &full);
    if (p.edit_cnt) {
        // Edited rows: every replay in double by the row's own warp; a row
        // with a NaN is left without a draw (next = -1, MXS_ROW_NAN).
        if (need && !(flags & FLAG_NAN)) exact_row_warp_edits(p, row, w);
        if (need && (flags & FLAG_NAN) && lane == 0) p.next[row] = -1;
        return;
    }
    // A row whose list stands for it (no NaN, no overflow, at least k entries)
    // is replayed by its own warp from the list and its chunks' first tiles;
    // the others read the whole row with the CTA.
    if (lane == 0 && need && !full) atomicAdd(&s_wn, 1);
    csync();
    const bool by_warp = s_wn >= p.replay_warp_min;
    if (by_warp && need && !full) {
        exact_row_warp_log(p, row, w, cnt_all);
    }
    if (lane == 0 && need && (full || !by_warp)) {
        const int at = atomicAdd(&s_xn, 1);
        s_xrow[at] = row;
        s_xflag[at] = flags;
    }
    csync();
    Misc& sm = *reinterpret_cast<Misc*>(fsmem + (F_REGION + 15) / 16 * 16);
    const int n = s_xn;
    MXS_PROF_T0(tx);
    for (int i = 0; i < n; ++i)
        exact_row_t<true>(p, s_xrow[i], (s_xflag[i] & FLAG_NAN) ? 1 : 0, fsmem, sm, s_heap);
    MXS_PROF_ADD(7, tx);
    MXS_PROF_COUNT(6, n);
    MXS_PROF_FLUSH();
#ifdef MXS_PROFILE
    if (lane == 0 && row < p.rows) {
        atomicAdd(&g_fin_prof[4], (unsigned long long)(clock64() - fw0));
        atomicAdd(&g_fin_prof[5], 1ull);
    }
    csync();
    if (threadIdx.x == 0) atomicMax(&g_fin_tl[3], (unsigned long long)globaltimer_ns());
#endif
}

#ifdef MXS_PROFILE
extern "C" __attribute__((visibility("default"))) int mxs_prof_read_fin(unsigned long long* host, int clear) {
    if (cudaMemcpyFromSymbol(host, g_fin_prof, sizeof(g_fin_prof)) != cudaSuccess) return -3;
    if (cudaMemcpyFromSymbol(host + 8, g_fin_tl, sizeof(g_fin_tl)) != cudaSuccess) return -3;
    if (clear) {
        static unsigned long long zeros[8];
        static const unsigned long long tl[4] = {~0ull, ~0ull, 0ull, 0ull};
        if (cudaMemcpyToSymbol(g_fin_prof, zeros, sizeof(zeros)) != cudaSuccess) return -3;
        if (cudaMemcpyToSymbol(g_fin_tl, tl, sizeof(tl)) != cudaSuccess) return -3;
    }
    return 0;
}
// Phase counters of the finish kernel's CTA replays (profiling build only).
extern "C" __attribute__((visibility("default"))) int mxs_prof_read_finish(unsigned long long* host, int clear) {
    if (cudaMemcpyFromSymbol(host, g_mxs_prof, sizeof(g_mxs_prof)) != cudaSuccess) return -3;
    if (clear) {
        static unsigned long long zeros[PROF_CTAS][PROF_PHASES];
        if (cudaMemcpyToSymbol(g_mxs_prof, zeros, sizeof(zeros)) != cudaSuccess) return -3;
    }
    return 0;
}
#endif

// MODE_EMIT's second kernel: one warp per row writes the shard's candidate
// list (its own kernel: the branch inside finish_rows_kernel slowed sampling).
__global__ void __launch_bounds__(F_WARPS * 32) emit_rows_kernel(Params p) {
    extern __shared__ __align__(128) unsigned char esmem[];
    FinishWarpSmem* ws = reinterpret_cast<FinishWarpSmem*>(esmem);
    const int warp = threadIdx.x >> 5;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int64_t row = (int64_t)blockIdx.x * F_WARPS + warp;
    if (row < p.rows) emit_row_warp(p, row, ws[warp]);
}

// ---------------------------------------------------------------------------
// Vocab-sharded tie rows. The reference's tie order is the heap process over
// the whole row in column order. Shard 0 holds the row's first columns, so
// rank 0 can run that process over its shard alone (first tiles reread, the
// rest from its streaming lists) and hand on the heap it leaves. A later shard
// s only has to supply, in column order, every logit that could still enter:
// those strictly above the k-th largest logit before them, which is at least
// the k-th largest of any earlier shard (that shard alone holds k logits at or
// above it); the shard lists of the first pass give those values.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(F_WARPS * 32) vocab_replay_emit_kernel(VocabReplayArgs a) {
    extern __shared__ __align__(128) unsigned char vsmem[];
    FinishWarpSmem& w = reinterpret_cast<FinishWarpSmem*>(vsmem)[threadIdx.x >> 5];
    const int lane = threadIdx.x & 31;
    const uint32_t lt = (1u << lane) - 1u;
    const int64_t i = (int64_t)blockIdx.x * F_WARPS + (threadIdx.x >> 5);
    if (i >= a.n) return;
    const int64_t r = a.list[i];
    const int k = a.k;
    const uint32_t bad_bits = FLAG_NAN | FLAG_OVERFLOW | FLAG_TIMEOUT;
    uint32_t flags = 0u;
    uint32_t lc = 0u;
    if (!a.log || (a.p1_flags[(int64_t)a.rank * a.rows + r] & bad_bits)) {
        flags = FLAG_OVERFLOW;
    } else {
        lc = a.log_count[r];
        if (lc > (uint32_t)a.log_cap || lc < (uint32_t)k) flags = FLAG_OVERFLOW;
    }
    const float* x = a.shard + r * a.ld;
    const uint64_t* log = flags ? nullptr : a.log + r * (int64_t)a.log_cap;
    uint64_t* dst = a.out + i * (int64_t)a.cap2;
    const int64_t C = a.cols;
    const int64_t chunk = (int64_t)a.tpc * S_TILE;
    int n_out = 0;
    if (!flags && a.rank == 0) {
        const PairHeap h{w.hp};
        Ent* slot = reinterpret_cast<Ent*>(w.keys);
        for (int j = lane; j < k; j += 32) w.hp[j + 1] = Ent{x[j], j};
        __syncwarp();
        if (lane == 0) pair_build(h, k);
        __syncwarp();
        float r0 = w.hp[1].v;
        for (int c = 0; c < a.S; ++c) {
            const int64_t c0 = c * chunk;
            if (c0 >= C) break;
            const int64_t t1 = min(C, c0 + S_TILE), ce = min(C, c0 + chunk);
            r0 = warp_replay_range(x, C, max(c0, (int64_t)k), t1, h, k, slot, r0);
            __syncwarp();
            r0 = warp_replay_list(log, (int)lc, t1, ce, h, k, slot, r0);
            __syncwarp();
        }
        for (int j = lane; j < k; j += 32)
            dst[j] = ((uint64_t)fkey(w.hp[j + 1].v) << 32) | (uint32_t)(w.hp[j + 1].i + (int32_t)a.col_offset);
        n_out = k;
    } else if (!flags) {
        uint32_t B = 0u;  // largest k-th largest key of the earlier shards
        for (int s2 = 0; s2 < a.rank && !flags; ++s2) {
            const int64_t at = (int64_t)s2 * a.rows + r;
            if (a.p1_flags[at] & bad_bits) {
                flags = FLAG_OVERFLOW;
                break;
            }
            const int n = (int)min(a.p1_count[at], (uint32_t)a.p1_cap);
            const uint64_t* src = a.p1_cand + at * a.p1_cap;
            uint32_t mn = 0xFFFFFFFFu;
            for (int j = lane; j < n; j += 32) mn = min(mn, (uint32_t)(src[j] >> 32));
            mn = __reduce_min_sync(0xffffffffu, mn);
            if (n > 0) B = max(B, mn);
        }
        int cnt = 0;
        auto put = [&](bool take, uint32_t key, int32_t col) {
            const uint32_t bal = __ballot_sync(0xffffffffu, take);
            const int at = cnt + __popc(bal & lt);
            if (take && at < FCAP) {
                w.keys[at] = key;
                w.idx[at] = col;
            }
            cnt += __popc(bal);
        };
        for (int c = 0; c < a.S && !flags; ++c) {
            const int64_t c0 = c * chunk;
            if (c0 >= C) break;
            const int64_t t1 = min(C, c0 + S_TILE), ce = min(C, c0 + chunk);
            // the chunk's first tile from memory, the later tiles from the list
            for (int64_t g = c0; g < t1; g += 128) {
                const int64_t j = g + 4 * lane;
                float4 v{0.f, 0.f, 0.f, 0.f};
                if (j < t1) xload4(x, j, C, v);
                const float e4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const bool in = j + t < t1;
                    const uint32_t key = in ? fkey(e4[t]) : 0u;
                    put(in && key > B && !(e4[t] != e4[t]), key, (int32_t)(j + t));
                }
            }
            for (int j0 = 0; j0 < (int)lc; j0 += 32) {
                const int j = j0 + lane;
                const uint64_t v = j < (int)lc ? log[j] : 0ull;
                const int64_t col = (int64_t)(uint32_t)v;
                put(j < (int)lc && col >= t1 && col < ce && (uint32_t)(v >> 32) > B, (uint32_t)(v >> 32),
                    (int32_t)col);
            }
            __syncwarp();
        }
        if (cnt > a.cap2 || cnt > FCAP) {
            flags = FLAG_OVERFLOW;
        } else {
            // column order: keys (~column << 32 | value key) sorted descending
            constexpr int NS = FCAP / 32;
            uint64_t b[NS];
#pragma unroll
            for (int q = 0; q < NS; ++q) {
                const int j = lane + 32 * q;
                b[q] = j < cnt ? ((uint64_t)(~(uint32_t)w.idx[j]) << 32) | w.keys[j] : 0ull;
            }
            warp_sort_desc<NS>(b);
#pragma unroll
            for (int q = 0; q < NS; ++q) {
                const int j = lane + 32 * q;
                if (j < cnt)
                    dst[j] = ((uint64_t)(uint32_t)b[q] << 32) |
                             (uint32_t)((int32_t)~(uint32_t)(b[q] >> 32) + (int32_t)a.col_offset);
            }
            n_out = cnt;
        }
    }
    if (lane == 0) {
        a.out_count[i] = flags ? 0u : (uint32_t)n_out;
        a.out_flags[i] = flags;
    }
}

__global__ void __launch_bounds__(F_WARPS * 32) vocab_replay_merge_kernel(VocabReplayArgs a, Params d) {
    extern __shared__ __align__(128) unsigned char vsmem[];
    FinishWarpSmem& w = reinterpret_cast<FinishWarpSmem*>(vsmem)[threadIdx.x >> 5];
    const int lane = threadIdx.x & 31;
    const int64_t i = (int64_t)blockIdx.x * F_WARPS + (threadIdx.x >> 5);
    if (i >= a.n) return;
    const int64_t r = a.list[i];
    const int k = a.k;
    uint32_t bad = 0u;
    for (int s2 = 0; s2 < a.world; ++s2) bad |= a.g_flags[(int64_t)s2 * a.n + i];
    if (bad || a.g_count[i] != (uint32_t)k) {
        if (lane == 0) a.need_full[i] = 1u;
        return;
    }
    const PairHeap h{w.hp};
    Ent* slot = reinterpret_cast<Ent*>(w.keys);
    const uint64_t* h0 = a.g_cand + i * (int64_t)a.cap2;  // rank 0's heap, heap order
    for (int j = lane; j < k; j += 32) {
        const uint64_t v = h0[j];
        w.hp[j + 1] = Ent{fkey_inv((uint32_t)(v >> 32)), (int32_t)(uint32_t)v};
    }
    __syncwarp();
    float r0 = w.hp[1].v;
    for (int s2 = 1; s2 < a.world; ++s2) {
        const int64_t at = (int64_t)s2 * a.n + i;
        const int n = (int)min(a.g_count[at], (uint32_t)a.cap2);
        const uint64_t* src = a.g_cand + at * a.cap2;
        for (int j0 = 0; j0 < n; j0 += XSLOT) {
            const int m = min(XSLOT, n - j0);
            for (int j = lane; j < m; j += 32) {
                const uint64_t v = src[j0 + j];
                slot[j] = Ent{fkey_inv((uint32_t)(v >> 32)), (int32_t)(uint32_t)v};
            }
            __syncwarp();
            if (lane == 0) r0 = pair_offer_list(h, k, slot, m, r0);
            r0 = __shfl_sync(0xffffffffu, r0, 0);
        }
    }
    if (lane == 0) pair_sort(h, k);
    __syncwarp();
    for (int j = lane; j < k; j += 32) w.e[j] = w.hp[j + 1];
    __syncwarp();
    warp_draw(d, r, w.e, k, w.pbuf);
    if (lane == 0) a.need_full[i] = 0u;
}

cudaError_t vocab_replay_emit_launch(const VocabReplayArgs& a, cudaStream_t stream) {
    if (a.n == 0) return cudaSuccess;
    vocab_replay_emit_kernel<<<(unsigned)((a.n + F_WARPS - 1) / F_WARPS), F_WARPS * 32,
                               sizeof(FinishWarpSmem) * F_WARPS, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t vocab_replay_merge_launch(const VocabReplayArgs& a, const Params& draw, cudaStream_t stream) {
    if (a.n == 0) return cudaSuccess;
    vocab_replay_merge_kernel<<<(unsigned)((a.n + F_WARPS - 1) / F_WARPS), F_WARPS * 32,
                                sizeof(FinishWarpSmem) * F_WARPS, stream>>>(a, draw);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// The reference's pre-sampler edits (src/api/minxfmr.cpp:2047-2089), one CTA
// per row: the special tokens' logits become -inf; each distinct token among
// the row's last penalty_n accepted tokens gets, in double, the repetition
// penalty (multiplied when <= 0, divided otherwise) and loses
// count * frequency_penalty + presence_penalty. The penalised values go to the
// row's edit list (sorted by column) and their logits to -inf, so the sampler
// sees them only as doubles.
// ---------------------------------------------------------------------------
constexpr int EDIT_MAX = EDIT_WINDOW_MAX;

__global__ void __launch_bounds__(256) edits_kernel(float* logits, int64_t ld, int64_t vocab, const int32_t* special,
                                                    int n_special, const int32_t* hist, int64_t hist_stride,
                                                    const int32_t* hist_len, int repeat_last_n, double rp, double fp,
                                                    double pp, int32_t* edit_col, double* edit_val,
                                                    uint32_t* edit_cnt, int edit_cap) {
    __shared__ int32_t tok[EDIT_MAX];
    __shared__ int wsum[8];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t r = blockIdx.x;
    float* row = logits + r * ld;
    int hl = hist_len ? hist_len[r] : 0;
    hl = (int)min((int64_t)max(hl, 0), hist_stride);
    int pn = repeat_last_n < 0 ? hl : min(repeat_last_n, hl);  // src/api/minxfmr.cpp:2061-2064
    if (!(pn > 0 && (rp != 1.0 || fp != 0.0 || pp != 0.0))) pn = 0;
    pn = min(pn, EDIT_MAX);
    int P = 1;
    while (P < pn) P <<= 1;
    for (int i = tid; i < P; i += blockDim.x)
        tok[i] = i < pn ? hist[r * hist_stride + (hl - pn) + i] : INT32_MAX;
    __syncthreads();
    for (int size = 2; size <= P; size <<= 1) {  // ascending bitonic sort
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < P / 2; i += blockDim.x) {
                const int a = 2 * i - (i & (stride - 1)), b2 = a + stride;
                const bool up = (a & size) == 0;
                const int32_t x = tok[a], y = tok[b2];
                if ((x > y) == up) {
                    tok[a] = y;
                    tok[b2] = x;
                }
            }
            __syncthreads();
        }
    }
    // run starts of distinct in-vocabulary tokens: one edit each
    int base = 0;
    for (int i0 = 0; i0 < pn; i0 += blockDim.x) {
        const int i = i0 + tid;
        const int32_t t = i < pn ? tok[i] : INT32_MAX;
        const bool start = i < pn && (i == 0 || tok[i - 1] != t) && t >= 0 && t < vocab;
        const uint32_t bal = __ballot_sync(0xffffffffu, start);
        if (lane == 0) wsum[warp] = __popc(bal);
        __syncthreads();
        int before = base;
        for (int w2 = 0; w2 < warp; ++w2) before += wsum[w2];
        int total = 0;
        for (int w2 = 0; w2 < 8; ++w2) total += wsum[w2];
        if (start) {
            int j = i + 1;
            while (j < pn && tok[j] == t) ++j;
            const int count = j - i;
            bool masked = false;
            for (int q = 0; q < n_special; ++q) masked |= special[q] == t;
            double logit = masked ? -INFINITY : (double)row[t];
            if (rp != 1.0) logit = (logit <= 0.0) ? logit * rp : logit / rp;
            logit -= (double)count * fp + (count > 0 ? pp : 0.0);
            const int at = before + __popc(bal & ((1u << lane) - 1u));
            if (at < edit_cap) {
                edit_col[r * (int64_t)edit_cap + at] = t;
                edit_val[r * (int64_t)edit_cap + at] = logit;
            }
        }
        __syncthreads();
        base += total;
    }
    if (tid == 0) edit_cnt[r] = (uint32_t)min(base, edit_cap);
    __syncthreads();  // every read of the row is done
    for (int q = tid; q < n_special; q += blockDim.x) {
        const int32_t t = special[q];
        if (t >= 0 && t < vocab) row[t] = -INFINITY;
    }
    for (int i = tid; i < base && i < edit_cap; i += blockDim.x) row[edit_col[r * (int64_t)edit_cap + i]] = -INFINITY;
}

cudaError_t edits_launch(float* logits, int64_t rows, int64_t ld, int64_t vocab, const int32_t* special,
                         int n_special, const int32_t* hist, int64_t hist_stride, const int32_t* hist_len,
                         int repeat_last_n, double rp, double fp, double pp, int32_t* edit_col, double* edit_val,
                         uint32_t* edit_cnt, int edit_cap, cudaStream_t stream) {
    edits_kernel<<<(unsigned)rows, 256, 0, stream>>>(logits, ld, vocab, special, n_special, hist, hist_stride,
                                                    hist_len, repeat_last_n, rp, fp, pp, edit_col, edit_val,
                                                    edit_cnt, edit_cap);
    return cudaGetLastError();
}

size_t stream_smem_bytes() { return S_SMEM; }

cudaError_t merge_rows_launch(const Params& p, cudaStream_t stream) {
    merge_rows_kernel<<<(unsigned)((p.rows + F_WARPS - 1) / F_WARPS), F_WARPS * 32, sizeof(FinishWarpSmem) * F_WARPS,
                        stream>>>(p);
    return cudaGetLastError();
}

cudaError_t stream_path_configure(int* blocks_per_sm) {
    cudaError_t e = cudaFuncSetAttribute(stream_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S_SMEM);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(finish_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)F_SMEM);
    if (e != cudaSuccess) return e;
    for (const void* f : {(const void*)merge_rows_kernel, (const void*)vocab_replay_emit_kernel,
                          (const void*)vocab_replay_merge_kernel, (const void*)emit_rows_kernel}) {
        e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(sizeof(FinishWarpSmem) * F_WARPS));
        if (e != cudaSuccess) return e;
    }
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, stream_select_kernel, NT_WS, S_SMEM);
}

cudaError_t stream_path_launch(const Params& p, int grid, cudaStream_t stream, cudaEvent_t ev_start,
                               cudaEvent_t ev_stop) {
    if (ev_start) cudaEventRecord(ev_start, stream);
    stream_select_kernel<<<grid, NT_WS, S_SMEM, stream>>>(p);
    cudaError_t e = cudaGetLastError();
    if (ev_stop) cudaEventRecord(ev_stop, stream);
    if (e != cudaSuccess) return e;
    if (p.mode == MODE_EMIT) {
        emit_rows_kernel<<<(unsigned)((p.rows + F_WARPS - 1) / F_WARPS), F_WARPS * 32, sizeof(FinishWarpSmem) * F_WARPS,
                           stream>>>(p);
        return cudaGetLastError();
    }
    const int64_t rpc = p.rows <= FINISH_ONE_ROW_PER_CTA ? 1 : F_WARPS;
    // Programmatic dependent launch: the finish grid is launched while the
    // streaming grid runs and its CTAs wait (griddepcontrol.wait) for it to
    // complete, which hides the launch gap between the two kernels. With a
    // profiling event recorded between them it is an ordinary launch.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((p.rows + rpc - 1) / rpc));
    cfg.blockDim = dim3(F_WARPS * 32);
    cfg.dynamicSmemBytes = F_SMEM;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = ev_stop ? 0 : 1;
    return cudaLaunchKernelEx(&cfg, finish_rows_kernel, p);
}

}  // namespace mxs
