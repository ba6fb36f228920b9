// The fused sampling kernel: temperature -> top-k -> softmax over the k
// survivors -> inverse-CDF draw, for rows of fp32 logits resident in HBM.
//
// Reference path: src/api/minxfmr.cpp:2091-2171 (minxfmr_generate's sampling
// block). Result contract: top-k index set, tie order and sampled id identical
// to that block on the same logits and the same uniform u; probabilities from
// the same double-precision operations in the same order.
//
// Work decomposition. A row of V logits is cut into S chunks of whole TILEs
// (S = 1 when there are enough rows to fill the GPU). A persistent grid of CTAs
// walks its (row, chunk) units; one elected thread streams every tile of every
// unit through a STAGES-deep ring of bulk copies (cp.async.bulk, completion on
// mbarriers), so the next unit's loads are already in flight while a unit
// finishes. Consumers compare each logit against a running threshold (the k-th
// largest key of the candidates so far, which never exceeds the row's k-th
// largest value) and append survivors to a shared-memory candidate buffer; when
// the buffer fills, a block radix-select raises the threshold and compacts it.
//
// Finishing a row (the CTA of an S = 1 unit, or the last CTA to finish a chunk
// of the row when S > 1, which merges the chunks' candidate lists):
//   - keep the candidates >= the k-th largest key; if more than k remain, a
//     tie straddles the cut;
//   - sort the k survivors by value; equal neighbours mean a tie inside;
//   - no tie: the order is the unique descending order and the draw runs;
//   - a tie, a NaN in the row or a candidate overflow: the CTA replays the
//     reference's heap process over the row (mxs_heap.cuh), reading only the
//     logits that can still enter the heap (those above the heap root at the
//     start of each XTILE step; the root only grows), then draws.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "mxs_common.cuh"
#include "mxs_heap.cuh"

namespace mxs {

struct Params {
    const float* logits;
    int64_t rows, vocab, ld;
    double temperature, top_p, min_p;
    int k_use;
    const double* u;
    int32_t* next;
    int32_t* topk_idx;     // rows x k_use, nullable
    double* topk_prob;     // rows x k_use, nullable
    uint32_t* row_flags;   // rows, nullable
    // schedule
    int S;                 // chunks per row
    int tiles_per_chunk;   // TILEs per chunk (last chunk may hold fewer)
    int64_t units;         // rows * S
    int outcap;            // candidate capacity of one chunk list (S > 1)
    // workspace
    uint32_t* row_counter; // rows: chunks finished (self-resetting)
    uint32_t* row_state;   // rows: OR of chunk flags (self-resetting)
    uint32_t* chunk_count; // rows * S
    uint64_t* chunk_cand;  // rows * S * outcap, (key << 32) | index
    Ent* heap_ws;          // gridDim.x * k_use when k_use > HEAP_SMEM_MAX
    double* prob_ws;       // gridDim.x * k_use when k_use > HEAP_SMEM_MAX
    uint32_t* status;      // OR of every row's flags
    // vocab-sharded modes
    int mode;              // MODE_SAMPLE, MODE_EMIT (shard candidate lists) or MODE_MERGE
    int64_t col_offset;    // MODE_EMIT: global column of the shard's column 0
    uint64_t* out_cand;    // MODE_EMIT: rows x out_cap
    uint32_t* out_count;   // MODE_EMIT: rows
    uint32_t* out_flags;   // MODE_EMIT: rows
    int out_cap;
    uint32_t* log_count;   // MODE_EMIT on the two-kernel path: rows, the streaming list's length (nullable)
    const uint64_t* in_cand;   // MODE_MERGE: nshards x rows x in_cap
    const uint32_t* in_count;  // MODE_MERGE: nshards x rows
    const uint32_t* in_flags;  // MODE_MERGE: nshards x rows (nullable)
    int nshards, in_cap;
    // two-kernel path (k <= KSPLIT): stream -> per-row candidate lists -> finish (+ replay)
    uint64_t* row_cand;        // rows x row_cap, (key << 32) | column
    uint32_t* row_cnt;         // rows: entries appended (may exceed row_cap: overflow)
    uint32_t* row_flag;        // rows: OR of FLAG_* seen while streaming
    uint32_t* row_bound;       // rows: key of a lower bound of the row's k-th largest logit, from the
                               // streaming warps (0: none); cleared by the finish kernel
    int row_cap;
    // pre-sampler edits (mxs_sample_topk_edits): per row, every penalised
    // token's exact double value, sorted by column (their logits read -inf in
    // the row, so the streaming pass never lists them); null edit_cnt: none
    const int32_t* edit_col;   // rows x edit_cap
    const double* edit_val;    // rows x edit_cap
    const uint32_t* edit_cnt;  // rows
    int edit_cap;
    int replay_warp_min;       // the finish kernel replays tie rows one per warp when its CTA holds at
                               // least this many of them, else with the whole CTA (MXS_REPLAY_WARP_MIN)
    int64_t debug_drop_tile;   // test hook (MXS_DEBUG_DROP_TILE): the streaming producer stops before
                               // the CTA-0 tile with this sequence number; -1 = off
};
constexpr int MODE_SAMPLE = 0;
constexpr int MODE_EMIT = 1;
constexpr int MODE_MERGE = 2;

// Shared memory: the bulk-copy ring, then a 32 KB region used in turn as the
// candidate buffer (keys | indices), the sort buffer + probabilities, or the
// exact path's heap + replay list, then small scalars.
struct Misc {
    uint64_t bar[STAGES];   // stage full (bytes landed)
    uint64_t ebar[STAGES];  // stage empty (every consumer warp is done with it)
    uint32_t thr_key;       // running threshold key shared by the consumer warps
    uint32_t pub[NWARPS];   // per consumer warp: the m-th largest key it has held (m = ceil(k / NWARPS))
    uint32_t hist[256];
    int warp_tot[NWARPS];
    uint32_t warp_or[NWARPS];
    int cnt;
    float thr;
    uint32_t digit;
    int krem;
    int last;
    uint32_t flags;
    int xn;
    double sum;
    int32_t pick_next;
    uint32_t dead;          // a bounded wait ran out: no more copies are issued
};
constexpr size_t RING_BYTES = size_t(STAGES) * TILE * sizeof(float);
constexpr size_t REGION_BYTES = size_t(CAP) * 8;
constexpr size_t SMEM_BYTES = RING_BYTES + REGION_BYTES + sizeof(Misc);
// The streaming kernel of the two-kernel path: 8 consumer warps + 1 producer warp.
constexpr int NT_WS = NT + 32;
static_assert(SORTMAX * 8 + KFAST * 8 <= REGION_BYTES, "sort + prob buffers exceed the region");
static_assert(HEAP_SMEM_MAX * 8 + XTILE * 8 <= REGION_BYTES, "heap + replay list exceed the region");

// ---------------------------------------------------------------------------
// Block primitives (all threads of the CTA call them together).
// ---------------------------------------------------------------------------

// Append up to 4 entries per thread (bit q of `m` set = entry q present) to the
// candidate buffer; warp-aggregated: one shared atomic per warp.
__device__ __forceinline__ void block_append4(uint32_t* ckey, int32_t* cidx, Misc& sm, uint32_t m,
                                              const uint32_t (&key)[4], const int32_t (&idx)[4]) {
    const int c = __popc(m);
    if (!__any_sync(0xffffffffu, c)) return;
    const int lane = threadIdx.x & 31;
    const int incl = warp_incl_scan(c);
    int base = 0;
    if (lane == 31 && incl) base = atomicAdd(&sm.cnt, incl);
    base = __shfl_sync(0xffffffffu, base, 31);
    int pos = base + incl - c;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        if (m & (1u << q)) {
            if (pos < CAP) {
                ckey[pos] = key[q];
                cidx[pos] = idx[q];
            }
            ++pos;
        }
    }
}

// Append the logits of a 16-logit group (bit 4q+c of m set = component c of
// f[q] passes; its column is i0 + 4*NT*q + c), warp-aggregated.
__device__ __forceinline__ void block_append16(uint32_t* ckey, int32_t* cidx, Misc& sm, uint32_t m,
                                               const float4 (&f)[4], int32_t i0) {
    const int c = __popc(m);
    if (!__any_sync(0xffffffffu, c)) return;
    const int lane = threadIdx.x & 31;
    const int incl = warp_incl_scan(c);
    int base = 0;
    if (lane == 31 && incl) base = atomicAdd(&sm.cnt, incl);
    base = __shfl_sync(0xffffffffu, base, 31);
    int pos = base + incl - c;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float vv[4] = {f[q].x, f[q].y, f[q].z, f[q].w};
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
            if (m & (1u << (4 * q + c4))) {
                if (pos < CAP) {
                    ckey[pos] = fkey(vv[c4]);
                    cidx[pos] = i0 + 4 * NT * q + c4;
                }
                ++pos;
            }
        }
    }
}

// AND and OR of all keys in ckey[0, cnt) (block-wide).
__device__ __forceinline__ void block_and_or(const uint32_t* ckey, int cnt, Misc& sm, uint32_t* a_out,
                                             uint32_t* o_out) {
    uint32_t a = ~0u, o = 0u;
    for (int i = threadIdx.x; i < cnt; i += NT) {
        const uint32_t key = ckey[i];
        a &= key;
        o |= key;
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
        a &= __shfl_xor_sync(0xffffffffu, a, d);
        o |= __shfl_xor_sync(0xffffffffu, o, d);
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        sm.warp_tot[w] = (int)a;
        sm.warp_or[w] = o;
    }
    csync();
    a = ~0u;
    o = 0u;
#pragma unroll
    for (int i = 0; i < NWARPS; ++i) {
        a &= (uint32_t)sm.warp_tot[i];
        o |= sm.warp_or[i];
    }
    csync();
    *a_out = a;
    *o_out = o;
}

// k-th largest key among ckey[0, cnt), 1 <= k <= cnt. Radix select from the
// most significant bit in which the keys differ, at most 8 bits per pass; lanes
// of a warp that hit the same bin add once (match_any), so a narrow key range
// does not serialise the shared-memory atomics.
__device__ inline uint32_t block_select_kth(const uint32_t* ckey, int cnt, int k, Misc& sm) {
    const int tid = threadIdx.x, lane = tid & 31;
    uint32_t a, o;
    block_and_or(ckey, cnt, sm, &a, &o);
    const uint32_t diff = a ^ o;
    if (diff == 0) return a;  // all keys equal
    int hi = 31 - __clz(diff);  // highest undecided bit
    uint32_t prefix = a & ~((2u << hi) - 1u);
    uint32_t mask = ~((2u << hi) - 1u);
    int krem = k;
#pragma unroll 1
    while (hi >= 0) {
        const int w = min(8, hi + 1);
        const int shift = hi + 1 - w;
        const int nb = 1 << w;
        sm.hist[tid] = 0;
        csync();
        for (int i0 = 0; i0 < cnt; i0 += NT) {
            const int i = i0 + tid;
            int bin = -1;
            if (i < cnt) {
                const uint32_t key = ckey[i];
                if ((key & mask) == prefix) bin = (int)((key >> shift) & (uint32_t)(nb - 1));
            }
            const uint32_t same = __match_any_sync(0xffffffffu, bin);
            if (bin >= 0 && lane == __ffs(same) - 1) atomicAdd(&sm.hist[bin], (uint32_t)__popc(same));
        }
        csync();
        if (tid < 32) {
            // lane l owns bins nb-1-l*per .. nb-per-l*per, scanned from the top down
            const int per = (nb + 31) / 32;
            int own = 0;
            for (int b = 0; b < per; ++b) {
                const int bin = nb - 1 - lane * per - b;
                if (bin >= 0) own += (int)sm.hist[bin];
            }
            const int incl = warp_incl_scan(own);
            const int excl = incl - own;
            if (excl < krem && incl >= krem) {
                int run = excl;
                for (int b = 0; b < per; ++b) {
                    const int bin = nb - 1 - lane * per - b;
                    const int h = (int)sm.hist[bin];
                    if (run + h >= krem) {
                        sm.digit = (uint32_t)bin;
                        sm.krem = krem - run;
                        break;
                    }
                    run += h;
                }
            }
        }
        csync();
        prefix |= sm.digit << shift;
        mask |= (uint32_t)(nb - 1) << shift;
        krem = sm.krem;
        hi = shift - 1;
    }
    return prefix;
}

// ---------------------------------------------------------------------------
// Warp primitives of the warp-specialised streaming path (one warp, no CTA sync).
// ---------------------------------------------------------------------------

// k-th largest key among keys[0, n), 1 <= k <= n, by one warp; hist: 256 words
// private to the warp.
__device__ inline uint32_t warp_select_kth(const uint32_t* keys, int n, int k, uint32_t* hist) {
    const int lane = threadIdx.x & 31;
    uint32_t a = ~0u, o = 0u;
    for (int i = lane; i < n; i += 32) {
        const uint32_t key = keys[i];
        a &= key;
        o |= key;
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
        a &= __shfl_xor_sync(0xffffffffu, a, d);
        o |= __shfl_xor_sync(0xffffffffu, o, d);
    }
    const uint32_t diff = a ^ o;
    if (diff == 0) return a;
    int hi = 31 - __clz(diff);
    uint32_t prefix = a & ~((2u << hi) - 1u);
    uint32_t mask = ~((2u << hi) - 1u);
    int krem = k;
#pragma unroll 1
    while (hi >= 0) {
        const int w = min(8, hi + 1);
        const int shift = hi + 1 - w;
        const int nb = 1 << w;
        for (int b = lane; b < 256; b += 32) hist[b] = 0;
        __syncwarp();
        for (int i0 = 0; i0 < n; i0 += 32) {
            const int i = i0 + lane;
            int bin = -1;
            if (i < n) {
                const uint32_t key = keys[i];
                if ((key & mask) == prefix) bin = (int)((key >> shift) & (uint32_t)(nb - 1));
            }
            const uint32_t same = __match_any_sync(0xffffffffu, bin);
            if (bin >= 0 && lane == __ffs(same) - 1) atomicAdd(&hist[bin], (uint32_t)__popc(same));
        }
        __syncwarp();
        const int per = (nb + 31) / 32;
        int own = 0;
        for (int b = 0; b < per; ++b) {
            const int bin = nb - 1 - lane * per - b;
            if (bin >= 0) own += (int)hist[bin];
        }
        const int incl = warp_incl_scan(own);
        const int excl = incl - own;
        const bool mine = (excl < krem && incl >= krem);
        int d = 0, kr = 0;
        if (mine) {
            int run = excl;
            for (int b = 0; b < per; ++b) {
                const int bin = nb - 1 - lane * per - b;
                const int h = (int)hist[bin];
                if (run + h >= krem) {
                    d = bin;
                    kr = krem - run;
                    break;
                }
                run += h;
            }
        }
        const int src = __ffs(__ballot_sync(0xffffffffu, mine)) - 1;
        d = __shfl_sync(0xffffffffu, d, src);
        kr = __shfl_sync(0xffffffffu, kr, src);
        prefix |= (uint32_t)d << shift;
        mask |= (uint32_t)(nb - 1) << shift;
        krem = kr;
        hi = shift - 1;
        __syncwarp();
    }
    return prefix;
}

// Keep the entries of keys/idx[0, n) with key >= kth, in place, in order; one warp.
__device__ __forceinline__ int warp_compact_ge(uint32_t* keys, int32_t* idx, int n, uint32_t kth) {
    const int lane = threadIdx.x & 31;
    const uint32_t lt = (1u << lane) - 1u;
    int out = 0;
    for (int i0 = 0; i0 < n; i0 += 32) {
        const int i = i0 + lane;
        uint32_t kk = 0;
        int32_t ii = 0;
        bool keep = false;
        if (i < n) {
            kk = keys[i];
            ii = idx[i];
            keep = kk >= kth;
        }
        const uint32_t bal = __ballot_sync(0xffffffffu, keep);
        if (keep) {
            const int pos = out + __popc(bal & lt);
            keys[pos] = kk;
            idx[pos] = ii;
        }
        out += __popc(bal);
    }
    __syncwarp();
    return out;
}

// Sort 64 packed entries held two per lane (a0 = element lane, a1 = element
// lane + 32) descending, with a register bitonic network (warp-synchronous).
__device__ __forceinline__ void warp_sort64_desc(uint64_t& a0, uint64_t& a1) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int size = 2; size <= 64; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride == 32) {
                const bool desc = ((lane & size) == 0);
                if ((a0 < a1) == desc) {
                    const uint64_t t = a0;
                    a0 = a1;
                    a1 = t;
                }
            } else {
#pragma unroll
                for (int slot = 0; slot < 2; ++slot) {
                    uint64_t& v = slot ? a1 : a0;
                    const int i = lane + 32 * slot;
                    const uint64_t o = __shfl_xor_sync(0xffffffffu, v, stride);
                    const bool desc = ((i & size) == 0);
                    const bool keep_max = (desc == ((i & stride) == 0));
                    v = keep_max ? (v > o ? v : o) : (v < o ? v : o);
                }
            }
        }
    }
}

// Keep the candidates with key >= kth; returns the new count.
__device__ inline int block_compact_ge(uint32_t* ckey, int32_t* cidx, Misc& sm, int cnt, uint32_t kth) {
    constexpr int PER = CAP / NT;
    uint32_t kk[PER];
    int32_t ii[PER];
    uint32_t keep = 0;
#pragma unroll
    for (int r = 0; r < PER; ++r) {
        const int i = threadIdx.x + r * NT;
        kk[r] = 0;
        ii[r] = 0;
        if (i < cnt) {
            kk[r] = ckey[i];
            ii[r] = cidx[i];
            if (kk[r] >= kth) keep |= 1u << r;
        }
    }
    csync();
    if (threadIdx.x == 0) sm.cnt = 0;
    csync();
#pragma unroll
    for (int r = 0; r < PER; r += 4) {
        const uint32_t m = (keep >> r) & 0xFu;
        const uint32_t k4[4] = {kk[r], kk[r + 1], kk[r + 2], kk[r + 3]};
        const int32_t i4[4] = {ii[r], ii[r + 1], ii[r + 2], ii[r + 3]};
        block_append4(ckey, cidx, sm, m, k4, i4);
    }
    csync();
    return sm.cnt;
}

// Sort 32*NS packed entries held NS per lane (slot s of lane l = element
// l + 32 s) descending, with a register bitonic network (warp-synchronous).
template <int NS>
__device__ __forceinline__ void warp_sort_desc(uint64_t (&a)[NS]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int size = 2; size <= 32 * NS; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride >= 32) {
                const int ss = stride / 32;
#pragma unroll
                for (int s = 0; s < NS; ++s) {
                    if ((s & ss) == 0) {
                        const int i = lane + 32 * s;
                        const bool desc = ((i & size) == 0);
                        const uint64_t x = a[s], y = a[s + ss];
                        if ((x < y) == desc) {
                            a[s] = y;
                            a[s + ss] = x;
                        }
                    }
                }
            } else {
#pragma unroll
                for (int s = 0; s < NS; ++s) {
                    const int i = lane + 32 * s;
                    const uint64_t o = __shfl_xor_sync(0xffffffffu, a[s], stride);
                    const bool desc = ((i & size) == 0);
                    const bool keep_max = (desc == ((i & stride) == 0));
                    a[s] = keep_max ? (a[s] > o ? a[s] : o) : (a[s] < o ? a[s] : o);
                }
            }
        }
    }
}

// Sort a[0, P) descending, P a power of two <= SORTMAX (bitonic network).
__device__ inline void block_sort_desc(uint64_t* a, int P) {
    if (P <= 64) {
        if (threadIdx.x < 32) {
            for (int size = 2; size <= P; size <<= 1) {
                for (int stride = size >> 1; stride > 0; stride >>= 1) {
                    for (int t = threadIdx.x; t < P / 2; t += 32) {
                        const int lo = 2 * t - (t & (stride - 1));
                        const int hi = lo + stride;
                        const bool desc = ((lo & size) == 0);
                        const uint64_t x = a[lo], y = a[hi];
                        if ((x < y) == desc) {
                            a[lo] = y;
                            a[hi] = x;
                        }
                    }
                    __syncwarp();
                }
            }
        }
        csync();
        return;
    }
    for (int size = 2; size <= P; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int t = threadIdx.x; t < P / 2; t += NT) {
                const int lo = 2 * t - (t & (stride - 1));
                const int hi = lo + stride;
                const bool desc = ((lo & size) == 0);
                const uint64_t x = a[lo], y = a[hi];
                if ((x < y) == desc) {
                    a[lo] = y;
                    a[hi] = x;
                }
            }
            csync();
        }
    }
}

// Exclusive block scan of one int per thread; returns the exclusive prefix and
// writes the total to *total.
__device__ __forceinline__ int block_excl_scan(int v, Misc& sm, int* total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int incl = warp_incl_scan(v);
    if (lane == 31) sm.warp_tot[w] = incl;
    csync();
    int off = 0, tot = 0;
#pragma unroll
    for (int i = 0; i < NWARPS; ++i) {
        const int t = sm.warp_tot[i];
        off += (i < w) ? t : 0;
        tot += t;
    }
    csync();
    *total = tot;
    return off + incl - v;
}

}  // namespace mxs
