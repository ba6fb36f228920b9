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
    const uint64_t* in_cand;   // MODE_MERGE: nshards x rows x in_cap
    const uint32_t* in_count;  // MODE_MERGE: nshards x rows
    const uint32_t* in_flags;  // MODE_MERGE: nshards x rows (nullable)
    int nshards, in_cap;
};
constexpr int MODE_SAMPLE = 0;
constexpr int MODE_EMIT = 1;
constexpr int MODE_MERGE = 2;

// Shared memory: the bulk-copy ring, then a 32 KB region used in turn as the
// candidate buffer (keys | indices), the sort buffer + probabilities, or the
// exact path's heap + replay list, then small scalars.
struct Misc {
    uint64_t bar[STAGES];
    uint32_t hist[256];
    int warp_tot[NWARPS];
    int cnt;
    float thr;
    uint32_t digit;
    int krem;
    int last;
    uint32_t flags;
    int xn;
    double sum;
    int32_t pick_next;
};
constexpr size_t RING_BYTES = size_t(STAGES) * TILE * sizeof(float);
constexpr size_t REGION_BYTES = size_t(CAP) * 8;
constexpr size_t SMEM_BYTES = RING_BYTES + REGION_BYTES + sizeof(Misc);
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

// k-th largest key among ckey[0, cnt), 1 <= k <= cnt: four 8-bit digit passes.
__device__ inline uint32_t block_select_kth(const uint32_t* ckey, int cnt, int k, Misc& sm) {
    const int tid = threadIdx.x;
    uint32_t prefix = 0, mask = 0;
    int krem = k;
#pragma unroll 1
    for (int shift = 24; shift >= 0; shift -= 8) {
        sm.hist[tid] = 0;
        __syncthreads();
        for (int i = tid; i < cnt; i += NT) {
            const uint32_t key = ckey[i];
            if ((key & mask) == prefix) atomicAdd(&sm.hist[(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (tid < 32) {
            // lane l owns bins 255-8l .. 248-8l, scanned from the top down
            int own = 0;
#pragma unroll
            for (int b = 0; b < 8; ++b) own += (int)sm.hist[255 - 8 * tid - b];
            const int incl = warp_incl_scan(own);
            const int excl = incl - own;
            if (excl < krem && incl >= krem) {
                int run = excl;
                for (int b = 0; b < 8; ++b) {
                    const int bin = 255 - 8 * tid - b;
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
        __syncthreads();
        prefix |= sm.digit << shift;
        mask |= 0xFFu << shift;
        krem = sm.krem;
    }
    return prefix;
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
    __syncthreads();
    if (threadIdx.x == 0) sm.cnt = 0;
    __syncthreads();
#pragma unroll
    for (int r = 0; r < PER; r += 4) {
        const uint32_t m = (keep >> r) & 0xFu;
        const uint32_t k4[4] = {kk[r], kk[r + 1], kk[r + 2], kk[r + 3]};
        const int32_t i4[4] = {ii[r], ii[r + 1], ii[r + 2], ii[r + 3]};
        block_append4(ckey, cidx, sm, m, k4, i4);
    }
    __syncthreads();
    return sm.cnt;
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
        __syncthreads();
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
            __syncthreads();
        }
    }
}

// Exclusive block scan of one int per thread; returns the exclusive prefix and
// writes the total to *total.
__device__ __forceinline__ int block_excl_scan(int v, Misc& sm, int* total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int incl = warp_incl_scan(v);
    if (lane == 31) sm.warp_tot[w] = incl;
    __syncthreads();
    int off = 0, tot = 0;
#pragma unroll
    for (int i = 0; i < NWARPS; ++i) {
        const int t = sm.warp_tot[i];
        off += (i < w) ? t : 0;
        tot += t;
    }
    __syncthreads();
    *total = tot;
    return off + incl - v;
}

}  // namespace mxs
