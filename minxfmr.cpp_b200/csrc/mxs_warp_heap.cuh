// A heap of at most 64 entries held in one warp's registers (node n in lane
// n % 32, slot n / 32), with the same operations and the same resulting
// arrangement as the serial emulation in mxs_heap.cuh.
//
// One replacement ("place entry e at hole `top` of a heap of `len`") in the
// serial form moves the hole from `top` down to a leaf, always into the child
// that does not come "before" its sibling, shifting each child on that path up
// one level, then lets e rise from the leaf while the parent holds a strictly
// greater value. Without NaNs the values along any root-to-leaf path are
// non-decreasing (a parent never holds a greater value than its child), so the
// result is: the path loses its top value, and e is inserted into the path just
// after every value <= e. The warp follows the path with shuffles, one level at
// a time, and then rewrites only the path's nodes. Rows holding NaNs must use
// the serial form (no order, no monotone path).
#pragma once

#include <cstdint>

#include "mxs_heap.cuh"

namespace mxs {

constexpr int WHEAP_MAX = 64;
constexpr int WHEAP_DEPTH = 6;  // levels below any node of a 64-entry heap

struct WarpHeap {
    uint64_t s0, s1;  // nodes lane and lane + 32: (float bits << 32) | index
};

__device__ __forceinline__ uint64_t wh_pack(float v, int32_t i) {
    return ((uint64_t)__float_as_uint(v) << 32) | (uint32_t)i;
}
__device__ __forceinline__ float wh_val(uint64_t w) { return __uint_as_float((uint32_t)(w >> 32)); }
__device__ __forceinline__ int32_t wh_idx(uint64_t w) { return (int32_t)(uint32_t)w; }

// Node n (warp-uniform n) broadcast to every lane.
__device__ __forceinline__ uint64_t wh_get(const WarpHeap& h, int n) {
    return __shfl_sync(0xffffffffu, n < 32 ? h.s0 : h.s1, n & 31);
}
__device__ __forceinline__ void wh_set(WarpHeap& h, int n, uint64_t w) {
    if ((n & 31) == (int)(threadIdx.x & 31)) {
        if (n < 32)
            h.s0 = w;
        else
            h.s1 = w;
    }
}

// Place entry e at hole `top` of the heap h[0, len) (all arguments warp-uniform).
__device__ __forceinline__ void wh_place(WarpHeap& h, int top, int len, uint64_t e) {
    int pn[WHEAP_DEPTH + 1];
    uint64_t pw[WHEAP_DEPTH + 1];
    pn[0] = top;
    pw[0] = wh_get(h, top);
    int d = 0, n = top;
    const int inner = (len - 1) / 2;
    const bool even = (len & 1) == 0;
    bool go = true;
#pragma unroll
    for (int s = 1; s <= WHEAP_DEPTH; ++s) {
        int nn = -1;
        uint64_t nw = 0;
        if (go) {
            if (n < inner) {  // two children: the right one unless it holds the greater value
                const uint64_t l = wh_get(h, 2 * n + 1);
                const uint64_t r = wh_get(h, 2 * n + 2);
                const bool take_left = wh_val(r) > wh_val(l);
                nn = take_left ? 2 * n + 1 : 2 * n + 2;
                nw = take_left ? l : r;
            } else if (even && n == inner) {  // the last parent of an even-length heap: one child
                nn = 2 * n + 1;
                nw = wh_get(h, nn);
            }
        }
        if (nn >= 0) {
            pn[s] = nn;
            pw[s] = nw;
            d = s;
            n = nn;
            if (nn >= inner && !(even && nn == inner)) go = false;
        } else {
            go = false;
            pn[s] = -1;
            pw[s] = 0;
        }
    }
    // e goes after every shifted path value <= e
    const float ev = wh_val(e);
    int p = 0;
#pragma unroll
    for (int j = 1; j <= WHEAP_DEPTH; ++j)
        if (j <= d && wh_val(pw[j]) <= ev) p = j;
#pragma unroll
    for (int j = 0; j <= WHEAP_DEPTH; ++j) {
        if (j <= d) {
            const uint64_t w = (j < WHEAP_DEPTH && j < p) ? pw[j < WHEAP_DEPTH ? j + 1 : j] : (j == p ? e : pw[j]);
            wh_set(h, pn[j], w);
        }
    }
}

// Load h[0, len) from an Ent array (any lanes' entries beyond len are unused).
__device__ __forceinline__ void wh_load(WarpHeap& h, const Ent* src, int len) {
    const int lane = threadIdx.x & 31;
    h.s0 = lane < len ? wh_pack(src[lane].v, src[lane].i) : 0ull;
    h.s1 = lane + 32 < len ? wh_pack(src[lane + 32].v, src[lane + 32].i) : 0ull;
}
__device__ __forceinline__ void wh_store(const WarpHeap& h, Ent* dst, int len) {
    const int lane = threadIdx.x & 31;
    if (lane < len) dst[lane] = Ent{wh_val(h.s0), wh_idx(h.s0)};
    if (lane + 32 < len) dst[lane + 32] = Ent{wh_val(h.s1), wh_idx(h.s1)};
}

__device__ __forceinline__ void wh_build(WarpHeap& h, int len) {
    if (len < 2) return;
    for (int p = (len - 2) / 2; p >= 0; --p) wh_place(h, p, len, wh_get(h, p));
}

// Offer e: replaces the root when e holds a strictly greater value.
__device__ __forceinline__ void wh_offer(WarpHeap& h, int len, uint64_t e) {
    const uint64_t root = wh_get(h, 0);
    if (wh_val(e) > wh_val(root)) wh_place(h, 0, len, e);
}

__device__ __forceinline__ void wh_sort(WarpHeap& h, int len) {
    while (len > 1) {
        --len;
        const uint64_t e = wh_get(h, len);
        wh_set(h, len, wh_get(h, 0));
        wh_place(h, 0, len, e);
    }
}

}  // namespace mxs
