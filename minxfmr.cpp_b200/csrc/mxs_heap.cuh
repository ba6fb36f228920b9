// Device emulation of the heap process behind std::partial_sort (libstdc++ 13),
// which the reference sampler calls at src/api/minxfmr.cpp:2099-2102 with the
// comparator "logits[a] > logits[b]". The tie order of the reference's top-k is
// whatever this heap process leaves, so it is reproduced step for step:
//
//   select: build a heap over the first k entries (Floyd order: parents from
//           (k-2)/2 down to 0); then for i = k .. V-1, if x[i] is strictly
//           greater than the root (the smallest kept value), the root is
//           replaced by entry i;
//   sort:   repeatedly swap the root to the end of the shrinking heap.
//
// Every replacement moves a hole from the start position down to a leaf,
// always into the child that does not come "before" its sibling (the right
// child unless it holds a strictly greater value than the left), then lets the
// new entry rise from that leaf while its parent holds a strictly greater value.
// Written from that description of the algorithm (GCC's bits/stl_heap.h,
// __adjust_heap / __push_heap / __make_heap / __sort_heap, bits/stl_algo.h:1631
// __heap_select); the oracle's own restatement is checked against the real
// std::partial_sort in the CPU tests and this device code against the oracle in
// the GPU tests.
#pragma once

#include <cstdint>

namespace mxs {

// 8-byte aligned: the heap's shared-memory accesses move an entry as one
// 8-byte (or a pair as one 16-byte) load or store.
struct __align__(8) Ent {
    float v;
    int32_t i;
};

// "a comes before b" in the reference's order: a holds the strictly greater value.
__device__ __forceinline__ bool before(float a, float b) { return a > b; }

// Heap over h[0, len) (generic pointer: shared or global memory). Serial: one
// thread runs these.
__device__ __forceinline__ void heap_sift_up(Ent* h, int hole, int top, Ent e) {
    int parent = (hole - 1) / 2;
    while (hole > top && before(h[parent].v, e.v)) {
        h[hole] = h[parent];
        hole = parent;
        parent = (hole - 1) / 2;
    }
    h[hole] = e;
}

__device__ __forceinline__ void heap_place(Ent* h, int hole, int len, Ent e) {
    const int top = hole;
    int c = hole;
    const int inner = (len - 1) / 2;
    while (c < inner) {
        c = 2 * (c + 1);
        const Ent r = h[c];
        const Ent l = h[c - 1];
        if (before(r.v, l.v)) {
            c--;
            h[hole] = l;
        } else {
            h[hole] = r;
        }
        hole = c;
    }
    if ((len & 1) == 0 && c == (len - 2) / 2) {
        c = 2 * (c + 1);
        h[hole] = h[c - 1];
        hole = c - 1;
    }
    heap_sift_up(h, hole, top, e);
}

__device__ __forceinline__ void heap_build(Ent* h, int len) {
    if (len < 2) return;
    for (int p = (len - 2) / 2;; --p) {
        heap_place(h, p, len, h[p]);
        if (p == 0) break;
    }
}

// Offer entry e (index > every index already offered): replaces the root when
// e's value is strictly greater than the root's.
__device__ __forceinline__ void heap_offer(Ent* h, int len, Ent e) {
    if (before(e.v, h[0].v)) heap_place(h, 0, len, e);
}

// After this, h[0, len) is in the reference's top-k order (greatest first).
__device__ __forceinline__ void heap_sort(Ent* h, int len) {
    while (len > 1) {
        --len;
        const Ent e = h[len];
        h[len] = h[0];
        heap_place(h, 0, len, e);
    }
}

// Top-down replacement of the root, for heaps holding no NaN: the hole takes
// the same child path as heap_place but stops at the first child holding a
// value strictly greater than e. With every value ordered, the heap property
// makes the values along that path non-decreasing, so heap_place's sift-up
// would stop at the same spot; the resulting heap is identical. The oracle's
// mode 2 restates this and is checked against std::partial_sort. Both
// versions return the new root value.
//
// One level per step: for warps that replay rows side by side (many warps
// hide each other's latency; fewer instructions and registers win there).
__device__ __forceinline__ float heap_place_top1(Ent* h, int len, Ent e) {
    int hole = 0;
    float root = e.v;
    for (;;) {
        int c = 2 * hole + 1;
        if (c >= len) break;
        Ent ch = h[c];
        if (c + 1 < len) {
            const Ent r = h[c + 1];
            if (!before(r.v, ch.v)) {
                ch = r;
                ++c;
            }
        }
        if (before(ch.v, e.v)) break;
        h[hole] = ch;
        if (hole == 0) root = ch.v;
        hole = c;
    }
    h[hole] = e;
    return root;
}

// The heap's loads and stores as explicit shared-memory accesses (32-bit
// shared addresses): the heap functions are reached through non-inlined
// replay functions that only see a generic pointer, and a generic access
// costs more latency than a shared one on every level of the chain.
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ int4 pair_ld(uint32_t a) {
    int4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a)
                 : "memory");
    return v;
}
__device__ __forceinline__ Ent ent_ld(uint32_t a) {
    uint32_t v, i;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v), "=r"(i) : "r"(a) : "memory");
    return Ent{__uint_as_float(v), (int32_t)i};
}
__device__ __forceinline__ void ent_st(uint32_t a, float v, int32_t i) {
    asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(a), "r"(__float_as_uint(v)), "r"((uint32_t)i) : "memory");
}

// Two levels per step: for a lone thread replaying a row (latency-bound).
__device__ __forceinline__ float heap_place_top2(Ent* h, int len, Ent e) {
    // Two levels per round: the children and the four grandchildren of the
    // hole are loaded together, so one shared-memory round trip serves both
    // decisions. Loads at or past len are skipped.
    int hole = 0;
    float root = e.v;
    for (;;) {
        const int c = 2 * hole + 1;
        if (c >= len) break;
        const int gc = 2 * c + 1;  // first grandchild
        Ent l = h[c], r = l, g0 = l, g1 = l, g2 = l, g3 = l;
        if (c + 1 < len) r = h[c + 1];
        if (gc < len) g0 = h[gc];
        if (gc + 1 < len) g1 = h[gc + 1];
        if (gc + 2 < len) g2 = h[gc + 2];
        if (gc + 3 < len) g3 = h[gc + 3];
        const bool take_r = (c + 1 < len) && !before(r.v, l.v);
        const Ent ch = take_r ? r : l;
        if (before(ch.v, e.v)) break;
        h[hole] = ch;
        if (hole == 0) root = ch.v;
        hole = c + (take_r ? 1 : 0);
        const int c2 = 2 * hole + 1;
        if (c2 >= len) break;
        const Ent l2 = take_r ? g2 : g0, r2 = take_r ? g3 : g1;
        const bool take_r2 = (c2 + 1 < len) && !before(r2.v, l2.v);
        const Ent ch2 = take_r2 ? r2 : l2;
        if (before(ch2.v, e.v)) break;
        h[hole] = ch2;
        hole = c2 + (take_r2 ? 1 : 0);
    }
    h[hole] = e;
    return root;
}

template <bool LOOKAHEAD>
__device__ __forceinline__ float heap_place_top(Ent* h, int len, Ent e) {
    return LOOKAHEAD ? heap_place_top2(h, len, e) : heap_place_top1(h, len, e);
}

// heap_place_top2 on a heap in shared memory, with explicit shared loads and
// stores (the same steps).
__device__ __forceinline__ float heap_place_top2_s(Ent* h, int len, Ent e) {
    const uint32_t base = smem_addr(h);
    auto ld = [&](int n) { return ent_ld(base + 8u * (uint32_t)n); };
    int hole = 0;
    float root = e.v;
    for (;;) {
        const int c = 2 * hole + 1;
        if (c >= len) break;
        const int gc = 2 * c + 1;
        Ent l = ld(c), r = l, g0 = l, g1 = l, g2 = l, g3 = l;
        if (c + 1 < len) r = ld(c + 1);
        if (gc < len) g0 = ld(gc);
        if (gc + 1 < len) g1 = ld(gc + 1);
        if (gc + 2 < len) g2 = ld(gc + 2);
        if (gc + 3 < len) g3 = ld(gc + 3);
        const bool take_r = (c + 1 < len) && !before(r.v, l.v);
        const Ent ch = take_r ? r : l;
        if (before(ch.v, e.v)) break;
        ent_st(base + 8u * (uint32_t)hole, ch.v, ch.i);
        if (hole == 0) root = ch.v;
        hole = c + (take_r ? 1 : 0);
        const int c2 = 2 * hole + 1;
        if (c2 >= len) break;
        const Ent l2 = take_r ? g2 : g0, r2 = take_r ? g3 : g1;
        const bool take_r2 = (c2 + 1 < len) && !before(r2.v, l2.v);
        const Ent ch2 = take_r2 ? r2 : l2;
        if (before(ch2.v, e.v)) break;
        ent_st(base + 8u * (uint32_t)hole, ch2.v, ch2.i);
        hole = c2 + (take_r2 ? 1 : 0);
    }
    ent_st(base + 8u * (uint32_t)hole, e.v, e.i);
    return root;
}

// Offers list[0, n) in order to a heap without NaN, both in shared memory;
// returns the root value.
__device__ __forceinline__ float heap_offer_list_top_s(Ent* h, int len, const Ent* list, int n, float root) {
    if (n <= 0) return root;
    const uint32_t la = smem_addr(list);
    Ent nx = ent_ld(la);
    for (int i = 0; i < n; ++i) {
        const Ent e = nx;
        if (i + 1 < n) nx = ent_ld(la + 8u * (uint32_t)(i + 1));
        if (before(e.v, root)) root = heap_place_top2_s(h, len, e);
    }
    return root;
}

// heap_sort_top<true> on a heap in shared memory.
__device__ __forceinline__ void heap_sort_top_s(Ent* h, int len) {
    while (len > 1) {
        --len;
        const Ent e = h[len];
        h[len] = h[0];
        heap_place_top2_s(h, len, e);
    }
}

// Offers list[0, n) in order to a heap without NaN; returns the root value.
template <bool LOOKAHEAD>
__device__ __forceinline__ float heap_offer_list_top(Ent* h, int len, const Ent* list, int n, float root) {
    if (n <= 0) return root;
    Ent nx = list[0];  // loaded ahead, as in pair_offer_list
    for (int i = 0; i < n; ++i) {
        const Ent e = nx;
        if (i + 1 < n) nx = list[i + 1];
        if (before(e.v, root)) root = heap_place_top<LOOKAHEAD>(h, len, e);
    }
    return root;
}

// heap_sort for heaps without NaN (same result, top-down replacements).
template <bool LOOKAHEAD>
__device__ __forceinline__ void heap_sort_top(Ent* h, int len) {
    while (len > 1) {
        --len;
        const Ent e = h[len];
        h[len] = h[0];
        heap_place_top<LOOKAHEAD>(h, len, e);
    }
}

// The same top-down heap for one thread, 1-based (node j of the 0-based heap
// is node j + 1 here), so the two children of node i, 2i and 2i + 1, sit in one
// aligned 16-byte pair: each level costs one dependent shared-memory load for
// both children and one store. `h` needs len + 2 entries and 16-byte
// alignment. Heaps without NaN only; the results equal heap_build /
// heap_place_top1 / heap_sort_top on the 0-based layout.
struct PairHeap {
    Ent* h;  // h[1 .. len], in shared memory
};

// Place e at hole `hole` of the subtree below it, top-down; returns the value
// left at `hole`. The heap is in shared memory.
__device__ __forceinline__ float pair_place(PairHeap hp, int hole, int len, Ent e) {
    const int top = hole;
    float top_v = e.v;
    const uint32_t base = smem_addr(hp.h);
    for (;;) {
        const int c = 2 * hole;
        if (c > len) break;
        const int4 pr = pair_ld(base + 8u * (uint32_t)c);
        const float lv = __int_as_float(pr.x), rv = __int_as_float(pr.z);
        const bool right = (c + 1 <= len) && !before(rv, lv);
        const float chv = right ? rv : lv;
        if (before(chv, e.v)) break;
        ent_st(base + 8u * (uint32_t)hole, chv, right ? pr.w : pr.y);
        if (hole == top) top_v = chv;
        hole = c + (right ? 1 : 0);
    }
    ent_st(base + 8u * (uint32_t)hole, e.v, e.i);
    return top_v;
}

// Floyd's build over nodes 1..len (parents len/2 down to 1).
__device__ __forceinline__ void pair_build(PairHeap hp, int len) {
    for (int p = len / 2; p >= 1; --p) pair_place(hp, p, len, hp.h[p]);
}

// Offers list[0, n) in order; returns the root value. The next entry is
// loaded before the current one is placed, so an offer that does not enter
// costs a compare, not a load round trip (list and heap never overlap).
__device__ __forceinline__ float pair_offer_list(PairHeap hp, int len, const Ent* list, int n, float root) {
    if (n <= 0) return root;
    const uint32_t la = smem_addr(list);  // list in shared memory
    Ent nx = ent_ld(la);
    for (int j = 0; j < n; ++j) {
        const Ent e = nx;
        if (j + 1 < n) nx = ent_ld(la + 8u * (uint32_t)(j + 1));
        if (before(e.v, root)) root = pair_place(hp, 1, len, e);
    }
    return root;
}

// sort_heap: afterwards nodes 1..len hold the reference's top-k order.
__device__ __forceinline__ void pair_sort(PairHeap hp, int len) {
    while (len > 1) {
        const Ent e = hp.h[len];
        hp.h[len] = hp.h[1];
        --len;
        pair_place(hp, 1, len, e);
    }
}

// The same 1-based top-down heap over double values, for rows whose logits
// were edited in double (penalties). 16-byte entries: a node's two children
// are two adjacent 16-byte loads. No NaN.
struct DEnt {
    double v;
    int32_t i;
    int32_t pad;
};

__device__ __forceinline__ double dpair_place(DEnt* h, int hole, int len, DEnt e) {
    const int top = hole;
    double top_v = e.v;
    for (;;) {
        const int c = 2 * hole;
        if (c > len) break;
        const DEnt l = h[c];
        const DEnt r = h[c + 1];  // read past len only within the array (len + 2 entries)
        const bool right = (c + 1 <= len) && !(r.v > l.v);
        const DEnt ch = right ? r : l;
        if (ch.v > e.v) break;
        h[hole] = ch;
        if (hole == top) top_v = ch.v;
        hole = c + (right ? 1 : 0);
    }
    h[hole] = e;
    return top_v;
}

__device__ __forceinline__ void dpair_build(DEnt* h, int len) {
    for (int p = len / 2; p >= 1; --p) dpair_place(h, p, len, h[p]);
}

__device__ __forceinline__ void dpair_sort(DEnt* h, int len) {
    while (len > 1) {
        const DEnt e = h[len];
        h[len] = h[1];
        --len;
        dpair_place(h, 1, len, e);
    }
}

}  // namespace mxs
