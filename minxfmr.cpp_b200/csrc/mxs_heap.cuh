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

struct Ent {
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

}  // namespace mxs
