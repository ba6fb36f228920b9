// Row finishing for the fused sampler: the draw (softmax over the k survivors,
// then the inverse-CDF pick) and the exact heap replay for rows with ties.
#pragma once

#include "mxs_sampler_kernel.cuh"

namespace mxs {

// First i in cp[0, n) with !(cp[i] < u): std::lower_bound's bisection, step for
// step, so NaNs in cp land where the reference's lower_bound lands.
__device__ __forceinline__ int lower_bound_cp(const double* cp, int n, double u) {
    int first = 0, len = n;
    while (len > 0) {
        const int half = len >> 1;
        if (cp[first + half] < u) {
            first += half + 1;
            len -= half + 1;
        } else {
            len = half;
        }
    }
    return first;
}

// ((p[0] + p[1]) + p[2]) + ... in this order (the reference's running sum),
// with the loads of each block of 8 issued together.
__device__ __forceinline__ double seq_sum(const double* p, int n) {
    double s = 0.0;
    int i = 0;
    for (; i + 8 <= n; i += 8) {
        double v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = p[i + j];
#pragma unroll
        for (int j = 0; j < 8; ++j) s += v[j];
    }
    for (; i < n; ++i) s += p[i];
    return s;
}

// Top-p then min-p on the normalised probabilities pbuf[0, k), renormalising
// in place as src/api/minxfmr.cpp:2128-2165 does; returns how many stay. Serial.
__device__ __forceinline__ int truncate_p(double* pbuf, int k, double top_p, double min_p) {
    int n = k;
    if (top_p < 1.0) {  // src/api/minxfmr.cpp:2128-2145
        double cum = 0.0;
        n = 0;
        for (int i = 0; i < k; ++i) {
            cum += pbuf[i];
            n = i + 1;
            if (cum >= top_p) break;
        }
        if (n < 1) n = 1;
        double renorm = 0.0;
        for (int i = 0; i < n; ++i) renorm += pbuf[i];
        if (renorm > 0.0)
            for (int i = 0; i < n; ++i) pbuf[i] /= renorm;
    }
    if (min_p > 0.0 && n > 1) {  // src/api/minxfmr.cpp:2147-2165
        const double thr = pbuf[0] * min_p;
        int keep = 1;
        for (int i = 1; i < n; ++i) {
            if (pbuf[i] >= thr) keep = i + 1;
            else break;
        }
        n = keep;
        double renorm = 0.0;
        for (int i = 0; i < n; ++i) renorm += pbuf[i];
        if (renorm > 0.0)
            for (int i = 0; i < n; ++i) pbuf[i] /= renorm;
    }
    return n;
}

// Running partial sums of pbuf[0, n) in place, last forced to 1.0, then the
// first index whose cumulative value is not below u (discrete_distribution's
// _M_initialize + operator(), bits/random.tcc:2657-2714). Serial.
__device__ __forceinline__ int cdf_pick(double* pbuf, int n, double u) {
    double run = 0.0;
    int i = 0;
    for (; i + 8 <= n; i += 8) {  // loads of a block of 8 issue together; the adds stay in order
        double v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = pbuf[i + j];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            run += v[j];
            pbuf[i + j] = run;
        }
    }
    for (; i < n; ++i) {
        run += pbuf[i];
        pbuf[i] = run;
    }
    pbuf[n - 1] = 1.0;
    return lower_bound_cp(pbuf, n, u);
}

// e[0, k): the row's top-k in the reference's order. pbuf: k doubles.
// Follows src/api/minxfmr.cpp:2104-2169 and libstdc++'s discrete_distribution
// (bits/random.tcc:2657-2714): each double operation of the reference happens
// here in the same order on the same operands. The k exps and the divisions are
// independent and run across the CTA; the three running sums stay sequential.
__device__ __forceinline__ void block_draw(const Params& p, int64_t row, const Ent* e, int k, double* pbuf, Misc& sm) {
    const int tid = threadIdx.x;
    if (p.topk_idx)
        for (int i = tid; i < k; i += NT) p.topk_idx[row * k + i] = e[i].i;
    const double T = p.temperature;
    bool greedy = (T <= 0.0);
    double sum = 0.0;
    if (!greedy) {
        const double maxs = (double)e[0].v;
        for (int i = tid; i < k; i += NT) pbuf[i] = exp(((double)e[i].v - maxs) / T);
        csync();
        if (tid == 0) sm.sum = seq_sum(pbuf, k);
        csync();
        sum = sm.sum;
        greedy = (sum <= 0.0);
    }
    if (greedy) {
        if (p.topk_prob)
            for (int i = tid; i < k; i += NT) p.topk_prob[row * k + i] = (i == 0) ? 1.0 : 0.0;
        if (tid == 0) p.next[row] = e[0].i;
        csync();
        return;
    }
    for (int i = tid; i < k; i += NT) {
        const double q = pbuf[i] / sum;
        pbuf[i] = q;
        if (p.topk_prob) p.topk_prob[row * k + i] = q;
    }
    csync();
    if (tid == 0) {
        const int n = truncate_p(pbuf, k, p.top_p, p.min_p);
        sm.krem = n;
        sm.sum = (n >= 2) ? seq_sum(pbuf, n) : 0.0;
    }
    csync();
    const int n = sm.krem;
    if (n < 2) {  // discrete_distribution with fewer than two weights returns 0
        if (tid == 0) p.next[row] = e[0].i;
        csync();
        return;
    }
    const double s2 = sm.sum;
    for (int i = tid; i < n; i += NT) pbuf[i] = pbuf[i] / s2;
    csync();
    if (tid == 0) p.next[row] = e[cdf_pick(pbuf, n, p.u[row])].i;
    csync();
}

// Exact replay of the reference's partial_sort heap process over row `row`,
// then the draw. `nan_state`: 1 = the row holds a NaN, 0 = it holds none,
// -1 = unknown (scanned here). With a NaN anywhere the heap order is no longer
// a total order, the root can shrink, and the lower-bound filter is not valid:
// every element is then offered serially.
template <bool SMALL>
__device__ __forceinline__ void exact_row_t(const Params& p, int64_t row, int nan_state, unsigned char* region,
                                            Misc& sm, Ent* sheap) {
    const int tid = threadIdx.x;
    const int k = p.k_use;
    const int64_t V = p.vocab;
    const float* x = p.logits + row * p.ld;
    // SMALL: the heap lives in shared memory (k <= HEAP_SMEM_MAX); each case is
    // its own instantiation so every heap access has a known address space.
    Ent* h = SMALL ? sheap : p.heap_ws + (int64_t)blockIdx.x * k;
    Ent* xl = reinterpret_cast<Ent*>(region + HEAP_SMEM_MAX * sizeof(Ent));
    double* pbuf = SMALL ? reinterpret_cast<double*>(region + HEAP_SMEM_MAX * sizeof(Ent))
                         : p.prob_ws + (int64_t)blockIdx.x * k;

    if (nan_state < 0) {
        int has = 0;
        for (int64_t j = tid; j < V; j += NT) has |= (x[j] != x[j]);
        nan_state = csync_or(has) ? 1 : 0;
    }
    MXS_PROF_T0(tb);
    for (int i = tid; i < k; i += NT) h[i] = Ent{x[i], i};
    csync();
    if (tid == 0) heap_build(h, k);
    csync();
    MXS_PROF_ADD(3, tb);
    if (k < V) {
        if (nan_state) {
            if (tid == 0)
                for (int64_t j = k; j < V; ++j) heap_offer(h, k, Ent{x[j], (int32_t)j});
            csync();
        } else {
            // Geometric steps: step s covers as many logits as came before it
            // (256, 512, ..., at most 65,536). Only logits above the root at
            // the step's start can enter, so a step yields about k offers
            // whatever its size, and the whole row takes ~10 steps. Each warp
            // filters a contiguous segment of the step in one pass (8 loads of
            // 32 consecutive logits in flight) into its own slot of the replay
            // list; thread 0 then offers slot 0, slot 1, ... in the logits'
            // order. A slot that overflows retakes the step at a quarter size.
            constexpr int SLOT = XTILE / NWARPS;
            const int lane = tid & 31, w = tid >> 5;
            const uint32_t lt = (1u << lane) - 1u;
            Ent* slot = xl + w * SLOT;
            int64_t base = k;
            int64_t size = NT;
            while (base < V) {
                const int64_t len = min(size, V - base);
                const int64_t seg = (len + NWARPS - 1) / NWARPS;
                const int64_t lo = base + min((int64_t)w * seg, len);
                const int64_t hi = base + min((int64_t)(w + 1) * seg, len);
                const float r0 = h[0].v;
                MXS_PROF_T0(tfl);
                int c = 0;
                for (int64_t g = lo; g < hi; g += 256) {
                    float xv[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const int64_t jj = g + 32 * q + lane;
                        xv[q] = (jj < hi) ? x[jj] : r0;
                    }
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const bool pass = xv[q] > r0;
                        const uint32_t bal = __ballot_sync(0xffffffffu, pass);
                        const int at = c + __popc(bal & lt);
                        if (pass && at < SLOT) slot[at] = Ent{xv[q], (int32_t)(g + 32 * q + lane)};
                        c += __popc(bal);
                    }
                }
                if (lane == 0) sm.warp_tot[w] = c;
                const int over = csync_or(c > SLOT);
                if (over) {  // retry smaller (NT logits always fit: 32 per warp)
                    size = max((int64_t)NT, len / 4);
                    continue;
                }
                MXS_PROF_ADD(0, tfl);
                MXS_PROF_T0(tof);
                if (tid == 0) {  // no NaN here: top-down replacements
                    float root = h[0].v;
                    for (int w2 = 0; w2 < NWARPS; ++w2)
                        root = SMALL ? heap_offer_list_top_s(h, k, xl + w2 * SLOT, sm.warp_tot[w2], root)
                                     : heap_offer_list_top<true>(h, k, xl + w2 * SLOT, sm.warp_tot[w2], root);
                }
                csync();
                MXS_PROF_ADD(1, tof);
                if (tid == 0) {
                    int n_off = 0;
                    for (int w2 = 0; w2 < NWARPS; ++w2) n_off += sm.warp_tot[w2];
                    MXS_PROF_COUNT(4, n_off);
                    MXS_PROF_COUNT(5, 1);
                }
                base += len;
                size = min(2 * size, (int64_t)65536);
            }
        }
    }
    MXS_PROF_T0(tsd);
    if (tid == 0) {
        if (nan_state)
            heap_sort(h, k);
        else if (SMALL)
            heap_sort_top_s(h, k);
        else
            heap_sort_top<true>(h, k);
    }
    csync();
    block_draw(p, row, h, k, pbuf, sm);
    MXS_PROF_ADD(2, tsd);
}

// Exact replay of the reference's partial_sort heap process over row `row`,
// then the draw (see exact_row_t).
// The heap of a small k lives at the start of `region` (finish_rows_kernel
// passes a static __shared__ array to exact_row_t directly instead).
__device__ __forceinline__ void exact_row(const Params& p, int64_t row, int nan_state, unsigned char* region,
                                          Misc& sm) {
    if (p.k_use <= HEAP_SMEM_MAX)
        exact_row_t<true>(p, row, nan_state, region, sm, reinterpret_cast<Ent*>(region));
    else
        exact_row_t<false>(p, row, nan_state, region, sm, nullptr);
}

}  // namespace mxs
