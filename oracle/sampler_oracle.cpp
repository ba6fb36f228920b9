// TEST INFRASTRUCTURE ONLY: the CPU oracle for the decode-step token sampler.
//
// Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load
// this library, and only as the checker. The product path (libmxs.so) never
// links or calls it.
//
// What it restates: the sampling block of minxfmr_generate in the reference,
// src/api/minxfmr.cpp:2091-2171, on fp32 logits rows (the reference widens fp32
// logits to double at src/api/minxfmr.cpp:1962/1992/2016, which preserves value
// and order, so comparing the floats is the same as comparing the doubles):
//
//   k_use clamp                         src/api/minxfmr.cpp:2091-2093 (+ :1567)
//   order[i] = i; partial_sort(k_use)   src/api/minxfmr.cpp:2095-2102
//   greedy when T <= 0                  src/api/minxfmr.cpp:1550, :2113-2115
//   p_i = exp((l_i - l_max) / T), sum   src/api/minxfmr.cpp:2117-2122
//   sum <= 0 -> order[0]; p_i /= sum    src/api/minxfmr.cpp:2123-2126
//   top-p, min-p truncation             src/api/minxfmr.cpp:2104-2111, :2128-2165
//   discrete_distribution draw          src/api/minxfmr.cpp:2167-2169
//
// The draw: the reference draws from a function-static std::mt19937 through
// std::discrete_distribution<int> (libstdc++ 13, bits/random.tcc:2657-2714).
// This oracle takes the uniform u per row as an input instead and reproduces the
// distribution's arithmetic: normalise again by a sequential sum, form the
// partial sums, force the last one to 1.0, return the first i with cp[i] >= u
// (a lower_bound bisection). mxs_oracle_uniforms() produces, per row, the exact
// u that std::discrete_distribution would draw from std::mt19937(seed + row),
// and mxs_oracle_check_draw() proves the equivalence against the real class.
//
// Two top-k modes:
//   mode 0: the real std::partial_sort of the container's libstdc++ (GCC 13),
//           called exactly as the reference calls it (the tie order is the
//           heap order of __heap_select + __sort_heap, not index order);
//   mode 1: this file's own restatement of that heap process (Floyd build,
//           hole sift-down to a leaf, then sift-up), which the CUDA kernels
//           also implement; tests cross-check mode 1 against mode 0;
//   mode 2: mode 1 with each replacement of the root (select and sort phases)
//           done top-down: the hole moves along the same child path but stops
//           at the first child holding a value strictly greater than the new
//           entry. While every value is ordered (no NaN) the heap property
//           makes the path's values non-decreasing, so this leaves exactly the
//           heap that the leaf-first descent plus sift-up leaves; the CUDA
//           replays use it for rows without NaN. Rows with NaN take mode 1.
//
// Parity pin: the reference has no sampler tests or golden vectors. The pin is
// oracle/_ref, which compiles the reference's own sampling block (sliced from
// the reference source at build time, never committed) inside a harness, plus
// the golden fixtures under tests/golden/ generated from it.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <random>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// ---------------------------------------------------------------------------
// Restated heap process (mode 1). "before(a, b)" is the reference comparator
// logits[a] > logits[b] (src/api/minxfmr.cpp:2102). A heap ordered by it keeps
// the smallest value at the root.
// ---------------------------------------------------------------------------
template <typename T>
struct HeapRow {
    const T* x;
    int32_t* h;  // heap of indices
    bool before(int32_t a, int32_t b) const { return x[a] > x[b]; }

    void sift_up(int64_t hole, int64_t top, int32_t v) {
        int64_t parent = (hole - 1) / 2;
        while (hole > top && before(h[parent], v)) {
            h[hole] = h[parent];
            hole = parent;
            parent = (hole - 1) / 2;
        }
        h[hole] = v;
    }
    // Move the hole from `hole` down to a leaf along the child that is not
    // "before" its sibling, then let v rise from there.
    void place(int64_t hole, int64_t len, int32_t v) {
        const int64_t top = hole;
        int64_t c = hole;
        while (c < (len - 1) / 2) {
            c = 2 * (c + 1);
            if (before(h[c], h[c - 1])) c--;
            h[hole] = h[c];
            hole = c;
        }
        if ((len & 1) == 0 && c == (len - 2) / 2) {
            c = 2 * (c + 1);
            h[hole] = h[c - 1];
            hole = c - 1;
        }
        sift_up(hole, top, v);
    }
    // Top-down replacement of the root (mode 2): same child choice as place().
    void place_top(int64_t len, int32_t v) {
        int64_t hole = 0;
        for (;;) {
            int64_t c = 2 * hole + 1;
            if (c >= len) break;
            if (c + 1 < len && !before(h[c + 1], h[c])) c++;
            if (before(h[c], v)) break;  // the child holds a strictly greater value
            h[hole] = h[c];
            hole = c;
        }
        h[hole] = v;
    }
    void build(int64_t len) {
        if (len < 2) return;
        for (int64_t p = (len - 2) / 2;; --p) {
            place(p, len, h[p]);
            if (p == 0) break;
        }
    }
};

template <typename T>
void restated_partial_sort(const T* x, int64_t vocab, int64_t k, int32_t* order, bool top_down = false) {
    HeapRow<T> hr{x, order};
    if (top_down)
        for (int64_t i = 0; i < vocab; ++i)
            if (x[i] != x[i]) top_down = false;
    for (int64_t i = 0; i < vocab; ++i) order[i] = (int32_t)i;
    hr.build(k);
    for (int64_t i = k; i < vocab; ++i) {
        if (hr.before((int32_t)i, order[0])) {
            const int32_t v = order[i];
            order[i] = order[0];
            if (top_down)
                hr.place_top(k, v);
            else
                hr.place(0, k, v);
        }
    }
    for (int64_t len = k; len > 1;) {
        --len;
        const int32_t v = order[len];
        order[len] = order[0];
        if (top_down)
            hr.place_top(len, v);
        else
            hr.place(0, len, v);
    }
}

// First i in cp[0, n) with !(cp[i] < u): the bisection of std::lower_bound.
int64_t lower_bound_cp(const double* cp, int64_t n, double u) {
    int64_t first = 0, len = n;
    while (len > 0) {
        const int64_t half = len >> 1;
        if (cp[first + half] < u) {
            first = first + half + 1;
            len = len - half - 1;
        } else {
            len = half;
        }
    }
    return first;
}

// One row of the sampling block (fp32 logits, or the double logits a row has
// after the pre-sampler edits). order must hold vocab ints; probs/cp k_use doubles.
template <typename T>
int32_t sample_row(const T* x, int64_t vocab, double temperature, int top_k, double top_p,
                   double min_p, double u, int mode, int32_t* order, double* probs, double* cp,
                   int32_t* topk_idx, double* topk_prob) {
    int64_t k_use = top_k <= 0 ? 1 : top_k;
    if (k_use > vocab) k_use = vocab;

    if (mode == 0) {
        for (int64_t i = 0; i < vocab; ++i) order[i] = (int32_t)i;
        std::partial_sort(order, order + k_use, order + vocab,
                          [&](int a, int b) { return (double)x[a] > (double)x[b]; });
    } else {
        restated_partial_sort(x, vocab, k_use, order, mode == 2);
    }
    if (topk_idx) std::memcpy(topk_idx, order, sizeof(int32_t) * (size_t)k_use);

    const double maxs = (double)x[order[0]];
    if (top_p <= 0.0 || top_p > 1.0) top_p = 1.0;
    if (min_p < 0.0) min_p = 0.0;
    if (min_p > 1.0) min_p = 1.0;

    auto greedy_probs = [&]() {
        if (topk_prob) {
            topk_prob[0] = 1.0;
            for (int64_t i = 1; i < k_use; ++i) topk_prob[i] = 0.0;
        }
    };
    if (temperature <= 0.0) {
        greedy_probs();
        return order[0];
    }
    double sum = 0.0;
    for (int64_t i = 0; i < k_use; ++i) {
        probs[i] = std::exp(((double)x[order[i]] - maxs) / temperature);
        sum += probs[i];
    }
    if (sum <= 0.0) {
        greedy_probs();
        return order[0];
    }
    for (int64_t i = 0; i < k_use; ++i) probs[i] /= sum;
    if (topk_prob) std::memcpy(topk_prob, probs, sizeof(double) * (size_t)k_use);

    int64_t n = k_use;
    if (top_p < 1.0) {
        double cum = 0.0;
        n = 0;
        for (int64_t i = 0; i < k_use; ++i) {
            cum += probs[i];
            n = i + 1;
            if (cum >= top_p) break;
        }
        if (n < 1) n = 1;
        double renorm = 0.0;
        for (int64_t i = 0; i < n; ++i) renorm += probs[i];
        if (renorm > 0.0)
            for (int64_t i = 0; i < n; ++i) probs[i] /= renorm;
    }
    if (min_p > 0.0 && n > 1) {
        const double thr = probs[0] * min_p;
        int64_t keep = 1;
        for (int64_t i = 1; i < n; ++i) {
            if (probs[i] >= thr) keep = i + 1;
            else break;
        }
        n = keep;
        double renorm = 0.0;
        for (int64_t i = 0; i < n; ++i) renorm += probs[i];
        if (renorm > 0.0)
            for (int64_t i = 0; i < n; ++i) probs[i] /= renorm;
    }
    // std::discrete_distribution over probs[0, n): fewer than two weights -> 0.
    if (n < 2) return order[0];
    double s2 = 0.0;
    for (int64_t i = 0; i < n; ++i) s2 += probs[i];
    double run = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        run += probs[i] / s2;
        cp[i] = run;
    }
    cp[n - 1] = 1.0;
    return order[lower_bound_cp(cp, n, u)];
}

}  // namespace

extern "C" {

// Samples `rows` rows of fp32 logits (row r at logits + r*ld). Outputs:
// next[rows]; topk_idx[rows * k_use] and topk_prob[rows * k_use] when non-null.
// Returns k_use, or -1 on bad arguments.
int mxs_oracle_sample(const float* logits, int64_t rows, int64_t vocab, int64_t ld,
                      double temperature, int top_k, double top_p, double min_p,
                      const double* u, int32_t* next, int32_t* topk_idx, double* topk_prob,
                      int mode, int threads) {
    if (!logits || !u || !next || rows < 0 || vocab <= 0 || ld < vocab) return -1;
    int64_t k_use = top_k <= 0 ? 1 : top_k;
    if (k_use > vocab) k_use = vocab;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads)
#endif
    {
        std::vector<int32_t> order((size_t)vocab);
        std::vector<double> probs((size_t)k_use), cp((size_t)k_use);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t r = 0; r < rows; ++r) {
            next[r] = sample_row(logits + r * ld, vocab, temperature, top_k, top_p, min_p, u[r],
                                 mode, order.data(), probs.data(), cp.data(),
                                 topk_idx ? topk_idx + r * k_use : nullptr,
                                 topk_prob ? topk_prob + r * k_use : nullptr);
        }
    }
    (void)threads;
    return (int)k_use;
}

// The reference's pre-sampler edits (src/api/minxfmr.cpp:2047-2089), on one
// row widened to double: the special tokens' logits become -inf (the caller
// passes their ids, EOS already left out, as :2050-2055 skip it), then, over
// the last penalty_n accepted tokens (repeat_last_n < 0: all of them; at most
// the history length), each distinct token's logit gets the repetition
// penalty (multiplied when <= 0, divided otherwise) and loses
// count * frequency_penalty + presence_penalty, in double. Tokens outside the
// vocabulary are skipped.
void apply_edits(double* row, int64_t vocab, const int32_t* special, int n_special, const int32_t* hist,
                 int hist_len, int repeat_last_n, double repeat_penalty, double frequency_penalty,
                 double presence_penalty) {
    for (int i = 0; i < n_special; ++i) {
        const int32_t sid = special[i];
        if (sid < 0 || sid >= vocab) continue;
        row[sid] = -std::numeric_limits<double>::infinity();
    }
    int penalty_n = repeat_last_n;
    if (penalty_n < 0) penalty_n = hist_len;
    if (penalty_n > hist_len) penalty_n = hist_len;
    if (penalty_n <= 0 || (repeat_penalty == 1.0 && frequency_penalty == 0.0 && presence_penalty == 0.0)) return;
    std::vector<int32_t> toks(hist + (hist_len - penalty_n), hist + hist_len);
    std::sort(toks.begin(), toks.end());
    for (size_t i = 0; i < toks.size();) {
        size_t j = i;
        while (j < toks.size() && toks[j] == toks[i]) ++j;
        const int32_t tid = toks[i];
        const int count = (int)(j - i);
        i = j;
        if (tid < 0 || tid >= vocab) continue;
        double logit = row[tid];
        if (repeat_penalty != 1.0) {
            if (logit <= 0.0)
                logit *= repeat_penalty;
            else
                logit /= repeat_penalty;
        }
        logit -= (double)count * frequency_penalty + (count > 0 ? presence_penalty : 0.0);
        row[tid] = logit;
    }
}

// mxs_oracle_sample after the pre-sampler edits: special token ids (shared by
// every row), and per row its accepted tokens hist[r * hist_stride, + hist_len[r]).
int mxs_oracle_sample_edits(const float* logits, int64_t rows, int64_t vocab, int64_t ld, double temperature,
                            int top_k, double top_p, double min_p, const double* u, const int32_t* special,
                            int n_special, const int32_t* hist, int64_t hist_stride, const int32_t* hist_len,
                            int repeat_last_n, double repeat_penalty, double frequency_penalty,
                            double presence_penalty, int32_t* next, int32_t* topk_idx, double* topk_prob, int mode,
                            int threads) {
    if (!logits || !u || !next || rows < 0 || vocab <= 0 || ld < vocab) return -1;
    int64_t k_use = top_k <= 0 ? 1 : top_k;
    if (k_use > vocab) k_use = vocab;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads)
#endif
    {
        std::vector<int32_t> order((size_t)vocab);
        std::vector<double> row((size_t)vocab), probs((size_t)k_use), cp((size_t)k_use);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t r = 0; r < rows; ++r) {
            const float* src = logits + r * ld;
            for (int64_t i = 0; i < vocab; ++i) row[(size_t)i] = (double)src[i];
            apply_edits(row.data(), vocab, special, n_special, hist ? hist + r * hist_stride : nullptr,
                        hist_len ? hist_len[r] : 0, repeat_last_n, repeat_penalty, frequency_penalty,
                        presence_penalty);
            next[r] = sample_row(row.data(), vocab, temperature, top_k, top_p, min_p, u[r], mode, order.data(),
                                 probs.data(), cp.data(), topk_idx ? topk_idx + r * k_use : nullptr,
                                 topk_prob ? topk_prob + r * k_use : nullptr);
        }
    }
    (void)threads;
    return (int)k_use;
}

// The reference's checks on the sampled token (src/api/minxfmr.cpp:2189-2205,
// :2232-2243) with the tokenizer's answers given per id in cls (bit 0: not
// usable as a first token -- invisible piece, EOS or role token; bit 1: EOS):
// on a row's first generated token a bit-0 token is replaced by the first
// order[1, k) token without bit 0; stop[r] = the final token is EOS.
void mxs_oracle_token_checks(int64_t rows, int64_t k, int64_t vocab, const int32_t* order, int32_t* next,
                             const uint8_t* cls, const uint8_t* first_step, uint8_t* stop) {
    auto bad_first = [&](int32_t t) { return t < 0 || t >= vocab || (cls[t] & 1u); };
    for (int64_t r = 0; r < rows; ++r) {
        if (first_step && first_step[r] && bad_first(next[r])) {
            for (int64_t i = 1; i < k; ++i) {
                const int32_t alt = order[r * k + i];
                if (!bad_first(alt)) {
                    next[r] = alt;
                    break;
                }
            }
        }
        if (stop) stop[r] = (next[r] >= 0 && next[r] < vocab && (cls[next[r]] & 2u)) ? 1 : 0;
    }
}

// u[r] = the double std::discrete_distribution<int> draws from
// std::mt19937(seed + r): generate_canonical<double, 53> over two 32-bit outputs.
void mxs_oracle_uniforms(uint32_t seed, int64_t n, double* out) {
    for (int64_t r = 0; r < n; ++r) {
        std::mt19937 eng((uint32_t)(seed + (uint32_t)r));
        out[r] = std::generate_canonical<double, std::numeric_limits<double>::digits>(eng);
    }
}

// Draws from the real std::discrete_distribution<int>(w, w + n) with
// std::mt19937(seed), and from this oracle's injected-u path with the u
// mxs_oracle_uniforms gives for the same seed. Writes both picks.
void mxs_oracle_check_draw(uint32_t seed, const double* w, int64_t n, int32_t* pick_std,
                           int32_t* pick_injected) {
    std::mt19937 eng(seed);
    std::discrete_distribution<int> dist(w, w + n);
    *pick_std = dist(eng);
    double u;
    mxs_oracle_uniforms(seed, 1, &u);
    if (n < 2) {
        *pick_injected = 0;
        return;
    }
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) s += w[i];
    std::vector<double> cp((size_t)n);
    double run = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        run += w[i] / s;
        cp[(size_t)i] = run;
    }
    cp[(size_t)n - 1] = 1.0;
    *pick_injected = (int32_t)lower_bound_cp(cp.data(), n, u);
}

// Top-k order only (no draw), for differential tests of the heap restatement.
void mxs_oracle_topk_order(const float* x, int64_t vocab, int top_k, int mode, int32_t* out) {
    int64_t k_use = top_k <= 0 ? 1 : top_k;
    if (k_use > vocab) k_use = vocab;
    std::vector<int32_t> order((size_t)vocab);
    if (mode == 0) {
        for (int64_t i = 0; i < vocab; ++i) order[(size_t)i] = (int32_t)i;
        std::partial_sort(order.begin(), order.begin() + k_use, order.end(),
                          [&](int a, int b) { return (double)x[a] > (double)x[b]; });
    } else {
        restated_partial_sort(x, vocab, k_use, order.data(), mode == 2);
    }
    std::memcpy(out, order.data(), sizeof(int32_t) * (size_t)k_use);
}

}  // extern "C"
