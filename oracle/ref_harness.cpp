// TEST INFRASTRUCTURE ONLY: runs the reference's own sampling block on the CPU.
//
// oracle/_ref/sampler_block.inc is the verbatim block of the reference's
// minxfmr_generate, src/api/minxfmr.cpp:2091-2171, sliced out of the reference
// tree at build time by extract_ref_block.py (never committed). This harness
// #includes it inside a loop body that declares the locals the block reads:
// logits (std::vector<double>, widened from fp32 as src/api/minxfmr.cpp:1962
// does), vocab_size, top_k (already clamped as :1567 does), temperature,
// top_p, min_p, sampler_greedy (:1550), next (:1858), ctx->order_buf (:73) and
// rng. The reference's rng is a function-static std::mt19937 seeded from
// std::random_device (:1568); here each row gets std::mt19937(seed + row), so
// the block's draw equals the oracle's injected u from mxs_oracle_uniforms.
//
// Rows run in parallel over OpenMP threads, each with its own context, which is
// how bench.py's reference arm uses every host core.
//
// mxs_ref_sample_edits also #includes the reference's pre-sampler edits
// (oracle/_ref/edits_block.inc, src/api/minxfmr.cpp:2047-2089) before the
// block: it declares ctx->special_tokens, token_history, repeat_last_n and
// the three penalties, and supplies the three tokenizer calls the edit block
// makes for a vocabulary whose token strings are "<id>".

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <random>
#include <string>
#include <unordered_map>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {
struct RefContext {
    std::vector<double> logits_buf;
    std::vector<int> order_buf;
    std::vector<std::string> special_tokens;
};

// The tokenizer calls the edit block makes, for a vocabulary whose token
// strings are "<id>": the harness passes the special tokens as such strings.
// No token is EOS here (the caller's special-token list leaves EOS out).
int tokenizer_token_to_id(const std::string& s) {
    if (s.size() < 3 || s.front() != '<' || s.back() != '>') return -1;
    return std::atoi(s.substr(1, s.size() - 2).c_str());
}
std::string tokenizer_id_to_token(int id) { return "<" + std::to_string(id) + ">"; }
bool is_eos_token(const std::string&) { return false; }
}  // namespace

extern "C" {

// Returns k_use (the clamped k), or -1 on bad arguments. topk_idx gets
// order[0..k_use); topk_prob gets the block's `probs` vector as it stands after
// the block (empty in greedy mode: then it is left untouched); probs_len[r]
// (when non-null) its length.
int mxs_ref_sample(const float* logits_f, int64_t rows, int64_t vocab, int64_t ld,
                   double temperature_in, int top_k_in, double top_p_in, double min_p_in,
                   uint32_t seed, int32_t* next_out, int32_t* topk_idx, double* topk_prob,
                   int32_t* probs_len, int threads) {
    if (!logits_f || !next_out || rows < 0 || vocab <= 0 || ld < vocab) return -1;
    int64_t k_out = top_k_in <= 0 ? 1 : top_k_in;
    if (k_out > vocab) k_out = vocab;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads)
#endif
    {
        RefContext c;
        RefContext* ctx = &c;
        c.logits_buf.assign((size_t)vocab, 0.0);
        c.order_buf.resize((size_t)vocab);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t r = 0; r < rows; ++r) {
            std::vector<double>& logits = ctx->logits_buf;
            const float* src = logits_f + r * ld;
            for (int64_t i = 0; i < vocab; ++i) logits[(size_t)i] = (double)src[i];
            const size_t vocab_size = (size_t)vocab;
            std::mt19937 rng((uint32_t)(seed + (uint32_t)r));
            double temperature = temperature_in;
            double top_p = top_p_in;
            double min_p = min_p_in;
            int top_k = top_k_in;
            if (top_k <= 0) top_k = 1;
            const bool sampler_greedy = (temperature <= 0.0);
            int next = 0;
#include "_ref/sampler_block.inc"
            next_out[r] = next;
            if (topk_idx) std::memcpy(topk_idx + r * k_out, order.data(), sizeof(int32_t) * (size_t)k_use);
            if (topk_prob && !probs.empty())
                std::memcpy(topk_prob + r * k_out, probs.data(), sizeof(double) * probs.size());
            if (probs_len) probs_len[r] = (int32_t)probs.size();
        }
    }
    (void)threads;
    return (int)k_out;
}

// mxs_ref_sample after the reference's own pre-sampler edits
// (src/api/minxfmr.cpp:2047-2089, oracle/_ref/edits_block.inc): special token
// ids (every row), and per row the accepted tokens hist[r * hist_stride, +
// hist_len[r]) as token_history.
int mxs_ref_sample_edits(const float* logits_f, int64_t rows, int64_t vocab, int64_t ld, double temperature_in,
                         int top_k_in, double top_p_in, double min_p_in, uint32_t seed, const int32_t* special,
                         int n_special, const int32_t* hist, int64_t hist_stride, const int32_t* hist_len,
                         int repeat_last_n_in, double repeat_penalty_in, double frequency_penalty_in,
                         double presence_penalty_in, int32_t* next_out, int32_t* topk_idx, double* topk_prob,
                         int32_t* probs_len, int threads) {
    if (!logits_f || !next_out || rows < 0 || vocab <= 0 || ld < vocab) return -1;
    int64_t k_out = top_k_in <= 0 ? 1 : top_k_in;
    if (k_out > vocab) k_out = vocab;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads)
#endif
    {
        RefContext c;
        RefContext* ctx = &c;
        c.logits_buf.assign((size_t)vocab, 0.0);
        c.order_buf.resize((size_t)vocab);
        for (int i = 0; i < n_special; ++i) c.special_tokens.push_back(tokenizer_id_to_token(special[i]));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t r = 0; r < rows; ++r) {
            std::vector<double>& logits = ctx->logits_buf;
            const float* src = logits_f + r * ld;
            for (int64_t i = 0; i < vocab; ++i) logits[(size_t)i] = (double)src[i];
            const size_t vocab_size = (size_t)vocab;
            std::vector<int> token_history;
            if (hist && hist_len)
                token_history.assign(hist + r * hist_stride, hist + r * hist_stride + hist_len[r]);
            const int repeat_last_n = repeat_last_n_in;
            const double repeat_penalty = repeat_penalty_in;
            const double frequency_penalty = frequency_penalty_in;
            const double presence_penalty = presence_penalty_in;
            std::mt19937 rng((uint32_t)(seed + (uint32_t)r));
            double temperature = temperature_in;
            double top_p = top_p_in;
            double min_p = min_p_in;
            int top_k = top_k_in;
            if (top_k <= 0) top_k = 1;
            const bool sampler_greedy = (temperature <= 0.0);
            int next = 0;
#include "_ref/edits_block.inc"
#include "_ref/sampler_block.inc"
            next_out[r] = next;
            if (topk_idx) std::memcpy(topk_idx + r * k_out, order.data(), sizeof(int32_t) * (size_t)k_use);
            if (topk_prob && !probs.empty())
                std::memcpy(topk_prob + r * k_out, probs.data(), sizeof(double) * probs.size());
            if (probs_len) probs_len[r] = (int32_t)probs.size();
        }
    }
    (void)threads;
    return (int)k_out;
}

}  // extern "C"
