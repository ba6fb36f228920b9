/*
 * mxs_sampler.h -- C ABI of the B200 (sm_100a) decode-step token sampler.
 *
 * The sampler replaces the sampling block of the reference's
 * minxfmr_generate (src/api/minxfmr.cpp:2091-2171):
 *
 *   k_use = clamp(top_k)                       src/api/minxfmr.cpp:1567, :2091-2093
 *   order = std::partial_sort top-k            src/api/minxfmr.cpp:2095-2102
 *   greedy when temperature <= 0               src/api/minxfmr.cpp:1550, :2113-2115
 *   p_i = exp((l_i - l_max) / T), normalise    src/api/minxfmr.cpp:2117-2126
 *   top-p / min-p truncation                   src/api/minxfmr.cpp:2104-2111, :2128-2165
 *   std::discrete_distribution draw            src/api/minxfmr.cpp:2167-2169
 *
 * for a batch of fp32 logits rows kept in device memory. Its results equal the
 * reference block's on the same logits and the same uniform: the top-k index
 * set and its tie order (the order libstdc++'s heap-based partial_sort leaves),
 * the sampled token id, and the probabilities (same double operations, same
 * order; exp is CUDA's double exp, within 1 ulp of glibc's).
 *
 * The reference draws u from a function-static std::mt19937
 * (src/api/minxfmr.cpp:1568); here the caller passes one u in [0, 1) per row,
 * which is what std::discrete_distribution draws (generate_canonical<double,53>)
 * from the engine. Given the engine's u the pick is the same.
 *
 * Conventions (as the reference's C API, include/minxfmr.h:9-37): functions
 * return 0 on success and a negative code on error; nothing throws. Device
 * pointers are owned by the caller. Calls are asynchronous on `stream`
 * (a cudaStream_t; NULL = legacy default stream) unless stated otherwise.
 * No CPU fallback exists: without a usable sm_100 device every call returns
 * MXS_ERR_NO_DEVICE.
 */
#ifndef MXS_SAMPLER_H
#define MXS_SAMPLER_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MXS_API __attribute__((visibility("default")))
#else
#define MXS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define MXS_OK 0
#define MXS_ERR_INVALID (-1)   /* bad argument (null pointer, rows < 0, vocab <= 0, ld < vocab) */
#define MXS_ERR_CUDA (-3)      /* a CUDA call failed (cf. the reference's -3 for backend failures) */
#define MXS_ERR_TIMEOUT (-4)   /* a bounded device wait gave up (see mxs_get_status) */
#define MXS_ERR_NO_DEVICE (-5) /* no sm_100 device current */
#define MXS_ERR_WORKSPACE (-6) /* caller workspace too small or misaligned */
#define MXS_ERR_COMM (-7)      /* NCCL not loaded in the process, or a collective failed */

/* Per-row flag bits written to d_row_flags (optional). */
#define MXS_ROW_EXACT 1u    /* the row had ties (or NaNs) and was resolved by the exact heap replay */
#define MXS_ROW_NAN 2u      /* the row holds a NaN logit */
#define MXS_ROW_OVERFLOW 4u /* candidate buffers overflowed (massive ties); exact replay used */
#define MXS_ROW_TIMEOUT 8u  /* a bounded wait gave up; next[row] = -1 */

/*
 * Sample one token per row.
 *   d_logits   rows x ld fp32 (row r at d_logits + r*ld), vocab <= ld valid columns
 *   temperature, top_k   as minxfmr_generate: T <= 0 is greedy; top_k <= 0 means 1;
 *              top_k > vocab means vocab
 *   d_u        rows doubles in [0, 1): the uniform of each row's draw
 *   d_next     rows int32: sampled token id
 *   d_topk_idx rows x k_use int32 (nullable): the reference's order[0, k_use)
 *   d_topk_prob rows x k_use double (nullable): p_i / sum (src/api/minxfmr.cpp:2123-2126);
 *              greedy rows (T <= 0, or sum <= 0) get 1, 0, 0, ...
 * Uses a library-owned workspace on the current device, allocated on the
 * first call that needs more than the last (make that first call before any
 * stream capture). Replaces src/api/minxfmr.cpp:2091-2171 (top_p = 1, min_p = 0).
 */
MXS_API int mxs_sample_topk(const float* d_logits, int64_t rows, int64_t vocab, int64_t ld, double temperature,
                    int top_k, const double* d_u, int32_t* d_next, int32_t* d_topk_idx, double* d_topk_prob,
                    void* stream);

/*
 * As mxs_sample_topk, plus top_p / min_p (clamped as src/api/minxfmr.cpp:2104-2111),
 * optional per-row flags, and an optional caller workspace. With
 * d_workspace == NULL the library-owned workspace is used; otherwise
 * workspace_bytes must be >= mxs_workspace_size(...) and the workspace must
 * have been zero-filled once (mxs_workspace_init); every call leaves it zeroed
 * again for the next. Calls sharing one workspace must not overlap on the GPU.
 */
MXS_API int mxs_sample_topk_ex(const float* d_logits, int64_t rows, int64_t vocab, int64_t ld, double temperature,
                       int top_k, double top_p, double min_p, const double* d_u, int32_t* d_next,
                       int32_t* d_topk_idx, double* d_topk_prob, uint32_t* d_row_flags, void* d_workspace,
                       size_t workspace_bytes, void* stream);

/*
 * mxs_sample_topk_ex after the reference's pre-sampler edits on the device
 * (src/api/minxfmr.cpp:2047-2089), applied in double as the reference does:
 *   d_special[0, n_special)  token ids whose logits become -inf in every row
 *                            (the reference's special tokens, EOS left out, as
 *                            :2050-2055 skip it); ids outside the vocabulary
 *                            are skipped
 *   d_history, hist_stride, d_hist_len  row r's accepted tokens are
 *                            d_history[r*hist_stride, + d_hist_len[r])
 *   repeat_last_n, repeat_penalty, frequency_penalty, presence_penalty
 *                            as minxfmr_generate: over the last repeat_last_n
 *                            tokens (< 0: all), each distinct token's logit is
 *                            multiplied (<= 0) or divided (> 0) by
 *                            repeat_penalty and loses count*frequency_penalty +
 *                            presence_penalty
 * A penalised logit is a double fp32 cannot hold: the sampler carries it
 * exactly (ids, tie order and probabilities as the reference's on the edited
 * double logits). d_logits is edited in place: the masked and penalised
 * tokens read -inf after the call. Limits: top_k <= 128, 16-byte aligned rows
 * with ld % 4 == 0, a penalty window of at most 1024 tokens (else
 * MXS_ERR_INVALID). A row holding a NaN logit is not drawn (next = -1,
 * MXS_ROW_NAN). Library-owned workspace; asynchronous on `stream`.
 */
MXS_API int mxs_sample_topk_edits(float* d_logits, int64_t rows, int64_t vocab, int64_t ld, double temperature,
                                  int top_k, double top_p, double min_p, const int32_t* d_special, int n_special,
                                  const int32_t* d_history, int64_t hist_stride, const int32_t* d_hist_len,
                                  int repeat_last_n, double repeat_penalty, double frequency_penalty,
                                  double presence_penalty, const double* d_u, int32_t* d_next, int32_t* d_topk_idx,
                                  double* d_topk_prob, uint32_t* d_row_flags, void* stream);

/*
 * The reference's checks on the sampled token, after a sampling call on the
 * same stream (src/api/minxfmr.cpp:2189-2205 first-token fallback, :2232-2243
 * EOS stop). The tokenizer stays with the caller, which classifies every
 * token id once in d_token_class[vocab]:
 *   MXS_TOKEN_NOT_FIRST  not usable as a row's first generated token (its
 *                        rendered piece is empty or white space, or it is EOS
 *                        or a role token: the reference's condition at :2189)
 *   MXS_TOKEN_EOS        EOS (:2232)
 * For rows with d_first_step[r] != 0 whose d_next is NOT_FIRST, d_next becomes
 * the first token of d_topk_idx[r][1, k_use) that is not (unchanged if none
 * is). d_stop[r] (nullable) gets 1 when the final d_next is EOS. d_topk_idx
 * (rows x k_use, from the sampling call) may be NULL when d_first_step is.
 */
#define MXS_TOKEN_NOT_FIRST 1u
#define MXS_TOKEN_EOS 2u
MXS_API int mxs_token_checks(int64_t rows, int top_k, int64_t vocab, const int32_t* d_topk_idx, int32_t* d_next,
                             const uint8_t* d_token_class, const uint8_t* d_first_step, uint8_t* d_stop,
                             void* stream);

/*
 * The output projection kept on the device, then mxs_sample_topk_ex: logits =
 * hidden . weight^T (the reference's lm_head step, src/api/minxfmr.cpp:1918-2036
 * and src/backend/cuda/cuda_backend.cu:731-780, whose logits it then copies to
 * the host at :1440-1442), as a cuBLAS GEMM with bf16 operands and fp32
 * accumulation and output, sampled where it lands in HBM.
 *   d_hidden   rows x d_model bf16 (row r at d_hidden + r*ld_hidden elements)
 *   d_weight   vocab x d_model bf16 (row v at d_weight + v*ld_weight elements)
 *   d_logits_out  rows x ld_logits fp32 (nullable: a library-owned buffer with
 *              a leading dimension rounded up to a multiple of 4)
 * The sampled ids equal the reference block's on these logits (the GEMM is
 * fp32-accumulated, not the reference's own dot-product order). cuBLAS is
 * looked up at run time (MXS_ERR_CUDA when absent). Calls on one device run
 * one at a time (a per-device lock).
 */
MXS_API int mxs_sample_from_hidden(const void* d_hidden, int64_t ld_hidden, const void* d_weight, int64_t ld_weight,
                                   int64_t rows, int64_t d_model, int64_t vocab, double temperature, int top_k,
                                   double top_p, double min_p, const double* d_u, int32_t* d_next,
                                   int32_t* d_topk_idx, double* d_topk_prob, float* d_logits_out,
                                   int64_t ld_logits, void* stream);

/* Bytes of workspace mxs_sample_topk_ex needs for this shape on the current device. */
MXS_API int mxs_workspace_size(int64_t rows, int64_t vocab, int top_k, size_t* bytes);

/* Zero-fill a caller workspace (once, before its first use). */
MXS_API int mxs_workspace_init(void* d_workspace, size_t workspace_bytes, void* stream);

/*
 * Host-buffer entry point: the drop-in for a caller whose logits are on the
 * host (the reference copies lm_head logits to the host, src/backend/cuda/
 * cuda_backend.cu:1440-1442, and samples there). Copies logits and u to the
 * device, samples, copies next (and the optional top-k outputs) back, and
 * returns when they are in host memory. Pinned host buffers make the copies
 * asynchronous DMA; pageable ones work too. The device-side copies are reused
 * from call to call, so calls on one device run one at a time (a per-device
 * lock), as the reference's single-threaded generate loop does.
 */
MXS_API int mxs_sample_topk_host(const float* h_logits, int64_t rows, int64_t vocab, int64_t ld, double temperature,
                         int top_k, double top_p, double min_p, const double* h_u, int32_t* h_next,
                         int32_t* h_topk_idx, double* h_topk_prob, void* stream);

/*
 * Vocab-sharded sampling, step 1 (one call per shard, e.g. one per GPU): the
 * candidate list of every row of a column shard. For row r the list holds all
 * logits of the shard >= the shard's k_use-th largest value, as
 * (order-preserving key << 32 | global column) words, at
 * d_cand + r*cap, with its length in d_count[r]; d_flags[r] gets MXS_ROW_NAN /
 * MXS_ROW_OVERFLOW when the list cannot stand for the shard (then the row
 * must be sampled from its full logits). On the two-kernel path (top_k <= 128,
 * 16-byte aligned rows) the list holds the logits above the k-th largest first,
 * then those equal to it; when more of those tie than the list holds, it keeps
 * as many as fit and d_flags[r] gets MXS_ROW_EXACT (every logit left out equals
 * the list's smallest value; mxs_merge_sample accounts for it). col_offset is
 * the shard's first global column. cap >= k_use.
 */
MXS_API int mxs_shard_candidates(const float* d_shard_logits, int64_t rows, int64_t shard_cols, int64_t ld,
                         int64_t col_offset, int top_k, int cap, uint64_t* d_cand, uint32_t* d_count,
                         uint32_t* d_flags, void* stream);

/*
 * Vocab-sharded sampling, step 2, after the shards' lists are gathered (e.g. by
 * an NCCL all-gather) as nshards consecutive blocks of [rows x cap] words
 * (d_cand_all) and [rows] counts and flags. Merges each row's lists, selects
 * the top-k, and draws. Not drawn, with d_row_flags MXS_ROW_EXACT (plus the
 * shard's MXS_ROW_NAN / MXS_ROW_OVERFLOW) and d_next -1: rows with a flagged
 * shard list, rows whose truncated list (MXS_ROW_EXACT from
 * mxs_shard_candidates) could hide some of the k largest, and tie rows whose
 * order matters (top-k list requested, or a draw landing on a tied position).
 * The caller samples them with mxs_sample_topk_ex on the full row (the tie
 * order depends on every logit of the row), or as mxs_sample_vocabsharded does.
 */
MXS_API int mxs_merge_sample(const uint64_t* d_cand_all, const uint32_t* d_count_all, const uint32_t* d_flags_all,
                     int nshards, int cap, int64_t rows, int64_t vocab, double temperature, int top_k,
                     double top_p, double min_p, const double* d_u, int32_t* d_next, int32_t* d_topk_idx,
                     double* d_topk_prob, uint32_t* d_row_flags, void* stream);

/*
 * Row-sharded sampling (no collective; rows are independent): rank `rank` of
 * `world` takes rows [rank*P, min(global_rows, (rank+1)*P)), P = ceil(global_rows
 * / world), of a batch split over the ranks. d_local_logits holds those rows
 * (row i at d_local_logits + i*ld); d_u_global holds every row's uniform (the
 * call reads this rank's range); the outputs are this rank's rows. The number of
 * local rows is written to *local_rows (nullable). Otherwise as
 * mxs_sample_topk_ex with the library workspace. The sharded form of
 * src/api/minxfmr.cpp:2091-2171 over a batch.
 */
MXS_API int mxs_sample_rowsharded(const float* d_local_logits, int64_t global_rows, int rank, int world,
                                  int64_t vocab, int64_t ld, double temperature, int top_k, double top_p,
                                  double min_p, const double* d_u_global, int32_t* d_next, int32_t* d_topk_idx,
                                  double* d_topk_prob, uint32_t* d_row_flags, int64_t* local_rows, void* stream);

/*
 * Vocab-sharded sampling in one call per rank (collective over nccl_comm, an
 * ncclComm_t of the NCCL the process has loaded; world = its size). Every rank
 * passes the same rows: its column shard [rank*shard_cols, (rank+1)*shard_cols)
 * of a vocabulary of world*shard_cols, and the same d_u. Runs
 * mxs_shard_candidates, one NCCL all-gather group of the lists, and
 * mxs_merge_sample on the given stream, so every rank ends with the same
 * outputs for every row, equal to mxs_sample_topk_ex on the full rows. Rows
 * whose merged lists show a tie that matters (their tie order depends on
 * logits no list holds) are resolved from lists too, when top_k <= 128 and
 * top_k <= shard_cols: rank 0 replays the reference's heap process over its
 * shard and every later rank lists the logits of its shard that can still
 * enter the heap; one more all-gather group, and every rank finishes the
 * replay. Rows that lists cannot resolve (a NaN, a list over its capacity, a
 * larger top_k) are gathered whole (one more all-gather) and sampled as full
 * rows. Synchronises the stream once to learn how many rows were handed back,
 * and once more when any were. d_row_flags (nullable) gets MXS_ROW_EXACT on
 * the handed-back rows. Above top_k = 2048 (the merge's limit) every row is
 * gathered whole. Calls on one device must not overlap (one lock per device;
 * ranks on different devices never wait for each other's lock). Returns
 * MXS_ERR_COMM when NCCL is not loaded or a collective fails.
 */
MXS_API int mxs_sample_vocabsharded(const float* d_shard_logits, int64_t rows, int64_t shard_cols, int64_t ld,
                                    double temperature, int top_k, double top_p, double min_p, const double* d_u,
                                    int32_t* d_next, int32_t* d_topk_idx, double* d_topk_prob,
                                    uint32_t* d_row_flags, void* nccl_comm, void* stream);

/*
 * Measurement hook (no counterpart in the reference): rows of the last
 * mxs_sample_vocabsharded call on the current device whose ties were resolved
 * from lists, and rows that were gathered whole. Either pointer may be NULL.
 */
MXS_API int mxs_vocabsharded_stats(int64_t* tie_rows_from_lists, int64_t* rows_gathered_whole);

/*
 * Measurement hook (no counterpart in the reference): when set, the next
 * sampling calls on the current device record `start` and `stop` (cudaEvent_t,
 * created by the caller) on the call's stream immediately around the launch of
 * the row-streaming kernel, the call's dominant kernel, so its duration can be
 * timed on the device apart from the short finishing kernels. NULL, NULL
 * turns it off.
 */
MXS_API int mxs_set_profile_events(void* start, void* stop);

/*
 * No counterpart in the reference: an addition of this library for callers that
 * cannot allocate device memory (hosts whose memory pool owns the whole GPU, or
 * that forbid allocation on the per-token path). Same arguments and results as
 * mxs_sample_topk_ex without a workspace: the scratch is a fixed array of
 * MXS_NOALLOC_SCRATCH_BYTES (48 MiB) compiled into the library, held by every
 * GPU that loads it until the process exits; no call allocates or frees memory.
 * Returns MXS_ERR_WORKSPACE when the shape needs more scratch than that
 * (mxs_workspace_size tells how much). On the default path (top_k <= 128,
 * 16-byte aligned rows) the need is about rows x max(1024, 12 top_k + 512) x 8
 * bytes at any vocabulary: about 5,600 rows fit at top_k = 50 (the 4096-row
 * batch of the throughput benchmark does), about 3,000 at top_k = 128; top_k
 * above 2048 needs the most (two k-entry slots per CTA).
 * Timeouts of these calls reach mxs_get_status like any other call's.
 * The first call on a device looks up the array's device address; make that
 * call before any stream capture. All calls share the one array, so calls
 * that overlap on the GPU (other streams, other threads) race and must be
 * serialised by the caller.
 */
#define MXS_NOALLOC_SCRATCH_BYTES (48u << 20)
MXS_API int mxs_sample_topk_noalloc(const float* d_logits, int64_t rows, int64_t vocab, int64_t ld,
                                    double temperature, int top_k, double top_p, double min_p, const double* d_u,
                                    int32_t* d_next, int32_t* d_topk_idx, double* d_topk_prob,
                                    uint32_t* d_row_flags, void* stream);

/*
 * Test hooks of this library's own tests (no counterpart in the reference).
 * Nothing else changes them: a sampling call never reads the environment.
 *   drop_tile        CTA 0's streaming producer stops before its tile with this
 *                    sequence number, so its consumers' bounded wait runs out and
 *                    the rows report MXS_ROW_TIMEOUT (-1: off, the default)
 *   replay_warp_min  a finish CTA replays its tie rows one per warp when it holds
 *                    at least this many, else with the whole CTA (default 1)
 *   path             0: default planning; 2: the CTA-synchronous kernel for every k
 * Process-wide; calls already enqueued keep the hooks they were launched with.
 */
MXS_API int mxs_set_test_hooks(int64_t drop_tile, int replay_warp_min, int path);

/* OR of MXS_ROW_* flags of every row that hit MXS_ROW_TIMEOUT since the last clear
 * on the current device, from every entry point and workspace (a sticky word per
 * device that every launch ORs into; synchronises the device). */
MXS_API int mxs_get_status(uint32_t* flags, int clear);

/* Library version string. */
MXS_API const char* mxs_version(void);

#ifdef __cplusplus
}
#endif
#endif /* MXS_SAMPLER_H */
