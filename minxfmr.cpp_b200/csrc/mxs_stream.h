// Launch interface of the two-kernel path (mxs_stream.cu).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace mxs {
struct Params;
constexpr int KSPLIT = 128;          // largest k the two-kernel path takes
constexpr int SPLIT_ROW_CAP = 1024;  // candidate list entries per row
constexpr int S_TILE = 8192;         // logits per ring stage of the streaming kernel (32 KB)
constexpr int S_STAGES = 3;          // ring depth (96 KB in flight per CTA)
size_t stream_smem_bytes();
cudaError_t stream_path_configure(int* blocks_per_sm);
cudaError_t merge_rows_launch(const Params& p, cudaStream_t stream);  // MODE_MERGE, k <= KSPLIT
constexpr int EDIT_WINDOW_MAX = 1024;  // longest penalty window of mxs_sample_topk_edits
// The reference's pre-sampler edits, one CTA per row (mxs_sample_topk_edits).
cudaError_t edits_launch(float* logits, int64_t rows, int64_t ld, int64_t vocab, const int32_t* special,
                         int n_special, const int32_t* hist, int64_t hist_stride, const int32_t* hist_len,
                         int repeat_last_n, double rp, double fp, double pp, int32_t* edit_col, double* edit_val,
                         uint32_t* edit_cnt, int edit_cap, cudaStream_t stream);

// Vocab-sharded tie rows (mxs_multi.cu): the rows a merge handed back for
// their tie order, resolved from lists instead of full rows.
struct VocabReplayArgs {
    const float* shard = nullptr;  // this rank's shard rows
    int64_t ld = 0, cols = 0, col_offset = 0;
    int rank = 0, world = 1, k = 1;
    const uint64_t* log = nullptr;  // this rank's streaming lists (ShardLog)
    int log_cap = 0, S = 1, tpc = 1;
    const uint32_t* log_count = nullptr;
    const int32_t* list = nullptr;  // tie rows, ascending; n of them (host count)
    int64_t n = 0, rows = 0;
    const uint64_t* p1_cand = nullptr;  // gathered shard lists [world][rows][p1_cap]
    const uint32_t* p1_count = nullptr;
    const uint32_t* p1_flags = nullptr;
    int p1_cap = 0;
    uint64_t* out = nullptr;  // this rank's replay lists [n][cap2]
    uint32_t* out_count = nullptr;
    uint32_t* out_flags = nullptr;
    const uint64_t* g_cand = nullptr;  // every rank's replay lists [world][n][cap2]
    const uint32_t* g_count = nullptr;
    const uint32_t* g_flags = nullptr;
    int cap2 = 0;
    uint32_t* need_full = nullptr;  // [n]: 1 when the row must be sampled from its full logits
};
// Per tie row: rank 0 replays the reference's heap process over its shard and
// lists the heap (k entries, heap order); every later rank lists its logits
// above a lower bound of the k-th largest logit of the earlier shards, in
// column order.
cudaError_t vocab_replay_emit_launch(const VocabReplayArgs& a, cudaStream_t stream);
// Per tie row, on every rank: rank 0's heap, then every later rank's list
// offered in order; sort, draw into the outputs of `draw` (rows of the batch).
cudaError_t vocab_replay_merge_launch(const VocabReplayArgs& a, const Params& draw, cudaStream_t stream);
cudaError_t stream_path_launch(const Params& p, int grid, cudaStream_t stream,
                               cudaEvent_t ev_start = nullptr, cudaEvent_t ev_stop = nullptr);
}  // namespace mxs
