// Internal launch interface between the C ABI (mxs_api.cu) and the kernels.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace mxs {
struct Params;
size_t sample_kernel_smem_bytes();
cudaError_t sample_kernel_configure(int* blocks_per_sm);
cudaError_t sample_kernel_launch(const Params& p, int grid, bool tma, cudaStream_t stream);
int workspace_zero_prefix(size_t* bytes);  // mxs_api.cu

// The row lists a vocab-sharded shard step leaves in the library workspace
// (two-kernel path only): every logit of a chunk's later tiles above a
// prefix-valid bound, as (key << 32 | shard column) words; they stay valid
// until the next sampling call on the device.
struct ShardLog {
    bool valid = false;
    const uint64_t* cand = nullptr;  // rows x cap
    int cap = 0, S = 1, tpc = 1;
};
// mxs_shard_candidates, plus (when d_log_count is given and the two-kernel path
// runs) each row's list length in d_log_count and the lists' location in *log.
int shard_step(const float* d_shard_logits, int64_t rows, int64_t shard_cols, int64_t ld, int64_t col_offset,
               int top_k, int cap, uint64_t* d_cand, uint32_t* d_count, uint32_t* d_flags, uint32_t* d_log_count,
               void* stream, ShardLog* log);
}  // namespace mxs
