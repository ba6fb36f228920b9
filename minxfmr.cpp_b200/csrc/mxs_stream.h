// Launch interface of the two-kernel path (mxs_stream.cu).
#pragma once
#include <cstddef>
#include <cuda_runtime.h>

namespace mxs {
struct Params;
constexpr int KSPLIT = 128;          // largest k the two-kernel path takes
constexpr int SPLIT_ROW_CAP = 1024;  // candidate list entries per row
constexpr int S_TILE = 8192;         // logits per ring stage of the streaming kernel (32 KB)
constexpr int S_STAGES = 3;          // ring depth (96 KB in flight per CTA)
size_t stream_smem_bytes();
cudaError_t stream_path_configure(int* blocks_per_sm);
cudaError_t stream_path_launch(const Params& p, int grid, cudaStream_t stream,
                               cudaEvent_t ev_start = nullptr, cudaEvent_t ev_stop = nullptr);
}  // namespace mxs
