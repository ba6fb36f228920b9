// Launch interface of the three-kernel path (mxs_stream.cu).
#pragma once
#include <cstddef>
#include <cuda_runtime.h>

namespace mxs {
struct Params;
constexpr int KSPLIT = 64;           // largest k the three-kernel path takes
constexpr int SPLIT_ROW_CAP = 1024;  // candidate list entries per row
size_t stream_smem_bytes();
cudaError_t stream_path_configure(int* blocks_per_sm);
cudaError_t stream_path_launch(const Params& p, int grid, int exact_grid, cudaStream_t stream,
                               cudaEvent_t ev_start = nullptr, cudaEvent_t ev_stop = nullptr);
}  // namespace mxs
