// Internal launch interface between the C ABI (mxs_api.cu) and the kernels.
#pragma once
#include <cstddef>
#include <cuda_runtime.h>

namespace mxs {
struct Params;
size_t sample_kernel_smem_bytes();
cudaError_t sample_kernel_configure(int* blocks_per_sm);
cudaError_t sample_kernel_launch(const Params& p, int grid, bool tma, cudaStream_t stream);
int workspace_zero_prefix(size_t* bytes);  // mxs_api.cu
}  // namespace mxs
