// mxs_sample_topk_noalloc: the sampler for callers that must not allocate
// device memory. Some hosts hand the whole GPU to their own memory pool up front
// (a serving engine that pre-plans every byte, a plugin host that only passes
// the tensors it owns) and treat any cudaMalloc behind their back as an error,
// or forbid allocation on the per-token path altogether. This entry point takes
// its scratch from a fixed array compiled into the library instead: every GPU
// that loads libmxs.so holds MXS_NOALLOC_SCRATCH_BYTES of it until the process
// exits, and no call here allocates or frees anything.
#include <cstdint>
#include <mutex>

#include <cuda_runtime.h>

#include "../../include/mxs_sampler.h"
#include "mxs_launch.h"

namespace {

// The shared scratch. In host code this name is only a stand-in for the
// device array: its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_mxs_noalloc_scratch[MXS_NOALLOC_SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_mu;
void* g_scratch_addr[MAX_DEVICES];  // device address of the array, per device (set up once)

// With `dev` current: look up (once) the device address of the scratch array.
int scratch_address(int dev, void** out) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_mxs_noalloc_scratch) != cudaSuccess || !p) return MXS_ERR_CUDA;
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return MXS_OK;
}

}  // namespace

extern "C" int mxs_sample_topk_noalloc(const float* d_logits, int64_t rows, int64_t vocab, int64_t ld,
                                       double temperature, int top_k, double top_p, double min_p, const double* d_u,
                                       int32_t* d_next, int32_t* d_topk_idx, double* d_topk_prob,
                                       uint32_t* d_row_flags, void* stream) {
    if (rows < 0 || vocab <= 0 || vocab > INT32_MAX || ld < vocab) return MXS_ERR_INVALID;
    if (rows == 0) return MXS_OK;
    if (!d_logits || !d_u || !d_next) return MXS_ERR_INVALID;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return MXS_ERR_NO_DEVICE;
    size_t need = 0;
    int rc = mxs_workspace_size(rows, vocab, top_k, &need);
    if (rc) return rc;
    if (need > (size_t)MXS_NOALLOC_SCRATCH_BYTES) return MXS_ERR_WORKSPACE;  // shape too large for the array
    void* scratch = nullptr;
    rc = scratch_address(dev, &scratch);
    if (rc) return rc;
    // The array keeps whatever the last call left. The counters that must read
    // zero at the start of a call are cleared on the call's stream (a memset
    // allocates nothing): the device-fixed prefix here, the per-row counters of
    // the two-kernel path inside mxs_sample_topk_ex. Everything else in the
    // array is written before it is read.
    size_t zero = 0;
    rc = mxs::workspace_zero_prefix(&zero);
    if (rc) return rc;
    if (cudaMemsetAsync(scratch, 0, zero, (cudaStream_t)stream) != cudaSuccess) return MXS_ERR_CUDA;
    return mxs_sample_topk_ex(d_logits, rows, vocab, ld, temperature, top_k, top_p, min_p, d_u, d_next, d_topk_idx,
                              d_topk_prob, d_row_flags, scratch, (size_t)MXS_NOALLOC_SCRATCH_BYTES, stream);
}
