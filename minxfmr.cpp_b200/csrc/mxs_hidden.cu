// mxs_sample_from_hidden: the output projection kept on the device, then the
// sampler. The reference computes the logits of a decode step from the last
// hidden state and the output weight matrix (src/api/minxfmr.cpp:1918-2036;
// on its CUDA backend, src/backend/cuda/cuda_backend.cu:731-780) and copies
// them to the host to sample (cuda_backend.cu:1440-1442). Here the logits are
// a cuBLAS GEMM (bf16 operands, fp32 accumulation and output) into HBM, and the
// sampler reads them there: only the hidden states cross PCIe.
//
// cuBLAS is looked up at run time in the library the process has loaded (torch
// loads one), else libcublas.so.12 from the loader's path, as NCCL is for the
// vocab-sharded call; the library does not link it.
#include <dlfcn.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include <cublas_v2.h>
#include <cuda_runtime.h>

#include "../../include/mxs_sampler.h"

namespace {

struct CublasFns {
    bool tried = false, ok = false;
    cublasStatus_t (*create)(cublasHandle_t*) = nullptr;
    cublasStatus_t (*set_stream)(cublasHandle_t, cudaStream_t) = nullptr;
    cublasStatus_t (*gemm_ex)(cublasHandle_t, cublasOperation_t, cublasOperation_t, int, int, int, const void*,
                              const void*, cudaDataType, int, const void*, cudaDataType, int, const void*, void*,
                              cudaDataType, int, cublasComputeType_t, cublasGemmAlgo_t) = nullptr;
};

template <typename F>
bool bind(void* h, const char* name, F& fn) {
    fn = reinterpret_cast<F>(dlsym(h, name));
    return fn != nullptr;
}

CublasFns& cublas() {
    static CublasFns f;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (!f.tried) {
        f.tried = true;
        void* h = dlopen("libcublas.so.12", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libcublas.so.12", RTLD_NOW);
        f.ok = h && bind(h, "cublasCreate_v2", f.create) && bind(h, "cublasSetStream_v2", f.set_stream) &&
               bind(h, "cublasGemmEx", f.gemm_ex);
    }
    return f;
}

constexpr int MAX_DEVICES = 64;
struct DeviceState {
    std::mutex mu;  // held for a whole call: the handle and the logits buffer are reused
    cublasHandle_t handle = nullptr;
    float* logits = nullptr;
    size_t logits_bytes = 0;
};
DeviceState g_state[MAX_DEVICES];

}  // namespace

extern "C" int mxs_sample_from_hidden(const void* d_hidden, int64_t ld_hidden, const void* d_weight,
                                      int64_t ld_weight, int64_t rows, int64_t d_model, int64_t vocab,
                                      double temperature, int top_k, double top_p, double min_p, const double* d_u,
                                      int32_t* d_next, int32_t* d_topk_idx, double* d_topk_prob,
                                      float* d_logits_out, int64_t ld_logits, void* stream) {
    if (rows < 0 || d_model <= 0 || vocab <= 0 || vocab > INT32_MAX || d_model > INT32_MAX || rows > INT32_MAX ||
        ld_hidden < d_model || ld_weight < d_model)
        return MXS_ERR_INVALID;
    if (rows == 0) return MXS_OK;
    if (!d_hidden || !d_weight || !d_u || !d_next) return MXS_ERR_INVALID;
    // the sampler's fast path wants 16-byte aligned rows: a leading dimension
    // that is a multiple of 4 floats
    const int64_t ldl = d_logits_out ? ld_logits : (vocab + 3) / 4 * 4;
    if (ldl < vocab) return MXS_ERR_INVALID;
    CublasFns& f = cublas();
    if (!f.ok) return MXS_ERR_CUDA;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return MXS_ERR_NO_DEVICE;
    DeviceState& s = g_state[dev];
    std::lock_guard<std::mutex> lk(s.mu);
    if (!s.handle && f.create(&s.handle) != CUBLAS_STATUS_SUCCESS) return MXS_ERR_CUDA;
    float* logits = d_logits_out;
    if (!logits) {
        const size_t need = sizeof(float) * (size_t)rows * (size_t)ldl;
        if (s.logits_bytes < need) {
            if (s.logits) {
                if (cudaDeviceSynchronize() != cudaSuccess) return MXS_ERR_CUDA;  // earlier calls may still read it
                cudaFree(s.logits);
                s.logits = nullptr;
                s.logits_bytes = 0;
            }
            if (cudaMalloc(&s.logits, need) != cudaSuccess) return MXS_ERR_CUDA;
            s.logits_bytes = need;
        }
        logits = s.logits;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (f.set_stream(s.handle, st) != CUBLAS_STATUS_SUCCESS) return MXS_ERR_CUDA;
    // logits (row-major rows x ldl) = hidden (rows x d) . weight (vocab x d)^T.
    // In cuBLAS's column-major terms: logits^T (vocab x rows, ld ldl) =
    // op(W) . hidden^T, op transposing the column-major d x vocab view of the
    // row-major weight; hidden^T is the column-major d x rows view of hidden.
    const float alpha = 1.0f, beta = 0.0f;
    if (f.gemm_ex(s.handle, CUBLAS_OP_T, CUBLAS_OP_N, (int)vocab, (int)rows, (int)d_model, &alpha, d_weight,
                  CUDA_R_16BF, (int)ld_weight, d_hidden, CUDA_R_16BF, (int)ld_hidden, &beta, logits, CUDA_R_32F,
                  (int)ldl, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT) != CUBLAS_STATUS_SUCCESS)
        return MXS_ERR_CUDA;
    return mxs_sample_topk_ex(logits, rows, vocab, ldl, temperature, top_k, top_p, min_p, d_u, d_next, d_topk_idx,
                              d_topk_prob, nullptr, nullptr, 0, stream);
}
