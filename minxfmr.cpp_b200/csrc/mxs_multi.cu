// Multi-GPU entry points of the C ABI (include/mxs_sampler.h):
//   mxs_sample_rowsharded   - this rank's rows of a batch split over the ranks,
//                             no collective (rows are independent);
//   mxs_sample_vocabsharded - every rank holds the same rows but only its own
//                             column shard; shard candidates -> one NCCL
//                             all-gather group -> merge and draw, then the rows
//                             whose merged lists show a tie are gathered whole
//                             and sampled again, because the reference's tie
//                             order depends on every logit of the row.
// The reference samples one row on the host (src/api/minxfmr.cpp:2091-2171);
// these are the sharded forms of that seam.
//
// NCCL is not linked: the communicator a caller passes was made by the NCCL the
// process has already loaded, so its functions are looked up at run time in
// that same library (the process's global symbols, then an already loaded
// libnccl.so.2, then libnccl.so.2 from the loader's search path).
#include <dlfcn.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include <cuda_runtime.h>
#include <nccl.h>

#include "../../include/mxs_sampler.h"
#include "mxs_launch.h"
#include "mxs_sampler_kernel.cuh"
#include "mxs_stream.h"

namespace {

struct NcclFns {
    bool tried = false, ok = false;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    ncclResult_t (*comm_count)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*comm_user_rank)(const ncclComm_t, int*) = nullptr;
};

template <typename F>
bool bind(void* h, const char* name, F& fn) {
    fn = reinterpret_cast<F>(dlsym(h, name));
    return fn != nullptr;
}

bool bind_all(void* h, NcclFns& f) {
    return bind(h, "ncclAllGather", f.all_gather) && bind(h, "ncclGroupStart", f.group_start) &&
           bind(h, "ncclGroupEnd", f.group_end) && bind(h, "ncclCommCount", f.comm_count) &&
           bind(h, "ncclCommUserRank", f.comm_user_rank);
}

NcclFns& nccl() {
    static NcclFns f;
    if (!f.tried) {
        f.tried = true;
        f.ok = bind_all(RTLD_DEFAULT, f);
        if (!f.ok) {
            void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
            if (!h) h = dlopen("libnccl.so.2", RTLD_NOW);
            f.ok = h && bind_all(h, f);
        }
    }
    return f;
}

// Device buffers of the vocab-sharded path, per device, grown on demand.
struct Buf {
    void* p = nullptr;
    size_t n = 0;
    int get(size_t bytes) {
        if (bytes <= n) return MXS_OK;
        if (p) {
            if (cudaDeviceSynchronize() != cudaSuccess) return MXS_ERR_CUDA;  // earlier calls may still use it
            cudaFree(p);
            p = nullptr;
            n = 0;
        }
        const size_t want = std::max<size_t>(bytes, 1 << 16);
        if (cudaMalloc(&p, want) != cudaSuccess) return MXS_ERR_CUDA;
        n = want;
        return MXS_OK;
    }
};

enum {
    B_CAND, B_CNT, B_FLG, B_CAND_ALL, B_CNT_ALL, B_FLG_ALL, B_RFLAGS, B_LIST, B_LIST2, B_LOGCNT,
    B_P2, B_P2CNT, B_P2FLG, B_P2ALL, B_P2CNTALL, B_P2FLGALL, B_NEEDFULL,
    B_SHARD_ROWS, B_SHARD_ALL, B_FULL, B_U, B_NEXT, B_IDX, B_PROB, B_SFLAGS, NBUF
};

constexpr int MAX_DEVICES = 64;
// One lock per device: ranks driven from threads of one process (one thread per
// GPU, each with its own communicator) never block each other, since each
// holds only its own device's lock across its collectives.
std::mutex g_mu[MAX_DEVICES];
Buf g_buf[MAX_DEVICES][NBUF];
uint32_t* g_count_host[MAX_DEVICES];  // pinned: the number of rows needing the full-row pass
// rows of the last call per device: resolved from lists (ties) / gathered whole
int64_t g_stat_list[MAX_DEVICES], g_stat_full[MAX_DEVICES];

// Tie rows are sampled whole in chunks of this many rows (bounds the gathered
// full rows to chunk x vocab fp32 per GPU).
constexpr int64_t FULL_CHUNK = 512;

// Rows with MXS_ROW_EXACT, in ascending order (one CTA: every rank must list
// the same rows in the same order, since the list orders the next all-gather).
__global__ void list_exact_rows(const uint32_t* flags, int64_t rows, int32_t* list, uint32_t* count) {
    __shared__ int warp_tot[32];
    __shared__ int base;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    if (tid == 0) base = 0;
    __syncthreads();
    for (int64_t r0 = 0; r0 < rows; r0 += blockDim.x) {
        const int64_t r = r0 + tid;
        const bool e = r < rows && (flags[r] & MXS_ROW_EXACT);
        const uint32_t bal = __ballot_sync(0xffffffffu, e);
        if (lane == 0) warp_tot[w] = __popc(bal);
        __syncthreads();
        int before = base;
        for (int i = 0; i < w; ++i) before += warp_tot[i];
        if (e) list[before + __popc(bal & ((1u << lane) - 1u))] = (int32_t)r;
        __syncthreads();
        if (tid == 0)
            for (int i = 0; i < (int)(blockDim.x >> 5); ++i) base += warp_tot[i];
        __syncthreads();
    }
    if (tid == 0) *count = (uint32_t)base;
}

// list2 = [list[i] for i < n if flag[i]], in order (one CTA, as list_exact_rows).
__global__ void list_flagged_rows(const uint32_t* flag, const int32_t* list, int64_t n, int32_t* list2,
                                  uint32_t* count) {
    __shared__ int warp_tot[32];
    __shared__ int base;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    if (tid == 0) base = 0;
    __syncthreads();
    for (int64_t r0 = 0; r0 < n; r0 += blockDim.x) {
        const int64_t r = r0 + tid;
        const bool e = r < n && flag[r] != 0u;
        const uint32_t bal = __ballot_sync(0xffffffffu, e);
        if (lane == 0) warp_tot[w] = __popc(bal);
        __syncthreads();
        int before = base;
        for (int i = 0; i < w; ++i) before += warp_tot[i];
        if (e) list2[before + __popc(bal & ((1u << lane) - 1u))] = list[r];
        __syncthreads();
        if (tid == 0)
            for (int i = 0; i < (int)(blockDim.x >> 5); ++i) base += warp_tot[i];
        __syncthreads();
    }
    if (tid == 0) *count = (uint32_t)base;
}

// out[i][c] = shard[list[i0 + i]][c]
__global__ void gather_shard_rows(const float* shard, int64_t ld, const int32_t* list, int64_t i0, int64_t n,
                                  int64_t cols, float* out) {
    const int64_t total = n * cols;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / cols, c = t - i * cols;
        out[t] = shard[(int64_t)list[i0 + i] * ld + c];
    }
}

// full[i][s * cols + c] = all[s][i][c]; u_sub[i] = u[list[i0 + i]]
__global__ void assemble_full_rows(const float* all, int world, int64_t n, int64_t cols, float* full,
                                   const double* u, const int32_t* list, int64_t i0, double* u_sub) {
    const int64_t vocab = cols * world, total = n * vocab;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / vocab, j = t - i * vocab;
        const int64_t s = j / cols, c = j - s * cols;
        full[t] = all[(s * n + i) * cols + c];
        if (j == 0) u_sub[i] = u[list[i0 + i]];
    }
}

// Put the full-row results of rows list[i0 .. i0 + n) in place.
__global__ void scatter_full_results(const int32_t* list, int64_t i0, int64_t n, int k, const int32_t* next_sub,
                                     const int32_t* idx_sub, const double* prob_sub, const uint32_t* flags_sub,
                                     int32_t* next, int32_t* idx, double* prob, uint32_t* flags) {
    const int64_t total = n * (int64_t)k;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / k, j = t - i * k;
        const int64_t r = list[i0 + i];
        if (idx) idx[r * k + j] = idx_sub[t];
        if (prob) prob[r * k + j] = prob_sub[t];
        if (j == 0) {
            next[r] = next_sub[i];
            flags[r] |= flags_sub[i];
        }
    }
}

__global__ void fill_flags(uint32_t* flags, int64_t rows, uint32_t v) {
    for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < rows; r += (int64_t)gridDim.x * blockDim.x)
        flags[r] = v;
}

// The merge keeps at most this many survivors per row (mxs_merge_sample's
// limit); above it every row takes the full-row pass.
constexpr int MERGE_K_MAX = 2048;

int grid_for(int64_t total) { return (int)std::min<int64_t>((total + 255) / 256, 148 * 8); }

int clamp_k(int top_k, int64_t vocab) {
    int64_t k = top_k <= 0 ? 1 : top_k;
    return (int)std::min<int64_t>(k, vocab);
}

}  // namespace

extern "C" {

int mxs_sample_rowsharded(const float* d_local_logits, int64_t global_rows, int rank, int world, int64_t vocab,
                          int64_t ld, double temperature, int top_k, double top_p, double min_p,
                          const double* d_u_global, int32_t* d_next, int32_t* d_topk_idx, double* d_topk_prob,
                          uint32_t* d_row_flags, int64_t* local_rows, void* stream) {
    if (global_rows < 0 || world <= 0 || rank < 0 || rank >= world) return MXS_ERR_INVALID;
    const int64_t per = (global_rows + world - 1) / world;
    const int64_t r0 = std::min<int64_t>(global_rows, (int64_t)rank * per);
    const int64_t n = std::min<int64_t>(global_rows, r0 + per) - r0;
    if (local_rows) *local_rows = n;
    if (n == 0) return MXS_OK;
    if (!d_u_global) return MXS_ERR_INVALID;
    return mxs_sample_topk_ex(d_local_logits, n, vocab, ld, temperature, top_k, top_p, min_p, d_u_global + r0,
                              d_next, d_topk_idx, d_topk_prob, d_row_flags, nullptr, 0, stream);
}

int mxs_sample_vocabsharded(const float* d_shard_logits, int64_t rows, int64_t shard_cols, int64_t ld,
                            double temperature, int top_k, double top_p, double min_p, const double* d_u,
                            int32_t* d_next, int32_t* d_topk_idx, double* d_topk_prob, uint32_t* d_row_flags,
                            void* nccl_comm, void* stream) {
    if (rows < 0 || shard_cols <= 0 || ld < shard_cols || !nccl_comm) return MXS_ERR_INVALID;
    if (rows == 0) return MXS_OK;
    if (!d_shard_logits || !d_u || !d_next) return MXS_ERR_INVALID;
    NcclFns& f = nccl();
    if (!f.ok) return MXS_ERR_COMM;
    const ncclComm_t comm = static_cast<ncclComm_t>(nccl_comm);
    int world = 0, rank = 0;
    if (f.comm_count(comm, &world) != ncclSuccess || f.comm_user_rank(comm, &rank) != ncclSuccess || world <= 0)
        return MXS_ERR_COMM;
    const int64_t vocab = shard_cols * world;
    if (vocab > INT32_MAX) return MXS_ERR_INVALID;
    const int k_use = clamp_k(top_k, vocab);
    const int k_shard = (int)std::min<int64_t>(k_use, shard_cols);
    // First-pass lists: each shard's logits above its k-th largest, and those
    // equal to it up to the cap (a list cut there is flagged and the merge
    // checks whether the cut matters).
    const int cap = (k_shard + 16 + 3) / 4 * 4;
    // Tie rows are resolved from lists when every rank can list its shard:
    // k <= KSPLIT (the two-kernel path keeps the streaming lists) and k within
    // a shard. The list of a later shard holds fewer than ~2k logits above the
    // earlier shards' k-th largest values for any but adversarial rows.
    const bool list_ties = k_use <= mxs::KSPLIT && k_use <= shard_cols;
    const int cap2 = std::min(256, 2 * k_use + 64);
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return MXS_ERR_NO_DEVICE;
    std::lock_guard<std::mutex> lk(g_mu[dev]);
    Buf* b = g_buf[dev];
    int rc;
    if ((rc = b[B_CAND].get(sizeof(uint64_t) * rows * cap)) || (rc = b[B_CNT].get(4 * rows)) ||
        (rc = b[B_FLG].get(4 * rows)) || (rc = b[B_CAND_ALL].get(sizeof(uint64_t) * rows * cap * world)) ||
        (rc = b[B_CNT_ALL].get(4 * rows * world)) || (rc = b[B_FLG_ALL].get(4 * rows * world)) ||
        (rc = b[B_RFLAGS].get(4 * rows)) || (rc = b[B_LIST].get(4 * rows + 16)) ||
        (rc = b[B_LIST2].get(4 * rows + 16)) || (rc = b[B_LOGCNT].get(4 * rows)))
        return rc;
    if (!g_count_host[dev] && cudaMallocHost(&g_count_host[dev], sizeof(uint32_t)) != cudaSuccess)
        return MXS_ERR_CUDA;
    uint64_t* cand = static_cast<uint64_t*>(b[B_CAND].p);
    uint32_t* cnt = static_cast<uint32_t*>(b[B_CNT].p);
    uint32_t* flg = static_cast<uint32_t*>(b[B_FLG].p);
    uint64_t* cand_all = static_cast<uint64_t*>(b[B_CAND_ALL].p);
    uint32_t* cnt_all = static_cast<uint32_t*>(b[B_CNT_ALL].p);
    uint32_t* flg_all = static_cast<uint32_t*>(b[B_FLG_ALL].p);
    uint32_t* rflags = d_row_flags ? d_row_flags : static_cast<uint32_t*>(b[B_RFLAGS].p);
    int32_t* list = static_cast<int32_t*>(b[B_LIST].p);
    uint32_t* list_count = reinterpret_cast<uint32_t*>(list + rows);
    uint32_t* log_count = static_cast<uint32_t*>(b[B_LOGCNT].p);
    mxs::ShardLog log;

    if (k_use > MERGE_K_MAX) {
        fill_flags<<<grid_for(rows), 256, 0, st>>>(rflags, rows, MXS_ROW_EXACT);
        if (cudaGetLastError() != cudaSuccess) return MXS_ERR_CUDA;
    } else {
        // 1. this shard's candidate lists (and its streaming lists, kept for tie rows)
        rc = mxs::shard_step(d_shard_logits, rows, shard_cols, ld, (int64_t)rank * shard_cols, top_k, cap, cand, cnt,
                             flg, list_ties ? log_count : nullptr, stream, &log);
        if (rc) return rc;
        // 2. every shard's lists on every rank, as [world][rows][cap]
        if (f.group_start() != ncclSuccess) return MXS_ERR_COMM;
        ncclResult_t r1 = f.all_gather(cand, cand_all, (size_t)rows * cap, ncclUint64, comm, st);
        ncclResult_t r2 = f.all_gather(cnt, cnt_all, (size_t)rows, ncclUint32, comm, st);
        ncclResult_t r3 = f.all_gather(flg, flg_all, (size_t)rows, ncclUint32, comm, st);
        if (f.group_end() != ncclSuccess || r1 != ncclSuccess || r2 != ncclSuccess || r3 != ncclSuccess)
            return MXS_ERR_COMM;
        // 3. merge and draw (identical on every rank)
        rc = mxs_merge_sample(cand_all, cnt_all, flg_all, world, cap, rows, vocab, temperature, top_k, top_p, min_p, d_u,
                              d_next, d_topk_idx, d_topk_prob, rflags, stream);
        if (rc) return rc;
    }
    // 4. rows the merge handed back
    list_exact_rows<<<1, 1024, 0, st>>>(rflags, rows, list, list_count);
    if (cudaGetLastError() != cudaSuccess) return MXS_ERR_CUDA;
    if (cudaMemcpyAsync(g_count_host[dev], list_count, sizeof(uint32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return MXS_ERR_CUDA;
    int64_t nx = *g_count_host[dev];
    g_stat_list[dev] = 0;
    g_stat_full[dev] = nx;
    if (nx == 0) return MXS_OK;
    const int32_t* full_list = list;
    if (list_ties && k_use <= MERGE_K_MAX) {
        // 5. tie rows from lists: rank 0's heap over its shard and every later
        // shard's logits that can still enter, gathered and replayed on every rank
        if ((rc = b[B_P2].get(sizeof(uint64_t) * nx * cap2)) || (rc = b[B_P2CNT].get(4 * nx)) ||
            (rc = b[B_P2FLG].get(4 * nx)) || (rc = b[B_P2ALL].get(sizeof(uint64_t) * nx * cap2 * world)) ||
            (rc = b[B_P2CNTALL].get(4 * nx * world)) || (rc = b[B_P2FLGALL].get(4 * nx * world)) ||
            (rc = b[B_NEEDFULL].get(4 * nx)))
            return rc;
        mxs::VocabReplayArgs a;
        a.shard = d_shard_logits;
        a.ld = ld;
        a.cols = shard_cols;
        a.col_offset = (int64_t)rank * shard_cols;
        a.rank = rank;
        a.world = world;
        a.k = k_use;
        a.log = log.valid ? log.cand : nullptr;  // a rank without lists flags every row: the full pass takes them
        a.log_cap = log.cap;
        a.S = log.S;
        a.tpc = log.tpc;
        a.log_count = log_count;
        a.list = list;
        a.n = nx;
        a.rows = rows;
        a.p1_cand = cand_all;
        a.p1_count = cnt_all;
        a.p1_flags = flg_all;
        a.p1_cap = cap;
        a.out = static_cast<uint64_t*>(b[B_P2].p);
        a.out_count = static_cast<uint32_t*>(b[B_P2CNT].p);
        a.out_flags = static_cast<uint32_t*>(b[B_P2FLG].p);
        a.g_cand = static_cast<uint64_t*>(b[B_P2ALL].p);
        a.g_count = static_cast<uint32_t*>(b[B_P2CNTALL].p);
        a.g_flags = static_cast<uint32_t*>(b[B_P2FLGALL].p);
        a.cap2 = cap2;
        a.need_full = static_cast<uint32_t*>(b[B_NEEDFULL].p);
        if (mxs::vocab_replay_emit_launch(a, st) != cudaSuccess) return MXS_ERR_CUDA;
        if (f.group_start() != ncclSuccess) return MXS_ERR_COMM;
        ncclResult_t r1 = f.all_gather(a.out, b[B_P2ALL].p, (size_t)nx * cap2, ncclUint64, comm, st);
        ncclResult_t r2 = f.all_gather(a.out_count, b[B_P2CNTALL].p, (size_t)nx, ncclUint32, comm, st);
        ncclResult_t r3 = f.all_gather(a.out_flags, b[B_P2FLGALL].p, (size_t)nx, ncclUint32, comm, st);
        if (f.group_end() != ncclSuccess || r1 != ncclSuccess || r2 != ncclSuccess || r3 != ncclSuccess)
            return MXS_ERR_COMM;
        mxs::Params d{};
        d.rows = rows;
        d.temperature = temperature;
        double tp = top_p, mp = min_p;
        if (tp <= 0.0 || tp > 1.0) tp = 1.0;  // src/api/minxfmr.cpp:2109-2111
        if (mp < 0.0) mp = 0.0;
        if (mp > 1.0) mp = 1.0;
        d.top_p = tp;
        d.min_p = mp;
        d.k_use = k_use;
        d.u = d_u;
        d.next = d_next;
        d.topk_idx = d_topk_idx;
        d.topk_prob = d_topk_prob;
        if (mxs::vocab_replay_merge_launch(a, d, st) != cudaSuccess) return MXS_ERR_CUDA;
        // rows still without a draw: NaN, overflowing lists
        int32_t* list2 = static_cast<int32_t*>(b[B_LIST2].p);
        uint32_t* list2_count = reinterpret_cast<uint32_t*>(list2 + rows);
        list_flagged_rows<<<1, 1024, 0, st>>>(a.need_full, list, nx, list2, list2_count);
        if (cudaGetLastError() != cudaSuccess) return MXS_ERR_CUDA;
        if (cudaMemcpyAsync(g_count_host[dev], list2_count, sizeof(uint32_t), cudaMemcpyDeviceToHost, st) !=
                cudaSuccess ||
            cudaStreamSynchronize(st) != cudaSuccess)
            return MXS_ERR_CUDA;
        g_stat_list[dev] = nx - *g_count_host[dev];
        nx = *g_count_host[dev];
        g_stat_full[dev] = nx;
        if (nx == 0) return MXS_OK;
        full_list = list2;
    }
    // 6. the remaining rows are gathered whole and sampled again
    const int64_t ch = std::min<int64_t>(nx, FULL_CHUNK);
    if ((rc = b[B_SHARD_ROWS].get(4 * ch * shard_cols)) || (rc = b[B_SHARD_ALL].get(4 * ch * vocab)) ||
        (rc = b[B_FULL].get(4 * ch * vocab)) || (rc = b[B_U].get(8 * ch)) || (rc = b[B_NEXT].get(4 * ch)) ||
        (rc = b[B_IDX].get(4 * ch * k_use)) || (rc = b[B_PROB].get(8 * ch * k_use)) ||
        (rc = b[B_SFLAGS].get(4 * ch)))
        return rc;
    for (int64_t i0 = 0; i0 < nx; i0 += ch) {
        const int64_t n = std::min<int64_t>(ch, nx - i0);
        float* mine = static_cast<float*>(b[B_SHARD_ROWS].p);
        float* all = static_cast<float*>(b[B_SHARD_ALL].p);
        float* full = static_cast<float*>(b[B_FULL].p);
        double* u_sub = static_cast<double*>(b[B_U].p);
        gather_shard_rows<<<grid_for(n * shard_cols), 256, 0, st>>>(d_shard_logits, ld, full_list, i0, n, shard_cols,
                                                                     mine);
        if (cudaGetLastError() != cudaSuccess) return MXS_ERR_CUDA;
        if (f.all_gather(mine, all, (size_t)(n * shard_cols), ncclFloat32, comm, st) != ncclSuccess)
            return MXS_ERR_COMM;
        assemble_full_rows<<<grid_for(n * vocab), 256, 0, st>>>(all, world, n, shard_cols, full, d_u, full_list, i0,
                                                                 u_sub);
        if (cudaGetLastError() != cudaSuccess) return MXS_ERR_CUDA;
        int32_t* next_sub = static_cast<int32_t*>(b[B_NEXT].p);
        int32_t* idx_sub = static_cast<int32_t*>(b[B_IDX].p);
        double* prob_sub = static_cast<double*>(b[B_PROB].p);
        uint32_t* flags_sub = static_cast<uint32_t*>(b[B_SFLAGS].p);
        rc = mxs_sample_topk_ex(full, n, vocab, vocab, temperature, top_k, top_p, min_p, u_sub, next_sub,
                                d_topk_idx ? idx_sub : nullptr, d_topk_prob ? prob_sub : nullptr, flags_sub, nullptr,
                                0, stream);
        if (rc) return rc;
        scatter_full_results<<<grid_for(n * k_use), 256, 0, st>>>(full_list, i0, n, k_use, next_sub, idx_sub, prob_sub,
                                                                   flags_sub, d_next, d_topk_idx, d_topk_prob, rflags);
        if (cudaGetLastError() != cudaSuccess) return MXS_ERR_CUDA;
    }
    return MXS_OK;
}

int mxs_vocabsharded_stats(int64_t* tie_rows_from_lists, int64_t* rows_gathered_whole) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return MXS_ERR_NO_DEVICE;
    std::lock_guard<std::mutex> lk(g_mu[dev]);
    if (tie_rows_from_lists) *tie_rows_from_lists = g_stat_list[dev];
    if (rows_gathered_whole) *rows_gathered_whole = g_stat_full[dev];
    return MXS_OK;
}

}  // extern "C"
