// C ABI of the sampler (include/mxs_sampler.h): argument checks with the
// reference's clamps, launch planning, workspace layout, host-buffer path.
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include <cuda_runtime.h>

#include "../../include/mxs_sampler.h"
#include "mxs_launch.h"
#include "mxs_stream.h"
#include "mxs_sampler_kernel.cuh"

namespace {

using mxs::Params;

constexpr int MAX_DEVICES = 64;

struct HostBuffers {
    float* logits = nullptr;
    size_t logits_bytes = 0;
    double* u = nullptr;
    int32_t* next = nullptr;
    int32_t* idx = nullptr;
    double* prob = nullptr;
    size_t rows_cap = 0, topk_cap = 0;
};

// Sticky status word of each device: every sampling launch ORs the flags of its
// timed-out rows into it, whichever workspace the call used (library-owned,
// caller-owned or the fixed array of the allocation-free entry point).
__device__ uint32_t g_status_word;

struct Device {
    bool ready = false;
    uint32_t* status = nullptr;  // device address of g_status_word on this device
    int sms = 0;
    int blocks_per_sm = 0;
    void* ws = nullptr;  // library-owned workspace (zeroed at allocation)
    cudaEvent_t ev_start = nullptr, ev_stop = nullptr;  // mxs_set_profile_events
    // The two-kernel path leaves its per-row counters clear; a call with the
    // same layout on the library workspace can skip clearing them again.
    int64_t clean_rows = -1;
    size_t clean_off = 0;
    size_t ws_bytes = 0;
    HostBuffers hb;
    std::mutex hb_mu;
    void* edits = nullptr;  // edit lists of mxs_sample_topk_edits, grown on demand
    size_t edits_bytes = 0;  // held for a whole host-buffer call: its buffers are reused by the next
};

std::mutex g_mu;
Device g_dev[MAX_DEVICES];

int current_device(Device** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return MXS_ERR_NO_DEVICE;
    Device& d = g_dev[dev];
    if (!d.ready) {
        cudaDeviceProp prop;
        if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return MXS_ERR_NO_DEVICE;
        if (prop.major != 10) return MXS_ERR_NO_DEVICE;  // built for sm_100a only
        int bps = 0;
        if (mxs::sample_kernel_configure(&bps) != cudaSuccess || bps < 1) return MXS_ERR_CUDA;
        int bps2 = 0;
        if (mxs::stream_path_configure(&bps2) != cudaSuccess || bps2 < 1) return MXS_ERR_CUDA;
        bps = std::min(bps, bps2);
        void* st = nullptr;
        if (cudaGetSymbolAddress(&st, g_status_word) != cudaSuccess || !st) return MXS_ERR_CUDA;
        d.status = static_cast<uint32_t*>(st);
        d.sms = prop.multiProcessorCount;
        d.blocks_per_sm = bps;
        d.ready = true;
    }
    *out = &d;
    return MXS_OK;
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Launch plan and workspace layout for one call.
struct Plan {
    int k_use = 1;
    int S = 1, tpc = 1, grid = 1, outcap = 0;
    bool split = false;  // two-kernel path (stream -> finish, which also replays tie rows)
    size_t off_rcand = 0, off_rcnt = 0, off_rflag = 0, off_rbound = 0, zero_bytes = 0;
    int64_t units = 0;
    size_t off_counter = 0, off_state = 0, off_status = 0, off_ccount = 0, off_cand = 0, off_heap = 0,
           off_prob = 0, total = 0;
};

int clamp_k(int top_k, int64_t vocab) {
    int64_t k = top_k <= 0 ? 1 : top_k;  // src/api/minxfmr.cpp:1567, :2091-2093
    if (k > vocab) k = vocab;
    return (int)k;
}

// Test hooks (mxs_set_test_hooks; off unless a test sets them). Plain values,
// never read from the environment, so nothing outside the caller's own calls
// can change what a sampling call does.
struct TestHooks {
    int64_t drop_tile = -1;     // CTA 0's streaming producer stops before this tile (-1: off)
    int replay_warp_min = 1;    // tie rows of a finish CTA replayed one per warp from this many
    int path = 0;               // 0: default planning; 2: the CTA-synchronous kernel for every k
};
TestHooks g_hooks;

// The two-kernel path takes sampling calls with k <= KSPLIT on 16-byte aligned
// rows, unless a test forced the CTA-synchronous kernel.
int path_override() { return g_hooks.path; }

// Candidate list entries per row on the two-kernel path: per chunk, the first
// tile's candidates (about 2k) and the would-enter superset of the later tiles
// (about k (1 + ln(tiles))); a simulation of the bound on N(0, 2^2) rows at
// V = 151,936 gives ~420 entries at k = 50 and ~900 at k = 128. A fuller list
// overflows and the row is replayed from its full logits.
int split_row_cap(int S, int k) { return S * std::max(mxs::SPLIT_ROW_CAP, 12 * k + 512); }

bool use_split(int64_t vocab, int64_t ld, const float* logits, int k_use) {
    const bool tma = (reinterpret_cast<uintptr_t>(logits) % 16 == 0) && (ld % 4 == 0);
    (void)vocab;
    return tma && k_use <= mxs::KSPLIT && path_override() == 0;
}

constexpr int64_t SPLIT_MIN_TILES = 4;

Plan make_plan(const Device& d, int64_t rows, int64_t vocab, int k_use, bool merge_mode, bool split = false) {
    Plan pl;
    pl.k_use = k_use;
    pl.split = split;
    const int64_t full = (int64_t)d.sms * d.blocks_per_sm;
    const int tile = split ? mxs::S_TILE : mxs::TILE;  // logits per ring stage of the chosen kernel
    const int64_t ntl = (vocab + tile - 1) / tile;
    if (merge_mode || k_use > mxs::KFAST) {
        pl.S = 1;
        pl.tpc = (int)ntl;
        pl.units = rows;
        pl.grid = (int)std::max<int64_t>(1, std::min<int64_t>(rows, full));
    } else {
        int64_t s0 = std::max<int64_t>(1, full / std::max<int64_t>(rows, 1));
        s0 = std::min(s0, ntl);
        // Two-kernel path: at least SPLIT_MIN_TILES tiles per unit. Every unit
        // keeps k or more candidates for the finish warp, so many one-tile units
        // make its list long (one row at k = 50: 62 us per call with one tile
        // per unit, 39 us with four).
        if (split) s0 = std::min<int64_t>(s0, std::max<int64_t>(1, ntl / SPLIT_MIN_TILES));
        const int64_t tpc = (ntl + s0 - 1) / s0;
        pl.S = (int)((ntl + tpc - 1) / tpc);
        pl.tpc = (int)tpc;
        pl.units = rows * pl.S;
        pl.grid = (int)std::max<int64_t>(1, std::min<int64_t>(pl.units, full));
    }
    pl.outcap = (pl.S > 1 && !split) ? k_use + 256 : 0;
    size_t o = 0;
    pl.off_status = o;
    o = align_up(o + 256, 256);
    // The per-row counters must read zero at the start of every call; the kernel
    // leaves them zero. They only exist for S > 1, which needs rows < `full`, so
    // they sit at offsets that depend on the device alone and never alias the
    // (call-dependent) candidate lists of an earlier call.
    pl.off_counter = o;
    o = align_up(o + sizeof(uint32_t) * (size_t)full, 256);
    pl.off_state = o;
    o = align_up(o + sizeof(uint32_t) * (size_t)full, 256);
    pl.off_ccount = o;
    if (split) {
        // per-row counters and flags: must read zero when a call starts; the
        // finish kernel clears them after use
        pl.off_rcnt = o;
        pl.off_rflag = pl.off_rcnt + sizeof(uint32_t) * (size_t)rows;
        pl.off_rbound = pl.off_rflag + sizeof(uint32_t) * (size_t)rows;
        pl.zero_bytes = 3 * sizeof(uint32_t) * (size_t)rows;
        o = align_up(pl.off_rbound + sizeof(uint32_t) * (size_t)rows, 256);
        pl.off_rcand = o;
        o = align_up(o + sizeof(uint64_t) * (size_t)rows * split_row_cap(pl.S, pl.k_use), 256);
    } else if (pl.S > 1) {
        o = align_up(o + sizeof(uint32_t) * (size_t)rows * pl.S, 256);
        pl.off_cand = o;
        o = align_up(o + sizeof(uint64_t) * (size_t)rows * pl.S * pl.outcap, 256);
    }
    if (k_use > mxs::HEAP_SMEM_MAX && !merge_mode) {
        pl.off_heap = o;
        o = align_up(o + sizeof(mxs::Ent) * (size_t)pl.grid * k_use, 256);
        pl.off_prob = o;
        o = align_up(o + sizeof(double) * (size_t)pl.grid * k_use, 256);
    }
    pl.total = o;
    return pl;
}

int ensure_library_ws(Device& d, size_t bytes, cudaStream_t stream) {
    if (d.ws_bytes >= bytes) return MXS_OK;
    if (d.ws) {
        // Earlier calls on any stream may still use the old buffer.
        if (cudaDeviceSynchronize() != cudaSuccess) return MXS_ERR_CUDA;
        cudaFree(d.ws);
        d.ws = nullptr;
        d.ws_bytes = 0;
    }
    d.clean_rows = -1;
    size_t want = std::max<size_t>(bytes, 1 << 20);
    if (cudaMalloc(&d.ws, want) != cudaSuccess) return MXS_ERR_CUDA;
    if (cudaMemsetAsync(d.ws, 0, want, stream) != cudaSuccess) return MXS_ERR_CUDA;
    d.ws_bytes = want;
    return MXS_OK;
}

void fill_workspace(Params& p, const Plan& pl, void* ws, const Device& d) {
    char* b = static_cast<char*>(ws);
    p.status = d.status;
    p.row_counter = reinterpret_cast<uint32_t*>(b + pl.off_counter);
    p.row_state = reinterpret_cast<uint32_t*>(b + pl.off_state);
    p.chunk_count = reinterpret_cast<uint32_t*>(b + pl.off_ccount);
    p.chunk_cand = pl.S > 1 ? reinterpret_cast<uint64_t*>(b + pl.off_cand) : nullptr;
    p.heap_ws = pl.off_heap ? reinterpret_cast<mxs::Ent*>(b + pl.off_heap) : nullptr;
    p.prob_ws = pl.off_prob ? reinterpret_cast<double*>(b + pl.off_prob) : nullptr;
    if (pl.split) {
        p.row_cand = reinterpret_cast<uint64_t*>(b + pl.off_rcand);
        p.row_cnt = reinterpret_cast<uint32_t*>(b + pl.off_rcnt);
        p.row_flag = reinterpret_cast<uint32_t*>(b + pl.off_rflag);
        p.row_bound = reinterpret_cast<uint32_t*>(b + pl.off_rbound);
        p.row_cap = split_row_cap(pl.S, pl.k_use);
    }
}

void clamp_p(double* top_p, double* min_p) {  // src/api/minxfmr.cpp:2109-2111
    if (*top_p <= 0.0 || *top_p > 1.0) *top_p = 1.0;
    if (*min_p < 0.0) *min_p = 0.0;
    if (*min_p > 1.0) *min_p = 1.0;
}

int launch(Params& p, const Plan& pl, cudaStream_t stream, int sms = 148, cudaEvent_t ev0 = nullptr,
           cudaEvent_t ev1 = nullptr, Device* lib_ws_owner = nullptr) {
    p.S = pl.S;
    p.tiles_per_chunk = pl.tpc;
    p.units = pl.units;
    p.outcap = pl.outcap;
    if (pl.split) {
        p.debug_drop_tile = g_hooks.drop_tile;
        p.replay_warp_min = g_hooks.replay_warp_min;
        const bool clean = lib_ws_owner && lib_ws_owner->clean_rows == p.rows && lib_ws_owner->clean_off == pl.off_rcnt;
        if (lib_ws_owner) lib_ws_owner->clean_rows = -1;
        if (!clean && cudaMemsetAsync(p.row_cnt, 0, pl.zero_bytes, stream) != cudaSuccess) return MXS_ERR_CUDA;
        if (mxs::stream_path_launch(p, pl.grid, stream, ev0, ev1) != cudaSuccess) return MXS_ERR_CUDA;
        if (lib_ws_owner) {
            lib_ws_owner->clean_rows = p.rows;
            lib_ws_owner->clean_off = pl.off_rcnt;
        }
        return MXS_OK;
    }
    if (lib_ws_owner) lib_ws_owner->clean_rows = -1;
    const bool tma = (reinterpret_cast<uintptr_t>(p.logits) % 16 == 0) && (p.ld % 4 == 0);
    if (ev0) cudaEventRecord(ev0, stream);
    if (mxs::sample_kernel_launch(p, pl.grid, tma, stream) != cudaSuccess) return MXS_ERR_CUDA;
    if (ev1) cudaEventRecord(ev1, stream);
    return MXS_OK;
}

bool ws_ok(const void* ws, size_t bytes, size_t need) {
    return ws && (reinterpret_cast<uintptr_t>(ws) % 256 == 0) && bytes >= need;
}

// The reference's checks on the sampled token (src/api/minxfmr.cpp:2189-2205,
// :2232-2243), one warp per row: on a row's first generated token, a token the
// caller's table marks unusable as a first token (an invisible piece, EOS or
// a role token) is replaced by the first usable one of order[1, k); then the
// row's stop flag says whether the token is EOS.
__global__ void token_checks_kernel(int64_t rows, int k, const int32_t* order, int32_t* next, const uint8_t* cls,
                                    int64_t vocab, const uint8_t* first_step, uint8_t* stop) {
    const int lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    auto bad_first = [&](int32_t t) { return t < 0 || t >= vocab || (cls[t] & MXS_TOKEN_NOT_FIRST); };
    int32_t nx = next[r];
    if (first_step && first_step[r] && bad_first(nx)) {
        for (int i0 = 1; i0 < k; i0 += 32) {
            const int i = i0 + lane;
            const int32_t alt = i < k ? order[r * k + i] : -1;
            const uint32_t ok = __ballot_sync(0xffffffffu, i < k && !bad_first(alt));
            if (ok) {
                nx = __shfl_sync(0xffffffffu, alt, __ffs(ok) - 1);
                break;
            }
        }
    }
    if (lane == 0) {
        next[r] = nx;
        if (stop) stop[r] = (nx >= 0 && nx < vocab && (cls[nx] & MXS_TOKEN_EOS)) ? 1 : 0;
    }
}

// The reference's pre-sampler edits of one call (mxs_sample_topk_edits).
struct EditSpec {
    float* logits = nullptr;
    const int32_t* special = nullptr;
    int n_special = 0;
    const int32_t* hist = nullptr;
    int64_t hist_stride = 0;
    const int32_t* hist_len = nullptr;
    int repeat_last_n = 0;
    double rp = 1.0, fp = 0.0, pp = 0.0;
    int cap = 1;
};

int sample_impl(const float* d_logits, int64_t rows, int64_t vocab, int64_t ld, double temperature, int top_k,
                double top_p, double min_p, const double* d_u, int32_t* d_next, int32_t* d_topk_idx,
                double* d_topk_prob, uint32_t* d_row_flags, void* d_workspace, size_t workspace_bytes, void* stream,
                const EditSpec* ed) {
    if (rows < 0 || vocab <= 0 || vocab > INT32_MAX || ld < vocab) return MXS_ERR_INVALID;
    if (rows == 0) return MXS_OK;
    if (!d_logits || !d_u || !d_next) return MXS_ERR_INVALID;
    std::lock_guard<std::mutex> lk(g_mu);
    Device* d;
    int rc = current_device(&d);
    if (rc) return rc;
    clamp_p(&top_p, &min_p);
    const int k_use = clamp_k(top_k, vocab);
    const Plan pl = make_plan(*d, rows, vocab, k_use, false, use_split(vocab, ld, d_logits, k_use));
    void* ws = d_workspace;
    if (!ws) {
        rc = ensure_library_ws(*d, pl.total, (cudaStream_t)stream);
        if (rc) return rc;
        ws = d->ws;
    } else if (!ws_ok(ws, workspace_bytes, pl.total)) {
        return MXS_ERR_WORKSPACE;
    }
    Params p{};
    p.logits = d_logits;
    p.rows = rows;
    p.vocab = vocab;
    p.ld = ld;
    p.temperature = temperature;
    p.top_p = top_p;
    p.min_p = min_p;
    p.k_use = pl.k_use;
    p.u = d_u;
    p.next = d_next;
    p.topk_idx = d_topk_idx;
    p.topk_prob = d_topk_prob;
    p.row_flags = d_row_flags;
    p.mode = mxs::MODE_SAMPLE;
    fill_workspace(p, pl, ws, *d);
    if (ed) {
        // the edit lists: [rows x cap] columns, [rows x cap] values, [rows] counts
        const size_t cb = align_up(sizeof(int32_t) * (size_t)rows * ed->cap, 256);
        const size_t vb = align_up(sizeof(double) * (size_t)rows * ed->cap, 256);
        const size_t need = cb + vb + sizeof(uint32_t) * (size_t)rows;
        if (d->edits_bytes < need) {
            if (d->edits) {
                if (cudaDeviceSynchronize() != cudaSuccess) return MXS_ERR_CUDA;  // earlier calls may still use it
                cudaFree(d->edits);
                d->edits = nullptr;
                d->edits_bytes = 0;
            }
            if (cudaMalloc(&d->edits, need) != cudaSuccess) return MXS_ERR_CUDA;
            d->edits_bytes = need;
        }
        char* eb = static_cast<char*>(d->edits);
        int32_t* ecol = reinterpret_cast<int32_t*>(eb);
        double* eval = reinterpret_cast<double*>(eb + cb);
        uint32_t* ecnt = reinterpret_cast<uint32_t*>(eb + cb + vb);
        if (mxs::edits_launch(ed->logits, rows, ld, vocab, ed->special, ed->n_special, ed->hist, ed->hist_stride,
                              ed->hist_len, ed->repeat_last_n, ed->rp, ed->fp, ed->pp, ecol, eval, ecnt, ed->cap,
                              (cudaStream_t)stream) != cudaSuccess)
            return MXS_ERR_CUDA;
        p.edit_col = ecol;
        p.edit_val = eval;
        p.edit_cnt = ecnt;
        p.edit_cap = ed->cap;
    }
    return launch(p, pl, (cudaStream_t)stream, d->sms, d->ev_start, d->ev_stop, d_workspace ? nullptr : d);
}

}  // namespace

namespace mxs {
// Bytes at the start of every workspace layout on the current device that must
// read zero when a call starts: the CTA-synchronous kernel's per-row chunk
// counters, which sit at offsets that depend on the device alone. (The
// two-kernel path's per-row counters are cleared by every call on a caller
// workspace before its launch.)
int workspace_zero_prefix(size_t* bytes) {
    std::lock_guard<std::mutex> lk(g_mu);
    Device* d;
    int rc = current_device(&d);
    if (rc) return rc;
    *bytes = make_plan(*d, 1, 1, 1, false).off_ccount;
    return MXS_OK;
}

int shard_step(const float* d_shard_logits, int64_t rows, int64_t shard_cols, int64_t ld, int64_t col_offset,
               int top_k, int cap, uint64_t* d_cand, uint32_t* d_count, uint32_t* d_flags, uint32_t* d_log_count,
               void* stream, ShardLog* log) {
    if (rows < 0 || shard_cols <= 0 || ld < shard_cols || col_offset < 0 || col_offset + shard_cols > INT32_MAX)
        return MXS_ERR_INVALID;
    if (rows == 0) return MXS_OK;
    if (!d_shard_logits || !d_cand || !d_count || !d_flags) return MXS_ERR_INVALID;
    const int k_use = clamp_k(top_k, shard_cols);
    if (cap < k_use) return MXS_ERR_INVALID;
    std::lock_guard<std::mutex> lk(g_mu);
    Device* d;
    int rc = current_device(&d);
    if (rc) return rc;
    // k <= KSPLIT on 16-byte aligned rows: the two-kernel path, whose finish
    // kernel writes the lists (MODE_EMIT); otherwise the CTA kernels.
    const Plan pl = make_plan(*d, rows, shard_cols, k_use, false, use_split(shard_cols, ld, d_shard_logits, k_use));
    rc = ensure_library_ws(*d, pl.total, (cudaStream_t)stream);
    if (rc) return rc;
    Params p{};
    p.logits = d_shard_logits;
    p.rows = rows;
    p.vocab = shard_cols;
    p.ld = ld;
    p.k_use = k_use;
    p.mode = mxs::MODE_EMIT;
    p.col_offset = col_offset;
    p.out_cand = d_cand;
    p.out_count = d_count;
    p.out_flags = d_flags;
    p.out_cap = cap;
    p.log_count = pl.split ? d_log_count : nullptr;
    d->clean_rows = -1;
    fill_workspace(p, pl, d->ws, *d);
    if (log) {
        log->valid = pl.split && d_log_count != nullptr;
        log->cand = p.row_cand;
        log->cap = p.row_cap;
        log->S = pl.S;
        log->tpc = pl.tpc;
    }
    return launch(p, pl, (cudaStream_t)stream);
}
}  // namespace mxs

extern "C" {

const char* mxs_version(void) { return "mxs-sampler 0.1 sm_100a"; }

int mxs_workspace_size(int64_t rows, int64_t vocab, int top_k, size_t* bytes) {
    if (!bytes || rows < 0 || vocab <= 0 || vocab > INT32_MAX) return MXS_ERR_INVALID;
    std::lock_guard<std::mutex> lk(g_mu);
    Device* d;
    int rc = current_device(&d);
    if (rc) return rc;
    const int k_use = clamp_k(top_k, vocab);
    size_t need = make_plan(*d, rows, vocab, k_use, false).total;
    if (k_use <= mxs::KSPLIT) need = std::max(need, make_plan(*d, rows, vocab, k_use, false, true).total);
    *bytes = need;
    return MXS_OK;
}

int mxs_workspace_init(void* d_workspace, size_t workspace_bytes, void* stream) {
    if (!d_workspace) return MXS_ERR_INVALID;
    return cudaMemsetAsync(d_workspace, 0, workspace_bytes, (cudaStream_t)stream) == cudaSuccess ? MXS_OK
                                                                                                : MXS_ERR_CUDA;
}

int mxs_sample_topk_ex(const float* d_logits, int64_t rows, int64_t vocab, int64_t ld, double temperature,
                       int top_k, double top_p, double min_p, const double* d_u, int32_t* d_next,
                       int32_t* d_topk_idx, double* d_topk_prob, uint32_t* d_row_flags, void* d_workspace,
                       size_t workspace_bytes, void* stream) {
    return sample_impl(d_logits, rows, vocab, ld, temperature, top_k, top_p, min_p, d_u, d_next, d_topk_idx,
                       d_topk_prob, d_row_flags, d_workspace, workspace_bytes, stream, nullptr);
}

int mxs_sample_topk_edits(float* d_logits, int64_t rows, int64_t vocab, int64_t ld, double temperature, int top_k,
                          double top_p, double min_p, const int32_t* d_special, int n_special,
                          const int32_t* d_history, int64_t hist_stride, const int32_t* d_hist_len, int repeat_last_n,
                          double repeat_penalty, double frequency_penalty, double presence_penalty, const double* d_u,
                          int32_t* d_next, int32_t* d_topk_idx, double* d_topk_prob, uint32_t* d_row_flags,
                          void* stream) {
    if (rows < 0 || vocab <= 0 || vocab > INT32_MAX || ld < vocab || n_special < 0 || hist_stride < 0)
        return MXS_ERR_INVALID;
    if (rows == 0) return MXS_OK;
    if (!d_logits || !d_u || !d_next || (n_special > 0 && !d_special) ||
        (hist_stride > 0 && (!d_history || !d_hist_len)))
        return MXS_ERR_INVALID;
    const int64_t window = repeat_last_n < 0 ? hist_stride : std::min<int64_t>(repeat_last_n, hist_stride);
    if (window > mxs::EDIT_WINDOW_MAX) return MXS_ERR_INVALID;
    const int k_use = clamp_k(top_k, vocab);
    if (!use_split(vocab, ld, d_logits, k_use)) return MXS_ERR_INVALID;  // top_k <= 128, 16-byte aligned rows
    EditSpec ed;
    ed.special = d_special;
    ed.n_special = n_special;
    ed.hist = d_history;
    ed.hist_stride = hist_stride;
    ed.hist_len = d_hist_len;
    ed.repeat_last_n = repeat_last_n;
    ed.rp = repeat_penalty;
    ed.fp = frequency_penalty;
    ed.pp = presence_penalty;
    ed.cap = (int)std::max<int64_t>(1, window);
    ed.logits = d_logits;
    return sample_impl(d_logits, rows, vocab, ld, temperature, top_k, top_p, min_p, d_u, d_next, d_topk_idx,
                       d_topk_prob, d_row_flags, nullptr, 0, stream, &ed);
}

int mxs_sample_topk(const float* d_logits, int64_t rows, int64_t vocab, int64_t ld, double temperature,
                    int top_k, const double* d_u, int32_t* d_next, int32_t* d_topk_idx, double* d_topk_prob,
                    void* stream) {
    return mxs_sample_topk_ex(d_logits, rows, vocab, ld, temperature, top_k, 1.0, 0.0, d_u, d_next, d_topk_idx,
                              d_topk_prob, nullptr, nullptr, 0, stream);
}

int mxs_sample_topk_host(const float* h_logits, int64_t rows, int64_t vocab, int64_t ld, double temperature,
                         int top_k, double top_p, double min_p, const double* h_u, int32_t* h_next,
                         int32_t* h_topk_idx, double* h_topk_prob, void* stream) {
    if (rows < 0 || vocab <= 0 || vocab > INT32_MAX || ld < vocab) return MXS_ERR_INVALID;
    if (rows == 0) return MXS_OK;
    if (!h_logits || !h_u || !h_next) return MXS_ERR_INVALID;
    cudaStream_t st = (cudaStream_t)stream;
    const int k_use = clamp_k(top_k, vocab);
    HostBuffers* hb;
    Device* d;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        int rc = current_device(&d);
        if (rc) return rc;
    }
    // One host-buffer call per device at a time: the device-side copies of the
    // logits and outputs are reused by every call on the device.
    std::lock_guard<std::mutex> hlk(d->hb_mu);
    {
        hb = &d->hb;
        const size_t lb = sizeof(float) * (size_t)rows * vocab;
        const size_t tk = (size_t)rows * k_use;
        if (hb->logits_bytes < lb || hb->rows_cap < (size_t)rows || hb->topk_cap < tk) {
            if (cudaDeviceSynchronize() != cudaSuccess) return MXS_ERR_CUDA;
            cudaFree(hb->logits);
            cudaFree(hb->u);
            cudaFree(hb->next);
            cudaFree(hb->idx);
            cudaFree(hb->prob);
            *hb = HostBuffers{};
            if (cudaMalloc(&hb->logits, lb) != cudaSuccess || cudaMalloc(&hb->u, sizeof(double) * rows) != cudaSuccess ||
                cudaMalloc(&hb->next, sizeof(int32_t) * rows) != cudaSuccess ||
                cudaMalloc(&hb->idx, sizeof(int32_t) * tk) != cudaSuccess ||
                cudaMalloc(&hb->prob, sizeof(double) * tk) != cudaSuccess)
                return MXS_ERR_CUDA;
            hb->logits_bytes = lb;
            hb->rows_cap = rows;
            hb->topk_cap = tk;
        }
    }
    // Logits are packed densely on the device (ld = vocab).
    cudaError_t e;
    if (ld == vocab)
        e = cudaMemcpyAsync(hb->logits, h_logits, sizeof(float) * rows * vocab, cudaMemcpyHostToDevice, st);
    else
        e = cudaMemcpy2DAsync(hb->logits, sizeof(float) * vocab, h_logits, sizeof(float) * ld, sizeof(float) * vocab,
                              rows, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return MXS_ERR_CUDA;
    if (cudaMemcpyAsync(hb->u, h_u, sizeof(double) * rows, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return MXS_ERR_CUDA;
    int rc = mxs_sample_topk_ex(hb->logits, rows, vocab, vocab, temperature, top_k, top_p, min_p, hb->u, hb->next,
                                h_topk_idx ? hb->idx : nullptr, h_topk_prob ? hb->prob : nullptr, nullptr, nullptr, 0,
                                stream);
    if (rc) return rc;
    if (cudaMemcpyAsync(h_next, hb->next, sizeof(int32_t) * rows, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return MXS_ERR_CUDA;
    if (h_topk_idx && cudaMemcpyAsync(h_topk_idx, hb->idx, sizeof(int32_t) * rows * k_use, cudaMemcpyDeviceToHost,
                                      st) != cudaSuccess)
        return MXS_ERR_CUDA;
    if (h_topk_prob && cudaMemcpyAsync(h_topk_prob, hb->prob, sizeof(double) * rows * k_use,
                                       cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return MXS_ERR_CUDA;
    return cudaStreamSynchronize(st) == cudaSuccess ? MXS_OK : MXS_ERR_CUDA;
}

int mxs_shard_candidates(const float* d_shard_logits, int64_t rows, int64_t shard_cols, int64_t ld,
                         int64_t col_offset, int top_k, int cap, uint64_t* d_cand, uint32_t* d_count,
                         uint32_t* d_flags, void* stream) {
    return mxs::shard_step(d_shard_logits, rows, shard_cols, ld, col_offset, top_k, cap, d_cand, d_count, d_flags,
                           nullptr, stream, nullptr);
}

int mxs_merge_sample(const uint64_t* d_cand_all, const uint32_t* d_count_all, const uint32_t* d_flags_all,
                     int nshards, int cap, int64_t rows, int64_t vocab, double temperature, int top_k, double top_p,
                     double min_p, const double* d_u, int32_t* d_next, int32_t* d_topk_idx, double* d_topk_prob,
                     uint32_t* d_row_flags, void* stream) {
    if (rows < 0 || vocab <= 0 || vocab > INT32_MAX || nshards <= 0 || cap <= 0) return MXS_ERR_INVALID;
    if (rows == 0) return MXS_OK;
    if (!d_cand_all || !d_count_all || !d_u || !d_next) return MXS_ERR_INVALID;
    const int k_use = clamp_k(top_k, vocab);
    if (k_use > mxs::KFAST) return MXS_ERR_INVALID;  // the merge keeps at most KFAST survivors
    std::lock_guard<std::mutex> lk(g_mu);
    Device* d;
    int rc = current_device(&d);
    if (rc) return rc;
    clamp_p(&top_p, &min_p);
    Params p{};
    if (k_use <= mxs::KSPLIT) {
        // one warp per row (no workspace)
        p.rows = rows;
        p.vocab = vocab;
        p.temperature = temperature;
        p.top_p = top_p;
        p.min_p = min_p;
        p.k_use = k_use;
        p.u = d_u;
        p.next = d_next;
        p.topk_idx = d_topk_idx;
        p.topk_prob = d_topk_prob;
        p.row_flags = d_row_flags;
        p.status = d->status;
        p.mode = mxs::MODE_MERGE;
        p.in_cand = d_cand_all;
        p.in_count = d_count_all;
        p.in_flags = d_flags_all;
        p.nshards = nshards;
        p.in_cap = cap;
        return mxs::merge_rows_launch(p, (cudaStream_t)stream) == cudaSuccess ? MXS_OK : MXS_ERR_CUDA;
    }
    const Plan pl = make_plan(*d, rows, vocab, k_use, true);
    rc = ensure_library_ws(*d, pl.total, (cudaStream_t)stream);
    if (rc) return rc;
    p.rows = rows;
    p.vocab = vocab;
    p.ld = vocab;
    p.temperature = temperature;
    p.top_p = top_p;
    p.min_p = min_p;
    p.k_use = k_use;
    p.u = d_u;
    p.next = d_next;
    p.topk_idx = d_topk_idx;
    p.topk_prob = d_topk_prob;
    p.row_flags = d_row_flags;
    p.mode = mxs::MODE_MERGE;
    p.in_cand = d_cand_all;
    p.in_count = d_count_all;
    p.in_flags = d_flags_all;
    p.nshards = nshards;
    p.in_cap = cap;
    d->clean_rows = -1;
    fill_workspace(p, pl, d->ws, *d);
    p.logits = nullptr;
    // no logits: launch the plain variant (no bulk copies are issued in merge mode)
    p.S = pl.S;
    p.tiles_per_chunk = pl.tpc;
    p.units = pl.units;
    p.outcap = 0;
    if (mxs::sample_kernel_launch(p, pl.grid, false, (cudaStream_t)stream) != cudaSuccess) return MXS_ERR_CUDA;
    return MXS_OK;
}

int mxs_token_checks(int64_t rows, int top_k, int64_t vocab, const int32_t* d_topk_idx, int32_t* d_next,
                     const uint8_t* d_token_class, const uint8_t* d_first_step, uint8_t* d_stop, void* stream) {
    if (rows < 0 || vocab <= 0 || vocab > INT32_MAX) return MXS_ERR_INVALID;
    if (rows == 0) return MXS_OK;
    if (!d_next || !d_token_class || (d_first_step && !d_topk_idx)) return MXS_ERR_INVALID;
    const int k_use = clamp_k(top_k, vocab);
    token_checks_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, (cudaStream_t)stream>>>(
        rows, k_use, d_topk_idx, d_next, d_token_class, vocab, d_first_step, d_stop);
    return cudaGetLastError() == cudaSuccess ? MXS_OK : MXS_ERR_CUDA;
}

int mxs_set_profile_events(void* start, void* stop) {
    if ((start == nullptr) != (stop == nullptr)) return MXS_ERR_INVALID;
    std::lock_guard<std::mutex> lk(g_mu);
    Device* d;
    int rc = current_device(&d);
    if (rc) return rc;
    d->ev_start = (cudaEvent_t)start;
    d->ev_stop = (cudaEvent_t)stop;
    return MXS_OK;
}

int mxs_set_test_hooks(int64_t drop_tile, int replay_warp_min, int path) {
    if (replay_warp_min < 1 || (path != 0 && path != 2)) return MXS_ERR_INVALID;
    std::lock_guard<std::mutex> lk(g_mu);
    g_hooks.drop_tile = drop_tile;
    g_hooks.replay_warp_min = replay_warp_min;
    g_hooks.path = path;
    return MXS_OK;
}

int mxs_get_status(uint32_t* flags, int clear) {
    if (!flags) return MXS_ERR_INVALID;
    std::lock_guard<std::mutex> lk(g_mu);
    Device* d;
    int rc = current_device(&d);
    if (rc) return rc;
    if (cudaDeviceSynchronize() != cudaSuccess) return MXS_ERR_CUDA;
    if (cudaMemcpy(flags, d->status, sizeof(uint32_t), cudaMemcpyDeviceToHost) != cudaSuccess) return MXS_ERR_CUDA;
    if (clear && cudaMemset(d->status, 0, sizeof(uint32_t)) != cudaSuccess) return MXS_ERR_CUDA;
    return MXS_OK;
}

}  // extern "C"
