// Fused sm_100a sampling kernel (see mxs_sampler_kernel.cuh for the design).
#include <cmath>
#include <cstdint>
#include <cuda_runtime.h>

#include "mxs_rowfinish.cuh"
#include "mxs_launch.h"

namespace mxs {

// Candidate buffer over the threshold: raise the threshold to the k-th largest
// key held and drop what falls below it. If ties keep the buffer too full to
// take another step, the row is marked for the exact replay and the threshold
// becomes NaN, which no logit passes.
__device__ __forceinline__ void shrink_candidates(uint32_t* ckey, int32_t* cidx, Misc& sm, int cnt, int k) {
    const uint32_t kth = block_select_kth(ckey, cnt, min(k, cnt), sm);
    const int n = block_compact_ge(ckey, cidx, sm, cnt, kth);
    if (threadIdx.x == 0) {
        if (n > CAP - SUB) {
            sm.thr = __int_as_float(0x7fc00000);
            sm.flags |= FLAG_OVERFLOW;
        } else {
            sm.thr = fkey_inv(kth);
        }
    }
    __syncthreads();
}

// Finish row `row` from the candidate buffer (every logit >= the row's k-th
// largest value is in it unless `flags` says otherwise).
__device__ void finish_row(const Params& p, int64_t row, uint32_t flags, unsigned char* region, Misc& sm) {
    const int tid = threadIdx.x;
    const int k = p.k_use;
    uint32_t* ckey = reinterpret_cast<uint32_t*>(region);
    int32_t* cidx = reinterpret_cast<int32_t*>(region + CAP * 4);
    bool exact = (flags & (FLAG_NAN | FLAG_OVERFLOW | FLAG_UNSCANNED)) != 0;
    if (!(flags & FLAG_TIMEOUT) && !exact) {
        int cnt = sm.cnt;
        if (cnt < k) {
            exact = true;
        } else if (cnt > k) {
            const uint32_t kth = block_select_kth(ckey, cnt, k, sm);
            cnt = block_compact_ge(ckey, cidx, sm, cnt, kth);
            exact = (cnt != k);  // more than k at or above the cut: a tie straddles it
        }
        if (!exact) {
            constexpr int PER = SORTMAX / NT;
            uint32_t kk[PER];
            int32_t ii[PER];
#pragma unroll
            for (int r = 0; r < PER; ++r) {
                const int i = tid + r * NT;
                kk[r] = (i < k) ? ckey[i] : 0u;
                ii[r] = (i < k) ? cidx[i] : 0;
            }
            __syncthreads();
            int P = 1;
            while (P < k) P <<= 1;
            uint64_t* sb = reinterpret_cast<uint64_t*>(region);
#pragma unroll
            for (int r = 0; r < PER; ++r) {
                const int i = tid + r * NT;
                if (i < P) sb[i] = (i < k) ? ((uint64_t)kk[r] << 32) | (uint32_t)ii[r] : 0ull;
            }
            __syncthreads();
            block_sort_desc(sb, P);
            int tie = 0;
            for (int i = tid; i + 1 < k; i += NT) tie |= ((sb[i] >> 32) == (sb[i + 1] >> 32));
            exact = __syncthreads_or(tie) != 0;
            if (!exact) {
                Ent* e = reinterpret_cast<Ent*>(region);
                for (int i = tid; i < k; i += NT) {
                    const uint64_t w = sb[i];
                    e[i] = Ent{fkey_inv((uint32_t)(w >> 32)), (int32_t)(uint32_t)w};
                }
                __syncthreads();
                block_draw(p, row, e, k, reinterpret_cast<double*>(region + SORTMAX * 8), sm);
            }
        }
    }
    // MODE_MERGE holds no logits: a row that needs the replay is handed back.
    const bool can_replay = (p.mode != MODE_MERGE);
    if (!(flags & FLAG_TIMEOUT) && exact && can_replay) exact_row(p, row, (flags & FLAG_NAN) ? 1 : ((flags & FLAG_UNSCANNED) ? -1 : 0), region, sm);
    if (tid == 0) {
        const uint32_t f = (flags & ~FLAG_UNSCANNED) | (exact ? FLAG_EXACT : 0u);
        if (p.row_flags) p.row_flags[row] = f;
        if ((f & FLAG_TIMEOUT) || (exact && !can_replay)) p.next[row] = -1;
        if (f & FLAG_TIMEOUT) atomicOr(p.status, f);
    }
    __syncthreads();
}

// MODE_EMIT: publish the row's candidate list (all logits of the shard >= the
// shard's k-th largest value) with global column indices.
__device__ void emit_list(const Params& p, int64_t row, uint32_t flags, unsigned char* region, Misc& sm) {
    uint32_t* ckey = reinterpret_cast<uint32_t*>(region);
    int32_t* cidx = reinterpret_cast<int32_t*>(region + CAP * 4);
    if (flags & FLAG_UNSCANNED) flags = (flags & ~FLAG_UNSCANNED) | FLAG_OVERFLOW;
    int cnt = (flags & FLAG_OVERFLOW) ? 0 : sm.cnt;
    if (!(flags & (FLAG_NAN | FLAG_OVERFLOW | FLAG_TIMEOUT)) && cnt > p.k_use) {
        const uint32_t kth = block_select_kth(ckey, cnt, p.k_use, sm);
        cnt = block_compact_ge(ckey, cidx, sm, cnt, kth);
    }
    if (cnt > p.out_cap) flags |= FLAG_OVERFLOW;
    if (flags & (FLAG_NAN | FLAG_OVERFLOW | FLAG_TIMEOUT)) cnt = 0;
    uint64_t* dst = p.out_cand + row * p.out_cap;
    for (int i = threadIdx.x; i < cnt; i += NT)
        dst[i] = ((uint64_t)ckey[i] << 32) | (uint32_t)(cidx[i] + (int32_t)p.col_offset);
    if (threadIdx.x == 0) {
        p.out_count[row] = (uint32_t)cnt;
        p.out_flags[row] = flags;
        if (flags & FLAG_TIMEOUT) atomicOr(p.status, flags);
    }
    __syncthreads();
}

__device__ __forceinline__ void row_done(const Params& p, int64_t row, uint32_t flags, unsigned char* region,
                                         Misc& sm) {
    if (p.mode == MODE_EMIT)
        emit_list(p, row, flags, region, sm);
    else
        finish_row(p, row, flags, region, sm);
}

// Append a list of packed (key << 32 | index) candidates to the buffer, taking
// only those at or above the running threshold.
__device__ void append_list(const uint64_t* src, int n, uint32_t* ckey, int32_t* cidx, Misc& sm, int k) {
    for (int i0 = 0; i0 < n; i0 += SUB) {
        const float thr = sm.thr;
        const uint32_t tk = fkey(thr);
        const bool thr_nan = thr != thr;
        uint32_t m = 0;
        uint32_t key[4];
        int32_t idx[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int i = i0 + threadIdx.x * 4 + q;
            key[q] = 0;
            idx[q] = 0;
            if (i < n) {
                const uint64_t w = __ldcg(src + i);
                key[q] = (uint32_t)(w >> 32);
                idx[q] = (int32_t)(uint32_t)w;
                if (!thr_nan && key[q] >= tk) m |= 1u << q;
            }
        }
        block_append4(ckey, cidx, sm, m, key, idx);
        __syncthreads();
        const int cn = sm.cnt;
        if (cn > CAP - SUB) shrink_candidates(ckey, cidx, sm, cn, k);
    }
}

template <bool TMA>
__global__ void __launch_bounds__(NT, 2) sample_kernel(Params p) {
    extern __shared__ __align__(128) unsigned char smem[];
    float* ring = reinterpret_cast<float*>(smem);
    unsigned char* region = smem + RING_BYTES;
    uint32_t* ckey = reinterpret_cast<uint32_t*>(region);
    int32_t* cidx = reinterpret_cast<int32_t*>(region + CAP * 4);
    Misc& sm = *reinterpret_cast<Misc*>(region + REGION_BYTES);
    const int tid = threadIdx.x;
    const int k = p.k_use;
    const int64_t V = p.vocab;

    if (p.mode == MODE_MERGE) {  // rows of gathered shard lists
        for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
            if (tid == 0) {
                uint32_t f = 0;
                for (int sh = 0; sh < p.nshards; ++sh) {
                    if (p.in_flags) f |= p.in_flags[(int64_t)sh * p.rows + row];
                    if (p.in_count[(int64_t)sh * p.rows + row] > (uint32_t)p.in_cap) f |= FLAG_OVERFLOW;
                }
                sm.flags = f;
                sm.cnt = 0;
                sm.thr = -INFINITY;
            }
            __syncthreads();
            if (!(sm.flags & (FLAG_NAN | FLAG_OVERFLOW | FLAG_TIMEOUT))) {
                for (int sh = 0; sh < p.nshards; ++sh) {
                    const int64_t sl = (int64_t)sh * p.rows + row;
                    append_list(p.in_cand + sl * p.in_cap, (int)p.in_count[sl], ckey, cidx, sm, k);
                }
            }
            finish_row(p, row, sm.flags, region, sm);
        }
        return;
    }
    if (k > KFAST) {  // no streaming select for very large k: every row is replayed
        for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) row_done(p, row, FLAG_UNSCANNED, region, sm);
        return;
    }

    const int64_t G = gridDim.x;
    const int64_t nj = (p.units > (int64_t)blockIdx.x) ? (p.units - blockIdx.x + G - 1) / G : 0;
    const int S = p.S, TPC = p.tiles_per_chunk;
    const int64_t NTL = (V + TILE - 1) / TILE;

    // Producer state (thread 0): the next tile to load, over this CTA's units.
    int64_t pj = 0;
    int pt = 0;
    uint32_t pseq = 0;
    uint64_t pol = 0;
    if (TMA && tid == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&sm.bar[s], 1);
        fence_mbar_init();
        pol = policy_evict_first();
    }
    __syncthreads();
    auto unit_tiles = [&](int64_t u) -> int {
        const int64_t t0 = (int64_t)(u % S) * TPC;
        return (int)min((int64_t)TPC, NTL - t0);
    };
    auto issue = [&]() {
        if (pj >= nj) return;
        const int64_t u = blockIdx.x + pj * G;
        const int64_t row = u / S;
        const int64_t a = ((int64_t)(u % S) * TPC + pt) * TILE;
        const int64_t b = min(a + TILE, V);
        const uint32_t bytes = (uint32_t)(((b - a) & ~int64_t(3)) * 4);
        const int s = pseq % STAGES;
        if (bytes) {
            mbar_arrive_expect_tx(&sm.bar[s], bytes);
            bulk_g2s(ring + s * TILE, p.logits + row * p.ld + a, bytes, &sm.bar[s], pol);
        } else {
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&sm.bar[s])) : "memory");
        }
        ++pseq;
        if (++pt == unit_tiles(u)) {
            pt = 0;
            ++pj;
        }
    };
    if (TMA && tid == 0)
        for (int s = 0; s < STAGES; ++s) issue();

    uint32_t cseq = 0;
    for (int64_t j = 0; j < nj; ++j) {
        const int64_t u = blockIdx.x + j * G;
        const int64_t row = u / S;
        const int c = (int)(u % S);
        const int nt = unit_tiles(u);
        const float* xr = p.logits + row * p.ld;
        if (tid == 0) {
            sm.cnt = 0;
            sm.thr = -INFINITY;
            sm.flags = 0;
        }
        __syncthreads();
        int nan = 0;
        for (int t = 0; t < nt; ++t) {
            const int64_t a = ((int64_t)c * TPC + t) * TILE;
            const int len = (int)(min(a + TILE, V) - a);
            const int bulk_n = len & ~3;
            const int s = cseq % STAGES;
            if (TMA) {
                if (!mbar_wait_bounded(&sm.bar[s], (cseq / STAGES) & 1)) atomicOr(&sm.flags, FLAG_TIMEOUT);
            }
            const float* st = ring + s * TILE;
            for (int sub = 0; sub * SUB < len; ++sub) {
                const int off = sub * SUB + tid * 4;
                float v[4];
                uint32_t valid = 0;
                if (TMA && off + 4 <= bulk_n) {
                    const float4 f = *reinterpret_cast<const float4*>(st + off);
                    v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
                    valid = 0xF;
                } else {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int jj = off + q;
                        v[q] = 0.f;
                        if (jj < len) {
                            v[q] = (TMA && jj < bulk_n) ? st[jj] : xr[a + jj];
                            valid |= 1u << q;
                        }
                    }
                }
                const float thr = sm.thr;
                uint32_t m = 0;
                uint32_t key[4];
                int32_t idx[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const bool ok = (valid >> q) & 1u;
                    nan |= (ok && v[q] != v[q]);
                    if (ok && v[q] >= thr) m |= 1u << q;
                    key[q] = fkey(v[q]);
                    idx[q] = (int32_t)(a + off + q);
                }
                block_append4(ckey, cidx, sm, m, key, idx);
                __syncthreads();
                const int cnt = sm.cnt;
                if (cnt > CAP - SUB) shrink_candidates(ckey, cidx, sm, cnt, k);
            }
            if (TMA && tid == 0) {
                fence_proxy_async_smem();
                issue();
            }
            ++cseq;
        }
        uint32_t flags = sm.flags | (__syncthreads_or(nan) ? FLAG_NAN : 0u);
        if (S == 1) {
            row_done(p, row, flags, region, sm);
            continue;
        }
        // S > 1: publish this chunk's candidates >= its k-th largest key; the
        // last chunk of the row to finish merges them and finishes the row.
        int cnt = sm.cnt;
        if (!(flags & (FLAG_NAN | FLAG_OVERFLOW | FLAG_TIMEOUT)) && cnt > k) {
            const uint32_t kth = block_select_kth(ckey, cnt, k, sm);
            cnt = block_compact_ge(ckey, cidx, sm, cnt, kth);
        }
        if (cnt > p.outcap) flags |= FLAG_OVERFLOW;
        const int64_t slot = row * S + c;
        if (!(flags & FLAG_OVERFLOW)) {
            uint64_t* dst = p.chunk_cand + slot * p.outcap;
            for (int i = tid; i < cnt; i += NT) dst[i] = ((uint64_t)ckey[i] << 32) | (uint32_t)cidx[i];
        }
        if (tid == 0) {
            p.chunk_count[slot] = (uint32_t)cnt;
            if (flags) atomicOr(&p.row_state[row], flags);
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) sm.last = (atomicAdd(&p.row_counter[row], 1u) == (uint32_t)(S - 1));
        __syncthreads();
        if (!sm.last) continue;
        __threadfence();
        if (tid == 0) {
            p.row_counter[row] = 0;
            sm.flags = atomicExch(&p.row_state[row], 0u);
            sm.cnt = 0;
            sm.thr = -INFINITY;
        }
        __syncthreads();
        const uint32_t rf = sm.flags;
        if (!(rf & (FLAG_NAN | FLAG_OVERFLOW | FLAG_TIMEOUT))) {
            for (int cc = 0; cc < S; ++cc) {
                const int64_t sl = row * S + cc;
                append_list(p.chunk_cand + sl * p.outcap, (int)__ldcg(p.chunk_count + sl), ckey, cidx, sm, k);
            }
        }
        row_done(p, row, sm.flags | rf, region, sm);
    }
    if (TMA && tid == 0)
        for (int s = 0; s < STAGES; ++s) mbar_inval(&sm.bar[s]);
}

// ---------------------------------------------------------------------------
// Host-side launch.
// ---------------------------------------------------------------------------
size_t sample_kernel_smem_bytes() { return SMEM_BYTES; }

cudaError_t sample_kernel_configure(int* blocks_per_sm) {
    cudaError_t e = cudaFuncSetAttribute(sample_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)SMEM_BYTES);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(sample_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, sample_kernel<true>, NT, SMEM_BYTES);
}

cudaError_t sample_kernel_launch(const Params& p, int grid, bool tma, cudaStream_t stream) {
    if (tma)
        sample_kernel<true><<<grid, NT, SMEM_BYTES, stream>>>(p);
    else
        sample_kernel<false><<<grid, NT, SMEM_BYTES, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace mxs
