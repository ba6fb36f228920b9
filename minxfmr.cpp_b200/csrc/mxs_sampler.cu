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
    csync();
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
        const bool small = (k <= 64);
        if (cnt < k) {
            exact = true;
        } else if (cnt > k && !(small && cnt <= 64)) {
            const uint32_t kth = block_select_kth(ckey, cnt, k, sm);
            cnt = block_compact_ge(ckey, cidx, sm, cnt, kth);
            exact = (cnt != k);  // more than k at or above the cut: a tie straddles it
        }
        MXS_PROF_T0(tsort);
        if (!exact && small) {
            // cnt <= 64 entries, every logit >= the k-th largest among them:
            // one warp sorts them in registers and looks for equal neighbours
            // among the first k (and across the cut when cnt > k).
            if (tid < 32) {
                const int lane = tid;
                const uint64_t a0 = lane < cnt ? ((uint64_t)ckey[lane] << 32) | (uint32_t)cidx[lane] : 0ull;
                const uint64_t a1 =
                    lane + 32 < cnt ? ((uint64_t)ckey[lane + 32] << 32) | (uint32_t)cidx[lane + 32] : 0ull;
                uint64_t b0 = a0, b1 = a1;
                warp_sort64_desc(b0, b1);
                const uint64_t first1 = __shfl_sync(0xffffffffu, b1, 0);
                const uint64_t dn0 = __shfl_down_sync(0xffffffffu, b0, 1);
                const uint64_t n1 = __shfl_down_sync(0xffffffffu, b1, 1);
                const uint64_t n0 = (lane == 31) ? first1 : dn0;
                const int lim = (cnt > k) ? k : k - 1;  // compare pairs (i, i+1) for i < lim
                const bool tie = (lane < lim && (b0 >> 32) == (n0 >> 32)) ||
                                 (lane + 32 < lim && (b1 >> 32) == (n1 >> 32));
                const bool any = __any_sync(0xffffffffu, tie);
                if (!any) {
                    Ent* e = reinterpret_cast<Ent*>(region);
                    __syncwarp();
                    if (lane < k) e[lane] = Ent{fkey_inv((uint32_t)(b0 >> 32)), (int32_t)(uint32_t)b0};
                    if (lane + 32 < k) e[lane + 32] = Ent{fkey_inv((uint32_t)(b1 >> 32)), (int32_t)(uint32_t)b1};
                }
                if (lane == 0) sm.xn = any ? 1 : 0;
            }
            csync();
            exact = sm.xn != 0;
            MXS_PROF_ADD(4, tsort);
            if (!exact) {
                MXS_PROF_T0(tdraw);
                block_draw(p, row, reinterpret_cast<Ent*>(region), k, reinterpret_cast<double*>(region + SORTMAX * 8),
                           sm);
                MXS_PROF_ADD(5, tdraw);
            }
        } else if (!exact) {
            constexpr int PER = SORTMAX / NT;
            uint32_t kk[PER];
            int32_t ii[PER];
#pragma unroll
            for (int r = 0; r < PER; ++r) {
                const int i = tid + r * NT;
                kk[r] = (i < k) ? ckey[i] : 0u;
                ii[r] = (i < k) ? cidx[i] : 0;
            }
            csync();
            int P = 1;
            while (P < k) P <<= 1;
            uint64_t* sb = reinterpret_cast<uint64_t*>(region);
#pragma unroll
            for (int r = 0; r < PER; ++r) {
                const int i = tid + r * NT;
                if (i < P) sb[i] = (i < k) ? ((uint64_t)kk[r] << 32) | (uint32_t)ii[r] : 0ull;
            }
            csync();
            block_sort_desc(sb, P);
            int tie = 0;
            for (int i = tid; i + 1 < k; i += NT) tie |= ((sb[i] >> 32) == (sb[i + 1] >> 32));
            exact = csync_or(tie) != 0;
            MXS_PROF_ADD(4, tsort);
            if (!exact) {
                MXS_PROF_T0(tdraw);
                Ent* e = reinterpret_cast<Ent*>(region);
                for (int i = tid; i < k; i += NT) {
                    const uint64_t w = sb[i];
                    e[i] = Ent{fkey_inv((uint32_t)(w >> 32)), (int32_t)(uint32_t)w};
                }
                csync();
                block_draw(p, row, e, k, reinterpret_cast<double*>(region + SORTMAX * 8), sm);
                MXS_PROF_ADD(5, tdraw);
            }
        }
    }
    // MODE_MERGE holds no logits: a row that needs the replay is handed back.
    const bool can_replay = (p.mode != MODE_MERGE);
    if (!(flags & FLAG_TIMEOUT) && exact && can_replay) {
        MXS_PROF_T0(tex);
        exact_row(p, row, (flags & FLAG_NAN) ? 1 : ((flags & FLAG_UNSCANNED) ? -1 : 0), region, sm);
        MXS_PROF_ADD(6, tex);
    }
    if (tid == 0) {
        const uint32_t f = (flags & ~FLAG_UNSCANNED) | (exact ? FLAG_EXACT : 0u);
        if (p.row_flags) p.row_flags[row] = f;
        if ((f & FLAG_TIMEOUT) || (exact && !can_replay)) p.next[row] = -1;
        if (f & FLAG_TIMEOUT) atomicOr(p.status, f);
    }
    csync();
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
    csync();
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
        csync();
        const int cn = sm.cnt;
        if (cn > CAP - SUB) shrink_candidates(ckey, cidx, sm, cn, k);
    }
}

// End of a (row, chunk) unit; the candidate buffer holds ckey/cidx[0, sm.cnt).
// S == 1: finish the row. S > 1: publish this chunk's candidates >= its k-th
// largest key; the last chunk of the row to finish merges all of them and
// finishes the row.
__device__ void unit_end(const Params& p, int64_t row, int c, uint32_t flags, unsigned char* region, Misc& sm) {
    const int tid = threadIdx.x;
    const int k = p.k_use;
    const int S = p.S;
    uint32_t* ckey = reinterpret_cast<uint32_t*>(region);
    int32_t* cidx = reinterpret_cast<int32_t*>(region + CAP * 4);
    if (S == 1) {
        row_done(p, row, flags, region, sm);
        return;
    }
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
    csync();
    if (tid == 0) sm.last = (atomicAdd(&p.row_counter[row], 1u) == (uint32_t)(S - 1));
    csync();
    if (!sm.last) return;
    __threadfence();
    if (tid == 0) {
        p.row_counter[row] = 0;
        sm.flags = atomicExch(&p.row_state[row], 0u);
        sm.cnt = 0;
        sm.thr = -INFINITY;
    }
    csync();
    const uint32_t rf = sm.flags;
    if (!(rf & (FLAG_NAN | FLAG_OVERFLOW | FLAG_TIMEOUT))) {
        for (int cc = 0; cc < S; ++cc) {
            const int64_t sl = row * S + cc;
            append_list(p.chunk_cand + sl * p.outcap, (int)__ldcg(p.chunk_count + sl), ckey, cidx, sm, k);
        }
    }
    row_done(p, row, sm.flags | rf, region, sm);
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
            csync();
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
        pol = policy_evict_normal();
    }
    if (tid == 0) sm.dead = 0u;
    csync();
    auto unit_tiles = [&](int64_t u) -> int {
        const int64_t t0 = (int64_t)(u % S) * TPC;
        return (int)min((int64_t)TPC, NTL - t0);
    };
    auto issue = [&]() {
        if (pj >= nj || *reinterpret_cast<volatile uint32_t*>(&sm.dead)) return;
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
    const int trig = min(CAP / 2, max(512, 4 * k));
    MXS_PROF_BEGIN();
    MXS_PROF_T0(ttot);
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
        csync();
        int nan = 0;
        // Tile in checked sub-steps of SUB logits (partial tiles, the plain-load
        // variant, and re-scans after an overflow).
        auto slow_tile = [&](const float* st, const float* xr, int64_t a, int len, int bulk_n) {
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
                csync();
                const int cnt = sm.cnt;
                if (cnt > CAP - SUB) {
                    MXS_PROF_T0(ts);
                    shrink_candidates(ckey, cidx, sm, cnt, k);
                    MXS_PROF_ADD(2, ts);
                }
            }
        };
        for (int t = 0; t < nt; ++t) {
            const int64_t a = ((int64_t)c * TPC + t) * TILE;
            const int len = (int)(min(a + TILE, V) - a);
            const int bulk_n = len & ~3;
            const int s = cseq % STAGES;
            MXS_PROF_T0(tw);
            if (TMA) {
                // Once a wait has run out, no further copies are issued: the
                // remaining tiles are not waited for and their rows are flagged.
                if (*reinterpret_cast<volatile uint32_t*>(&sm.dead)) {
                    atomicOr(&sm.flags, FLAG_TIMEOUT);
                } else if (!mbar_wait_bounded(&sm.bar[s], (cseq / STAGES) & 1)) {
                    atomicOr(&sm.flags, FLAG_TIMEOUT);
                    *reinterpret_cast<volatile uint32_t*>(&sm.dead) = 1u;
                }
            }
            MXS_PROF_ADD(0, tw);
            MXS_PROF_T0(tc);
            const float* st = ring + s * TILE;
            if (TMA && len == TILE) {
                // Whole tile in shared memory: 16 logits per thread, one sync.
                const float4* st4 = reinterpret_cast<const float4*>(st);
                float4 f[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) f[q] = st4[tid + NT * q];
                float thr = sm.thr;
                if (t == 0 && k <= NT) {
                    // Seed the threshold with the k-th largest of the 256
                    // per-thread maxima: k distinct logits are >= it, so it
                    // cannot exceed the unit's k-th largest value.
                    float mx = -INFINITY;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        mx = f[q].x > mx ? f[q].x : mx;
                        mx = f[q].y > mx ? f[q].y : mx;
                        mx = f[q].z > mx ? f[q].z : mx;
                        mx = f[q].w > mx ? f[q].w : mx;
                    }
                    ckey[tid] = fkey(mx);  // the buffer is empty at a unit's first tile
                    csync();
                    thr = fkey_inv(block_select_kth(ckey, NT, k, sm));
                    if (tid == 0) sm.thr = thr;
                }
                const int cnt0 = sm.cnt;
                // max.NaN screen: NaN in any of the 16 flags the row (the exact
                // replay takes it); otherwise only lanes whose max passes build bits
                const float mxn = max16_nan(f);
                nan |= (mxn != mxn);
                if (__any_sync(0xffffffffu, mxn >= thr)) {
                    uint32_t m16 = 0;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float vv[4] = {f[q].x, f[q].y, f[q].z, f[q].w};
#pragma unroll
                        for (int c4 = 0; c4 < 4; ++c4)
                            if (vv[c4] >= thr) m16 |= 1u << (4 * q + c4);
                    }
                    block_append16(ckey, cidx, sm, m16, f, (int32_t)(a + 4 * tid));
                }
                csync();
                const int cnt = sm.cnt;
                if (cnt > CAP) {
                    // Entries were lost: drop this tile's, raise the threshold,
                    // and take the tile again in checked sub-steps.
                    csync();
                    if (tid == 0) sm.cnt = cnt0;
                    csync();
                    if (cnt0 > 0) shrink_candidates(ckey, cidx, sm, cnt0, k);
                    slow_tile(st, xr, a, len, bulk_n);
                } else if (cnt > trig) {
                    MXS_PROF_T0(ts);
                    shrink_candidates(ckey, cidx, sm, cnt, k);
                    MXS_PROF_ADD(2, ts);
                }
            } else {
                slow_tile(st, xr, a, len, bulk_n);
            }
            MXS_PROF_ADD(1, tc);
            if (TMA && tid == 0) {
                fence_proxy_async_smem();
                issue();
            }
            ++cseq;
        }
        const uint32_t flags = sm.flags | (csync_or(nan) ? FLAG_NAN : 0u);
        MXS_PROF_T0(tf);
        unit_end(p, row, c, flags, region, sm);
        MXS_PROF_ADD(3, tf);
    }
    MXS_PROF_ADD(7, ttot);
    MXS_PROF_FLUSH();
    if (TMA && tid == 0) {
        // Every issued copy must land before the CTA retires. After a timeout
        // the waits above stopped; only the last STAGES copies can be in
        // flight (a stage is reissued only after all threads waited for it).
        for (uint32_t q = pseq > STAGES ? pseq - STAGES : 0; q < pseq; ++q)
            (void)mbar_wait_bounded(&sm.bar[q % STAGES], (q / STAGES) & 1);
        for (int s = 0; s < STAGES; ++s) mbar_inval(&sm.bar[s]);
    }
}

#ifdef MXS_PROFILE
extern "C" __attribute__((visibility("default"))) int mxs_prof_read(unsigned long long* host, int clear) {
    if (cudaMemcpyFromSymbol(host, g_mxs_prof, sizeof(g_mxs_prof)) != cudaSuccess) return -3;
    if (clear) {
        static unsigned long long zeros[PROF_CTAS][PROF_PHASES];
        if (cudaMemcpyToSymbol(g_mxs_prof, zeros, sizeof(zeros)) != cudaSuccess) return -3;
    }
    return 0;
}
#endif


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
