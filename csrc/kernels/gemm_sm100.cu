// bf16 GEMM on the 5th-generation tensor cores: C[M,N] = act(A[M,K] * B[N,K]^T), f32 accumulate,
// plus the two fused tensor-parallel modes (AllGather->GEMM and GEMM->ReduceScatter).
//
// Persistent, warp-specialised, one CTA per SM (320 threads):
//   warp 0     TMA producer: A and B tiles (128-byte swizzle) into a ring of shared-memory stages
//   warp 1     allocates 512 TMEM columns; one thread issues tcgen05.mma into one of two TMEM
//              accumulators and tcgen05.commit's the stage/accumulator barriers
//   warps 2-5  epilogue: tcgen05.ld 32 columns at a time from their TMEM lane quarter, optional
//              SiLU, bf16 rounding, store to global
//   warps 6-9  communication (fused modes only): push this rank's activation shard to every peer
//              (AllGather), or pull and sum the partial tiles this rank owns (ReduceScatter)
// Two kernels: 1-SM tiles of 128x256 (M=128 MMAs, 4 stages) and 2-SM tiles of 256x256 (a CTA pair
// runs tcgen05.mma.cta_group::2; each CTA loads half of A and half of B, 6 stages), the default.
// The two accumulators let the epilogue of tile i overlap the MMAs of tile i+1. Every mbarrier
// and flag wait is bounded; a role that gives up raises a shared abort word that stops the
// others, the MMA thread drains its in-flight MMAs and the producer its in-flight TMA loads
// before the TMEM columns are freed, and the failure is recorded in the caller's error word.
// TMA reads only this GPU's memory, and no load uses cluster multicast.
// The plain tile schedule walks N fastest so consecutive CTAs share an A row block in L2.
#include <cuda_bf16.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "kernels/gemm.h"
#include "kernels/sm100.cuh"

namespace bccl {
namespace gemm {
namespace {

using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int kABytes = BM * BK * 2;
constexpr int kBBytes = BN * BK * 2;
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kTmemCols = 2 * BN;
constexpr int kThreads = 320;   // 6 GEMM warps + 4 communication warps (fused modes)
constexpr int kSmemBytes = STAGES * kStageBytes + 1024 /*alignment*/ + 256 /*barriers*/;

struct Args {
    __nv_bfloat16* C;
    int M, N, K, ldc;
    int act;      // 0 none, 1 SiLU
    int* err;     // device word: non-zero after a failed wait
    TpArgs tp;    // fused tensor-parallel modes only
};

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void red_add_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("red.relaxed.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// One 16-byte store that the switch writes into every GPU's copy of a multicast-bound buffer.
__device__ __forceinline__ void multimem_st16(void* p, const uint4& v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Bounded spin until *p >= target (relaxed polls, then one acquire fence).
__device__ __forceinline__ bool wait_geq_sys(const unsigned long long* p, unsigned long long target,
                                             const volatile int* abort) {
    for (uint32_t i = 0;; ++i) {
        if (ld_relaxed_sys_u64(p) >= target) {
            fence_sys();
            return true;
        }
        if ((i & 255u) == 255u && *abort) return false;
        if (i > (1u << 24)) return false;
        __nanosleep(i < 256 ? 32 : 256);
    }
}

// Row block `rb` of the A operand in AG mode: ranks' shards are ms/BM row blocks each;
// the schedule takes this rank's row blocks first, then chunk 0 of every peer, chunk 1 of
// every peer, ... (the order in which every rank pushes its shard).
__device__ __forceinline__ int ag_row_block(int i, const TpArgs& tp, int num_m, int block_rows = BM) {
    const int per = tp.ms / block_rows;
    const int r = tp.rank, n = tp.nranks;
    if (i < per) return r * per + i;
    i -= per;
    const int c = i / (n - 1), k = i % (n - 1);
    const int src = (r + 1 + k) % n;
    (void)num_m;
    return src * per + c;
}

// GEMM->ReduceScatter tile schedule: row blocks cycle through the owners (owner 0 chunk 0,
// owner 1 chunk 0, ..., owner 0 chunk 1, ...), the same order on every rank, so every owner's
// tiles complete (on all ranks at about the same time) all through the GEMM and its sums overlap
// the math instead of piling up behind it.
__device__ __forceinline__ int rs_row_block(int i, const TpArgs& tp, int block_rows = BM) {
    const int per = tp.ms / block_rows;
    return (i % tp.nranks) * per + i / tp.nranks;
}

// Communication warps of the fused modes (warps 6-9): AllGather pushes / ReduceScatter sums.
// TBN: the GEMM's tile width (the ReduceScatter tiles this rank owns are TBN columns wide).
template <int MODE, int TBN = BN>
__device__ __forceinline__ void comm_warps(const Args& g, int num_n, volatile int* s_abort, volatile int* s_comm_stop) {
    auto fail = [&]() {
        *s_abort = 1;
        atomicExch(g.err, 1);
    };
        const int ctid = threadIdx.x - 6 * 32, cnt_threads = kThreads - 6 * 32;
        if (MODE == kModeAllGather) {
            // Push this rank's shard, chunk by chunk, into every peer's gathered-X buffer;
            // CTA b owns slice b of every chunk. One counter bump per (peer, chunk) per CTA.
            // With a multicast-bound buffer each vector leaves this GPU once (multimem.st; the
            // switch writes every copy) instead of once per peer.
            const int per = g.tp.ms / BM;
            const size_t chunk_bytes = (size_t)BM * g.K * 2;
            const size_t slice = ((chunk_bytes + gridDim.x - 1) / gridDim.x + 15) / 16 * 16;
            const size_t lo = min(chunk_bytes, (size_t)blockIdx.x * slice), hi = min(chunk_bytes, lo + slice);
            // Only the first push_threads threads push (fewer pushing warps leave more issue slots
            // to the epilogue warps on the same SM); the others just keep the barrier company.
            const int pushers = g.tp.push_threads > 0 ? min(g.tp.push_threads, cnt_threads) : cnt_threads;
            // No waits here: the loop always runs to the end (uniform named barriers).
            for (int c = 0; c < per; ++c) {
                const char* srcp = reinterpret_cast<const char*>(g.tp.x_local) + (size_t)c * chunk_bytes;
                const size_t dst_off = ((size_t)g.tp.rank * per + c) * chunk_bytes;
                if (g.tp.xg_mc != nullptr) {
                    char* mc = reinterpret_cast<char*>(g.tp.xg_mc) + dst_off;
                    size_t o = lo + (size_t)ctid * 16;
                    const size_t step = (size_t)pushers * 16;
                    for (; ctid < pushers && o + 3 * step < hi; o += 4 * step) {  // four loads in flight
                        uint4 v[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) v[u] = *reinterpret_cast<const uint4*>(srcp + o + u * step);
#pragma unroll
                        for (int u = 0; u < 4; ++u) multimem_st16(mc + o + u * step, v[u]);
                    }
                    for (; ctid < pushers && o < hi; o += step) multimem_st16(mc + o, *reinterpret_cast<const uint4*>(srcp + o));
                } else {
                    for (size_t o = lo + (size_t)ctid * 16; ctid < pushers && o < hi; o += (size_t)pushers * 16) {
                        const uint4 v = *reinterpret_cast<const uint4*>(srcp + o);
                        for (int q = 0; q < g.tp.nranks; ++q) {
                            if (q == g.tp.rank) continue;
                            __stcg(reinterpret_cast<uint4*>(reinterpret_cast<char*>(g.tp.xg[q]) + dst_off + o), v);
                        }
                    }
                }
                asm volatile("bar.sync 2, %0;" ::"r"(cnt_threads) : "memory");
                if (ctid < g.tp.nranks && ctid != g.tp.rank) {
                    fence_sys();
                    red_add_sys(g.tp.ag_counters_peer[ctid] + (size_t)g.tp.rank * kTpMaxChunks + c, 1ull);
                }
            }
        } else if (MODE == kModeReduceScatter) {
            // Announce this call, then sum the tiles this rank owns as their N partials land.
            if (blockIdx.x == 0 && ctid < g.tp.nranks && ctid != g.tp.rank) {
                st_relaxed_sys_u64(g.tp.rs_started_peer[ctid] + g.tp.rank, g.tp.seq);
            }
            const int per = g.tp.ms / BM;
            const int own_tiles = per * num_n;
            for (int t = blockIdx.x; t < own_tiles; t += gridDim.x) {
                // Only ctid 0 writes s_comm_stop, before the barrier: every thread reads the same value.
                if (ctid == 0 && !wait_geq_sys(g.tp.rs_counters[g.tp.rank] + t,
                                               g.tp.seq * 4ull * (unsigned long long)g.tp.nranks, s_abort)) {
                    fail();
                    *s_comm_stop = 1;
                }
                asm volatile("bar.sync 2, %0;" ::"r"(cnt_threads) : "memory");
                if (*s_comm_stop) break;
                const int lrb = t / num_n, nb = t % num_n;
                const int ncols = min(TBN, g.N - nb * TBN);
                // 8 bf16 per vector; rows x ncols of the tile. kU vectors per thread per step, all
                // N partials of all kU loaded before any is summed: enough loads in flight to
                // cover memory latency with only four warps.
                constexpr int kU = 4;
                const int vec_per_row = ncols / 8;
                const int total = BM * vec_per_row;
                // Partials are pulled from every rank's staging ([M][N], this rank's rows):
                // coalesced 16-byte loads over NVLink instead of scattered remote stores.
                const size_t my_rows = (size_t)g.tp.rank * g.tp.ms * g.N;
                for (int e0 = ctid; e0 < total; e0 += kU * cnt_threads) {
                    uint4 v[kU][kMaxRanks];
                    size_t off[kU];
                    bool live[kU];
#pragma unroll
                    for (int u = 0; u < kU; ++u) {
                        const int e = e0 + u * cnt_threads;
                        const int rr = e / vec_per_row, cc = (e % vec_per_row) * 8;
                        const int lrow = lrb * BM + rr;
                        live[u] = e < total && lrow < g.tp.ms;
                        off[u] = (size_t)lrow * g.N + nb * TBN + cc;
#pragma unroll
                        for (int q = 0; q < kMaxRanks; ++q) {
                            if (live[u] && q < g.tp.nranks)
                                v[u][q] = __ldcg(reinterpret_cast<const uint4*>(g.tp.rs_stage[q] + my_rows + off[u]));
                        }
                    }
#pragma unroll
                    for (int u = 0; u < kU; ++u) {
                        if (!live[u]) continue;
                        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
                        for (int q = 0; q < kMaxRanks; ++q) {
                            if (q >= g.tp.nranks) break;
                            const uint32_t w[4] = {v[u][q].x, v[u][q].y, v[u][q].z, v[u][q].w};
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                acc[2 * j] += __uint_as_float(w[j] << 16);
                                acc[2 * j + 1] += __uint_as_float(w[j] & 0xffff0000u);
                            }
                        }
                        uint4 o = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                                             pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
                        *reinterpret_cast<uint4*>(g.tp.out + off[u]) = o;
                    }
                }
            }
        }
    }

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                const __grid_constant__ CUtensorMap tmB,
                                                                const __grid_constant__ CUtensorMap tmG,
                                                                const __grid_constant__ Args g) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);
    // full[0..S) empty[S..2S) acc_full[2S..2S+2) acc_empty[2S+2..2S+4) drain[2S+4]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
    volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* s_comm_stop = s_abort + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    auto bar = [&](int i) { return smem_u32(bars + i); };
    auto smemA = [&](int s) { return smem_u32(smem + s * kStageBytes); };
    auto smemB = [&](int s) { return smem_u32(smem + s * kStageBytes + kABytes); };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(bar(s), 1);
            mbar_init(bar(STAGES + s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(bar(2 * STAGES + a), 1);
            mbar_init(bar(2 * STAGES + 2 + a), 4);
        }
        mbar_init(bar(2 * STAGES + 4), 1);
        *s_abort = 0;
        *s_comm_stop = 0;
        fence_proxy_async_shared();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int num_m = (g.M + BM - 1) / BM, num_n = (g.N + BN - 1) / BN;
    const int tiles = num_m * num_n;
    const int kblocks = (g.K + BK - 1) / BK;
    // Tile t -> (row block, column block); N walks fastest.
    auto tile_rb = [&](int t) {
        if (MODE == kModeAllGather) return ag_row_block(t / num_n, g.tp, num_m);
        if (MODE == kModeReduceScatter) return rs_row_block(t / num_n, g.tp);
        return t / num_n;
    };
    auto fail = [&]() {
        *s_abort = 1;
        atomicExch(g.err, 1);
    };

    if (warp == 0) {
        if (lane == 0) {
            uint32_t kb = 0;
            for (int tile = blockIdx.x; tile < tiles && !*s_abort; tile += gridDim.x) {
                const int rb = tile_rb(tile);
                const int n0 = (tile % num_n) * BN;
                const CUtensorMap* amap = &tmA;
                int arow = rb * BM;
                if (MODE == kModeAllGather) {
                    const int per = g.tp.ms / BM, src = rb / per, chunk = rb % per;
                    if (src == g.tp.rank) {
                        arow = chunk * BM;  // own shard, straight from the caller's tensor
                    } else {
                        // Peer rows: wait until every CTA of rank `src` pushed this chunk here.
                        const unsigned long long* cnt = g.tp.ag_counters + (size_t)src * kTpMaxChunks + chunk;
                        if (!wait_geq_sys(cnt, g.tp.seq * (uint64_t)g.tp.contributors, s_abort)) {
                            fail();
                            break;
                        }
                        fence_proxy_async_global();  // generic-proxy writes -> TMA reads
                        amap = &tmG;
                    }
                }
                for (int k = 0; k < kblocks; ++k, ++kb) {
                    const int s = kb % STAGES;
                    const uint32_t ph = (kb / STAGES) & 1;
                    if (!mbar_wait(bar(STAGES + s), ph ^ 1, s_abort)) {
                        fail();
                        break;
                    }
                    mbar_arrive_expect_tx(bar(s), kStageBytes);
                    tma_load_2d(smemA(s), amap, bar(s), k * BK, arow);
                    tma_load_2d(smemB(s), &tmB, bar(s), k * BK, n0);
                }
            }
            // Drain: every load this thread issued lands before the CTA can exit.
            for (uint32_t i = (kb > STAGES ? kb - STAGES : 0); i < kb; ++i) {
                mbar_wait(bar(i % STAGES), (i / STAGES) & 1, s_abort, 1u << 22);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16_f32(BM, BN);
            uint32_t kb = 0, local = 0;
            for (int tile = blockIdx.x; tile < tiles && !*s_abort; tile += gridDim.x, ++local) {
                const int a = local & 1;
                const uint32_t use = local >> 1;
                if (!mbar_wait(bar(2 * STAGES + 2 + a), (use & 1) ^ 1, s_abort)) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + static_cast<uint32_t>(a * BN);
                bool ok = true;
                for (int k = 0; k < kblocks; ++k, ++kb) {
                    const int s = kb % STAGES;
                    if (!mbar_wait(bar(s), (kb / STAGES) & 1, s_abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad = smem_desc_sw128(smemA(s)), bd = smem_desc_sw128(smemB(s));
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        // +32 bytes per K=16 step inside the 128-byte swizzle atom (encoded >> 4).
                        umma_f16(d, ad + static_cast<uint64_t>(kk * 2), bd + static_cast<uint64_t>(kk * 2), idesc,
                                 (k > 0 || kk > 0) ? 1u : 0u);
                    }
                    umma_commit(bar(STAGES + s));
                }
                if (!ok) {
                    fail();
                    break;
                }
                umma_commit(bar(2 * STAGES + a));
            }
            // Drain every MMA this thread issued before TMEM is freed.
            umma_commit(bar(2 * STAGES + 4));
            mbar_wait(bar(2 * STAGES + 4), 0, s_abort, 1u << 22);
        }
    } else if (warp < 6) {
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int row_in_tile = q * 32 + lane;
        uint32_t local = 0;
        unsigned char rs_ready_checked[kMaxRanks] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int tile = blockIdx.x; tile < tiles && !*s_abort; tile += gridDim.x, ++local) {
            const int a = local & 1;
            const uint32_t use = local >> 1;
            if (!mbar_wait(bar(2 * STAGES + a), use & 1, s_abort)) {
                if (lane == 0) fail();
                break;
            }
            tc_fence_after();
            const int rb = tile_rb(tile);
            const int m0 = rb * BM, n0 = (tile % num_n) * BN;
            const int row = m0 + row_in_tile;
            __nv_bfloat16* crow = g.C + static_cast<size_t>(row) * g.ldc;
            int owner = 0;
            if (MODE == kModeReduceScatter) {
                // The partial tile stays in this rank's own staging (g.C, [M][N]); its owner
                // pulls it. The owner must have started the previous call (so it finished
                // reading this parity's staging two calls ago) before the first overwrite.
                const int per = g.tp.ms / BM;
                owner = rb / per;
                if (owner != g.tp.rank && !rs_ready_checked[owner]) {
                    if (lane == 0 && !wait_geq_sys(g.tp.rs_started + owner, g.tp.seq - 1, s_abort)) fail();
                    __syncwarp();
                    rs_ready_checked[owner] = 1;
                }
            }
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp, converged
                uint32_t v[32];
                tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(a * BN + c),
                                   v);
                tmem_ld_wait();
                const int col = n0 + c;
                if (row >= g.M || col >= g.N) continue;
                float f[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    f[j] = __uint_as_float(v[j]);
                    if (g.act == 1) f[j] = silu(f[j]);
                }
                if (col + 32 <= g.N && (reinterpret_cast<uintptr_t>(crow + col) & 15) == 0) {
                    uint4* dst = reinterpret_cast<uint4*>(crow + col);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        dst[j] = make_uint4(pack_bf16x2(f[8 * j], f[8 * j + 1]), pack_bf16x2(f[8 * j + 2], f[8 * j + 3]),
                                            pack_bf16x2(f[8 * j + 4], f[8 * j + 5]),
                                            pack_bf16x2(f[8 * j + 6], f[8 * j + 7]));
                    }
                } else {
                    for (int j = 0; j < 32 && col + j < g.N; ++j) crow[col + j] = __float2bfloat16_rn(f[j]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(2 * STAGES + 2 + a));
            if (MODE == kModeReduceScatter && lane == 0) {
                // This warp's 32 rows of the tile are stored: release them to the owner (the
                // owner waits for 4 warps x nranks bumps per call).
                const int per = g.tp.ms / BM;
                const int owner_tile = (rb % per) * num_n + (tile % num_n);
                fence_sys();
                red_add_sys(g.tp.rs_counters[owner] + owner_tile, 1ull);
            }
        }
    } else {
        comm_warps<MODE>(g, num_n, s_abort, s_comm_stop);
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// ---------------------------------------------------------------------------------------
// 2-SM variant: a CTA pair (cluster of 2) computes a 256x256 tile with tcgen05.mma.cta_group::2.
// Each CTA TMA-loads its own 128 rows of A and its own 128 rows of B (N/2) into a 6-stage ring
// and its loads complete on the leader's full barrier, where the leader alone expects both CTAs'
// bytes; the leader's single MMA thread reads both
// CTAs' shared memory, and its commits arrive on both CTAs' barriers. Each CTA's TMEM holds its
// 128 rows x 256 columns of the accumulator, so the epilogue is the same as the 1-SM kernel.
// Per FLOP this moves a third less data from L2 into shared memory than 128x256 tiles. No load
// uses cluster multicast.
//
// PBN, the tile width, is 256 or 224. Narrower tiles exist for wave quantisation: with 74 CTA
// pairs, N = 3584 (a TP=8 shard of a 28672-wide FFN) gives 14 columns of 256-wide tiles, e.g.
// 448 tiles = 6.05 waves for M = 8192, so the seventh wave is nearly empty; 224-wide tiles make
// 512 tiles = 6.9 waves. Each CTA holds PBN/2 rows of B (a multiple of the 8-row swizzle atom).
constexpr int PSTAGES = 6;
template <int PBN>
constexpr int PStageBytes() { return BM * BK * 2 + (PBN / 2) * BK * 2; }  // A rows + this CTA's half of B
template <int PBN>
constexpr int PSmemBytes() { return PSTAGES * PStageBytes<PBN>() + 1024 + 256; }
static_assert(PStageBytes<224>() % 1024 == 0 && PStageBytes<256>() % 1024 == 0, "stages must keep 1 KiB alignment");
static_assert(PSmemBytes<256>() <= 227 * 1024, "shared memory");

template <int MODE, int PBN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_bf16_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const __grid_constant__ CUtensorMap tmG, const __grid_constant__ Args g) {
    static_assert(PBN % 32 == 0 && PBN <= 256 && (PBN / 2) % 8 == 0, "tile width");
    constexpr int kPStageBytes = PStageBytes<PBN>();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + PSTAGES * kPStageBytes);
    // full[0..S) (leader's count both CTAs) empty[S..2S) acc_full[2S..2S+2) acc_empty[2S+2..2S+4) drain[2S+4]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * PSTAGES + 5);
    volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* s_comm_stop = s_abort + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t cta = cluster_ctarank();
    const bool leader = cta == 0;
    auto bar = [&](int i) { return smem_u32(bars + i); };
    auto smemA = [&](int s) { return smem_u32(smem + s * kPStageBytes); };
    auto smemB = [&](int s) { return smem_u32(smem + s * kPStageBytes + BM * BK * 2); };

    if (threadIdx.x == 0) {
        for (int s = 0; s < PSTAGES; ++s) {
            mbar_init(bar(s), 1);
            mbar_init(bar(PSTAGES + s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(bar(2 * PSTAGES + a), 1);
            mbar_init(bar(2 * PSTAGES + 2 + a), 8);
        }
        mbar_init(bar(2 * PSTAGES + 4), 1);
        *s_abort = 0;
        *s_comm_stop = 0;
        fence_proxy_async_shared();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    cluster_sync();  // both CTAs' barriers exist before any remote arrive
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int PM = 2 * BM;  // rows per pair tile
    const int num_m = (g.M + PM - 1) / PM, num_n = (g.N + PBN - 1) / PBN;
    const int tiles = num_m * num_n;
    const int kblocks = (g.K + BK - 1) / BK;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    auto tile_rb = [&](int t) {
        if (MODE == kModeAllGather) return ag_row_block(t / num_n, g.tp, num_m, PM);
        if (MODE == kModeReduceScatter) return rs_row_block(t / num_n, g.tp, PM);
        return t / num_n;
    };
    auto fail = [&]() {
        *s_abort = 1;
        atomicExch(g.err, 1);
    };

    if (warp == 0) {
        if (lane == 0) {
            uint32_t kb = 0;
            for (int tile = pair; tile < tiles && !*s_abort; tile += npairs) {
                const int rb = tile_rb(tile);
                const int n0 = (tile % num_n) * PBN + static_cast<int>(cta) * (PBN / 2);  // this CTA's half of N
                const CUtensorMap* amap = &tmA;
                int arow = rb * PM + static_cast<int>(cta) * BM;
                if (MODE == kModeAllGather) {
                    const int per = g.tp.ms / BM, rb128 = rb * 2 + static_cast<int>(cta);
                    const int src = rb128 / per, chunk = rb128 % per;
                    if (src == g.tp.rank) {
                        arow = chunk * BM;
                    } else {
                        const unsigned long long* cnt = g.tp.ag_counters + (size_t)src * kTpMaxChunks + chunk;
                        if (!wait_geq_sys(cnt, g.tp.seq * (uint64_t)g.tp.contributors, s_abort)) {
                            fail();
                            break;
                        }
                        fence_proxy_async_global();
                        amap = &tmG;
                    }
                }
                bool ok = true;
                for (int k = 0; k < kblocks; ++k, ++kb) {
                    const int s = kb % PSTAGES;
                    if (!mbar_wait(bar(PSTAGES + s), ((kb / PSTAGES) & 1) ^ 1, s_abort)) {
                        ok = false;
                        break;
                    }
                    // Only the leader arrives (locally, once for both CTAs' bytes): a remote
                    // arrive with cluster-scope release per stage costs a memory barrier that
                    // stalled the producers longer than the MMAs of a stage take.
                    const uint32_t lfull = mapa_shared(bar(s), 0);
                    if (leader) mbar_arrive_expect_tx(bar(s), 2 * kPStageBytes);
                    tma_load_2d_pair(smemA(s), amap, lfull, k * BK, arow);
                    tma_load_2d_pair(smemB(s), &tmB, lfull, k * BK, n0);
                }
                if (!ok) {
                    fail();
                    break;
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            const uint32_t idesc = idesc_bf16_f32(2 * BM, PBN);
            uint32_t kb = 0, local = 0;
            for (int tile = pair; tile < tiles && !*s_abort; tile += npairs, ++local) {
                const int a = local & 1;
                const uint32_t use = local >> 1;
                if (!mbar_wait(bar(2 * PSTAGES + 2 + a), (use & 1) ^ 1, s_abort)) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + static_cast<uint32_t>(a * PBN);
                bool ok = true;
                for (int k = 0; k < kblocks; ++k, ++kb) {
                    const int s = kb % PSTAGES;
                    if (!mbar_wait(bar(s), (kb / PSTAGES) & 1, s_abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad = smem_desc_sw128(smemA(s)), bd = smem_desc_sw128(smemB(s));
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        umma_f16_pair(d, ad + static_cast<uint64_t>(kk * 2), bd + static_cast<uint64_t>(kk * 2), idesc,
                                      (k > 0 || kk > 0) ? 1u : 0u);
                    }
                    umma_commit_pair(bar(PSTAGES + s), 0x3);
                }
                if (!ok) {
                    fail();
                    break;
                }
                umma_commit_pair(bar(2 * PSTAGES + a), 0x3);
            }
            umma_commit_pair(bar(2 * PSTAGES + 4), 0x1);
            mbar_wait(bar(2 * PSTAGES + 4), 0, s_abort, 1u << 22);
            // Every TMA load counted on this CTA's full barriers has landed (both CTAs').
            for (uint32_t i = (kb > PSTAGES ? kb - PSTAGES : 0); i < kb; ++i)
                mbar_wait(bar(i % PSTAGES), (i / PSTAGES) & 1, s_abort, 1u << 22);
        }
    } else if (warp < 6) {
        const int q = warp & 3;
        const int row_in_cta = q * 32 + lane;
        uint32_t local = 0;
        unsigned char rs_ready_checked[kMaxRanks] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int tile = pair; tile < tiles && !*s_abort; tile += npairs, ++local) {
            const int a = local & 1;
            const uint32_t use = local >> 1;
            if (!mbar_wait(bar(2 * PSTAGES + a), use & 1, s_abort)) {
                if (lane == 0) fail();
                break;
            }
            tc_fence_after();
            const int rb = tile_rb(tile);
            const int rb128 = rb * 2 + static_cast<int>(cta);
            const int n0 = (tile % num_n) * PBN;
            const int row = rb128 * BM + row_in_cta;
            __nv_bfloat16* crow = g.C + static_cast<size_t>(row) * g.ldc;
            int owner = 0;
            if (MODE == kModeReduceScatter) {  // as in the 1-SM kernel: own staging, owner pulls
                const int per = g.tp.ms / BM;
                owner = rb128 / per;
                if (owner != g.tp.rank && !rs_ready_checked[owner]) {
                    if (lane == 0 && !wait_geq_sys(g.tp.rs_started + owner, g.tp.seq - 1, s_abort)) fail();
                    __syncwarp();
                    rs_ready_checked[owner] = 1;
                }
            }
#pragma unroll 1
            for (int c = 0; c < PBN; c += 32) {
                __syncwarp();
                uint32_t v[32];
                tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(a * PBN + c),
                                   v);
                tmem_ld_wait();
                const int col = n0 + c;
                if (row >= g.M || col >= g.N) continue;
                float f[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    f[j] = __uint_as_float(v[j]);
                    if (g.act == 1) f[j] = silu(f[j]);
                }
                if (col + 32 <= g.N && (reinterpret_cast<uintptr_t>(crow + col) & 15) == 0) {
                    uint4* dst = reinterpret_cast<uint4*>(crow + col);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        dst[j] = make_uint4(pack_bf16x2(f[8 * j], f[8 * j + 1]), pack_bf16x2(f[8 * j + 2], f[8 * j + 3]),
                                            pack_bf16x2(f[8 * j + 4], f[8 * j + 5]),
                                            pack_bf16x2(f[8 * j + 6], f[8 * j + 7]));
                    }
                } else {
                    for (int j = 0; j < 32 && col + j < g.N; ++j) crow[col + j] = __float2bfloat16_rn(f[j]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(bar(2 * PSTAGES + 2 + a), 0));
            if (MODE == kModeReduceScatter && lane == 0) {
                const int per = g.tp.ms / BM;
                const int owner_tile = (rb128 % per) * num_n + (tile % num_n);
                fence_sys();
                red_add_sys(g.tp.rs_counters[owner] + owner_tile, 1ull);
            }
        }
    } else {
        comm_warps<MODE, PBN>(g, num_n, s_abort, s_comm_stop);
    }
    __syncthreads();
    cluster_sync();  // the peer's shared memory and TMEM stay valid until both CTAs are done
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, kTmemCols);
    }
}

bool MakeMap(CUtensorMap* map, const void* base, int rows, int cols, int box_rows) {
    const DriverApi* d = Driver();
    if (d == nullptr || d->cuTensorMapEncodeTiled == nullptr) return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = d->cuTensorMapEncodeTiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int MODE>
cudaError_t LaunchMode(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tg, const Args& g, int grid,
                       bool pair, int pbn, cudaStream_t stream) {
    static bool attr_set[3][64] = {};
    const int which = !pair ? 0 : (pbn == 224 ? 2 : 1);
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[which][dev]) {
        cudaError_t e = which == 0 ? cudaFuncSetAttribute(gemm_bf16_kernel<MODE>,
                                                          cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes)
                        : which == 1 ? cudaFuncSetAttribute(gemm_bf16_pair_kernel<MODE, 256>,
                                                            cudaFuncAttributeMaxDynamicSharedMemorySize, PSmemBytes<256>())
                                     : cudaFuncSetAttribute(gemm_bf16_pair_kernel<MODE, 224>,
                                                            cudaFuncAttributeMaxDynamicSharedMemorySize, PSmemBytes<224>());
        if (e != cudaSuccess) return e;
        attr_set[which][dev] = true;
    }
    if (which == 1) {
        gemm_bf16_pair_kernel<MODE, 256><<<grid & ~1, kThreads, PSmemBytes<256>(), stream>>>(ta, tb, tg, g);
    } else if (which == 2) {
        gemm_bf16_pair_kernel<MODE, 224><<<grid & ~1, kThreads, PSmemBytes<224>(), stream>>>(ta, tb, tg, g);
    } else {
        gemm_bf16_kernel<MODE><<<grid, kThreads, kSmemBytes, stream>>>(ta, tb, tg, g);
    }
    return cudaGetLastError();
}

// Tile width of the 2-SM kernel: BCCL_GEMM_BN=256 or 224 forces one; "auto" picks the one with
// the smaller ceil(tiles / pairs) * width (waves times the work of a tile; ties keep 256).
// The default is 256 until the 224-wide kernel has been measured on a B200.
int ChoosePairBN(int M, int N, int pairs) {
    const char* v = std::getenv("BCCL_GEMM_BN");
    if (v != nullptr && std::strcmp(v, "224") == 0) return 224;
    if (v == nullptr || std::strcmp(v, "auto") != 0) return 256;
    const long rows = (M + 2 * BM - 1) / (2 * BM);
    long best_cost = -1;
    int best = 256;
    for (int bn : {256, 224}) {
        const long tiles = rows * ((N + bn - 1) / bn);
        const long cost = (tiles + pairs - 1) / pairs * bn;
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best = bn;
        }
    }
    return best;
}

// BCCL_GEMM_PAIR=1 forces the 2-SM kernel, =0 the 1-SM kernel; otherwise kPairDefault decides.
constexpr bool kPairDefault = true;
bool UsePair() {
    const char* v = std::getenv("BCCL_GEMM_PAIR");
    if (v != nullptr && (v[0] == '0' || v[0] == '1')) return v[0] == '1';
    return kPairDefault;
}

int NumSms() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

}  // namespace
}  // namespace gemm

bool GemmUsesPair() { return gemm::UsePair(); }

int GemmTileWidth(int M, int N) { return gemm::UsePair() ? gemm::ChoosePairBN(M, N, gemm::NumSms() / 2) : gemm::BN; }

cudaError_t LaunchGemmBf16(const void* A, const void* B, void* C, int M, int N, int K, int ldc, int act, int* err,
                           int max_ctas, cudaStream_t stream) {
    using namespace gemm;
    if (M <= 0 || N <= 0 || K <= 0 || (K % 8) != 0 || (reinterpret_cast<uintptr_t>(A) & 15) ||
        (reinterpret_cast<uintptr_t>(B) & 15) || err == nullptr) {
        return cudaErrorInvalidValue;
    }
    CUtensorMap ta, tb;
    const bool pair = UsePair();
    const int pbn = pair ? ChoosePairBN(M, N, (max_ctas > 0 ? std::min(max_ctas, NumSms()) : NumSms()) / 2) : BN;
    if (!MakeMap(&ta, A, M, K, BM) || !MakeMap(&tb, B, N, K, pair ? pbn / 2 : BN)) return cudaErrorInvalidValue;
    const int tiles = ((M + (pair ? 2 * BM : BM) - 1) / (pair ? 2 * BM : BM)) * ((N + pbn - 1) / pbn);
    int grid = std::min(pair ? 2 * tiles : tiles, NumSms());
    if (max_ctas > 0 && grid > max_ctas) grid = max_ctas;
    if (pair && grid < 2) grid = 2;
    Args g{static_cast<__nv_bfloat16*>(C), M, N, K, ldc, act, err, TpArgs{}};
    return LaunchMode<kModePlain>(ta, tb, tb, g, grid, pair, pbn, stream);
}

cudaError_t LaunchTpGemm(int mode, const void* A_local, const void* A_gathered, const void* B, void* C, int M, int N,
                         int K, int act, int* err, const TpArgs& tp, cudaStream_t stream) {
    using namespace gemm;
    if (M <= 0 || N <= 0 || K <= 0 || (K % 8) != 0 || (N % 8) != 0 || tp.ms % BM != 0 || tp.ms / BM > kTpMaxChunks ||
        tp.nranks < 1 || tp.nranks > kMaxRanks || err == nullptr || M != tp.ms * tp.nranks) {
        return cudaErrorInvalidValue;
    }
    CUtensorMap ta, tb, tg;
    const bool pair = UsePair() && tp.ms % (2 * BM) == 0;
    const int grid = NumSms() & ~1;
    TpArgs t = tp;
    t.contributors = grid;
    // BCCL_TP_PUSH_WARPS (1-4): communication warps that push the activation shard (default 4).
    const char* pw = std::getenv("BCCL_TP_PUSH_WARPS");
    t.push_threads = 32 * std::max(1, std::min(4, pw != nullptr ? std::atoi(pw) : 4));
    Args g{static_cast<__nv_bfloat16*>(C), M, N, K, N, act, err, t};
    if (mode == kModeAllGather) {
        const int pbn = pair ? ChoosePairBN(M, N, grid / 2) : BN;
        if (!MakeMap(&ta, A_local, tp.ms, K, BM) || !MakeMap(&tb, B, N, K, pair ? pbn / 2 : BN) ||
            !MakeMap(&tg, A_gathered, M, K, BM)) {
            return cudaErrorInvalidValue;
        }
        return LaunchMode<kModeAllGather>(ta, tb, tg, g, grid, pair, pbn, stream);
    }
    if (mode == kModeReduceScatter) {
        // 256-wide tiles only: the owners' tile counters are laid out for them.
        if (!MakeMap(&ta, A_local, M, K, BM) || !MakeMap(&tb, B, N, K, pair ? BM : BN)) return cudaErrorInvalidValue;
        return LaunchMode<kModeReduceScatter>(ta, tb, ta, g, grid, pair, 256, stream);
    }
    return cudaErrorInvalidValue;
}

}  // namespace bccl
