// Host launchers of the sm_100a GEMM kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "device/cuda_driver.h"

#include "device/dev_types.h"

namespace bccl {

enum GemmMode : int { kModePlain = 0, kModeAllGather = 1, kModeReduceScatter = 2 };
constexpr int kTpMaxChunks = 64;  // row blocks (128 rows) per rank shard

// Peer-memory plumbing of the fused tensor-parallel GEMMs (one row per rank).
struct TpArgs {
    int rank, nranks;
    int ms;                                   // rows per rank (multiple of 128)
    unsigned long long seq;                   // call index, 1-based, same on every rank
    int contributors;                         // CTAs per rank that bump each counter (set by the launcher)
    int push_threads;                         // AllGather: threads per CTA that push (set by the launcher)
    // AllGather -> GEMM
    const void* x_local;                      // this rank's shard [ms, K]
    void* xg[kMaxRanks];                      // every rank's gathered-X buffer (this call's half)
    void* xg_mc;                              // its NVLS multicast address (null: one store per peer)
    const unsigned long long* ag_counters;    // here: [src][kTpMaxChunks]
    unsigned long long* ag_counters_peer[kMaxRanks];  // the same array on every rank
    // GEMM -> ReduceScatter
    __nv_bfloat16* rs_stage[kMaxRanks];       // every rank's partial product [M][N] (this call's half)
    unsigned long long* rs_counters[kMaxRanks];       // every rank's per-own-tile counters
    const unsigned long long* rs_started;     // here: [src] = last call index src started
    unsigned long long* rs_started_peer[kMaxRanks];
    __nv_bfloat16* out;                       // this rank's reduced rows [ms, N]
};

// C[M,N] (row-major, leading dimension ldc) = act(A[M,K] * B[N,K]^T); A, B row-major bf16,
// f32 accumulation in TMEM, bf16 output. act: 0 none, 1 SiLU. *err (device memory) becomes
// non-zero if a bounded wait inside the kernel gave up. K must be a multiple of 8 (TMA row
// pitch) and A/B 16-byte aligned; M, N and K need not be multiples of the tile sizes.
// True when the GEMMs run on 2-SM (cta_group::2) 256x256 tiles instead of 1-SM 128x256 tiles.
bool GemmUsesPair();
// Tile width (columns of C per tile) the GEMMs use for an M x N product: 256, or 224 for 2-SM
// tiles when BCCL_GEMM_BN=224 (or =auto and narrower tiles fill the last wave better).
int GemmTileWidth(int M, int N);

cudaError_t LaunchGemmBf16(const void* A, const void* B, void* C, int M, int N, int K, int ldc, int act, int* err,
                           int max_ctas, cudaStream_t stream);

// Fused tensor-parallel GEMMs (one persistent kernel each, one CTA per SM):
//   kModeAllGather:     C[M,N] = act(AllGather(A_local)[M,K] * B[N,K]^T), M = nranks*ms; the kernel
//                       pushes A_local into every peer's A_gathered while it multiplies.
//   kModeReduceScatter: tp.out[ms,N] = rows [rank*ms, (rank+1)*ms) of sum_ranks(A[M,K] * B[N,K]^T);
//                       partial tiles go to their owner's staging as they are produced.
cudaError_t LaunchTpGemm(int mode, const void* A_local, const void* A_gathered, const void* B, void* C, int M, int N,
                         int K, int act, int* err, const TpArgs& tp, cudaStream_t stream);

}  // namespace bccl
