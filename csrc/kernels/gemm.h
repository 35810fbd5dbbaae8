// Host launchers of the sm_100a GEMM kernels.
#pragma once

#include <cuda_runtime.h>

#include "device/cuda_driver.h"

namespace bccl {

// C[M,N] (row-major, leading dimension ldc) = act(A[M,K] * B[N,K]^T); A, B row-major bf16,
// f32 accumulation in TMEM, bf16 output. act: 0 none, 1 SiLU. *err (device memory) becomes
// non-zero if a bounded wait inside the kernel gave up. K must be a multiple of 8 (TMA row
// pitch) and A/B 16-byte aligned; M, N and K need not be multiples of the tile sizes.
cudaError_t LaunchGemmBf16(const void* A, const void* B, void* C, int M, int N, int K, int ldc, int act, int* err,
                           int max_ctas, cudaStream_t stream);

}  // namespace bccl
