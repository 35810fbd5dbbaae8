// Line epochs of the low-latency kernel (ll.cu), shared with the CPU checks of the protocol
// (bcclLLEpoch in the C API).
//
// A launch's lines carry the launch's epoch and go to the line buffers of parity epoch & 1. The
// epoch of the launch that follows `seq` earlier low-latency launches of a communicator is
// 1, 2, ..., 2^32 - 2, then 1 again: never 0 (the value of a line that was never written, the
// buffers being zeroed at Init), and always the other parity than the previous launch's, also
// across the wrap (2^32 - 2 is even, 1 is odd). Equal epochs are 2^32 - 2 launches apart.
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define BCCL_LL_HD __host__ __device__
#else
#define BCCL_LL_HD
#endif

namespace bccl {

constexpr unsigned long long kLLEpochPeriod = 4294967294ull;  // 2^32 - 2

BCCL_LL_HD inline uint32_t LLEpoch(unsigned long long seq) {
    return static_cast<uint32_t>(seq % kLLEpochPeriod) + 1u;
}

}  // namespace bccl
