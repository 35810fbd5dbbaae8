// Two-shot AllReduce over peer memory (used when NVLS is unavailable or does not support
// the dtype/op, e.g. f32 MAX).
//
// Per round (a chunk of N shards):
//   1. push   : shard p of the chunk -> peer p's inbox slot [rank]        (NVLink egress S(N-1)/N)
//   2. barrier
//   3. reduce : own shard = input shard + N-1 inbox slots -> local result area
//   4. barrier
//   5. pull   : shard p <- peer p's result area (remote loads); own shard <- local result
// This is the reference's ring ReduceScatter + AllGather (OriginCCL
// src/topology/topology_ring.cpp:255-290) collapsed to one hop each, since every GPU
// reaches every other through the switch at full bandwidth.
#include "kernels/common.cuh"
#include "kernels/launch.h"

namespace bccl {
namespace dev {
namespace {

struct TwoShotParams {
    DevComm comm;
    const void* src;
    void* dst;
    unsigned long long bytes;
    unsigned long long shard_cap;  // bytes of one shard slot (multiple of 16)
    int nrounds;
    int dtype;
    int op;
    float scale;
};

// Data region layout: inbox [2][N][shard_cap], then result [2][shard_cap].
__device__ __forceinline__ char* ts_inbox(const DevComm& c, int owner, int half, int src, size_t cap) {
    return c.uc[owner] + kCtrlBytes + ((size_t)half * c.nranks + src) * cap;
}
__device__ __forceinline__ char* ts_result(const DevComm& c, int owner, int half, size_t cap) {
    return c.uc[owner] + kCtrlBytes + (size_t)2 * c.nranks * cap + (size_t)half * cap;
}

__global__ void __launch_bounds__(512, 1) twoshot_kernel(const __grid_constant__ TwoShotParams p) {
    const DevComm& c = p.comm;
    const int r = c.rank, n = c.nranks;
    const uint64_t round0 = load_state_u64(&c.state->round_seq);
    uint64_t bar = load_state_u64(&c.state->barrier_seq);
    const size_t cap = p.shard_cap;
    const size_t chunk = cap * n;
    for (int j = 0; j < p.nrounds; ++j) {
        const int half = (int)((round0 + (uint64_t)j) & 1ull);
        const size_t cbeg = (size_t)j * chunk;
        const size_t clen = min((size_t)p.bytes - cbeg, chunk);
        const size_t shard = round_up((clen + n - 1) / n, 16);
        const size_t piece = round_up((shard + gridDim.x - 1) / gridDim.x, 16);
        const size_t s0 = min(shard, (size_t)blockIdx.x * piece);
        const size_t s1 = min(shard, s0 + piece);
        const char* src = static_cast<const char*>(p.src) + cbeg;
        char* dst = static_cast<char*>(p.dst) + cbeg;
        // [lo, hi) of shard q restricted to this CTA's piece and the chunk.
        auto range = [&](int q, size_t* lo, size_t* hi) {
            size_t base = (size_t)q * shard;
            *lo = min(clen, base + s0);
            *hi = min(clen, base + s1);
        };
        size_t lo, hi;
        for (int q = 0; q < n; ++q) {
            if (q == r) continue;
            range(q, &lo, &hi);
            if (lo < hi) cta_copy(ts_inbox(c, q, half, r, cap) + s0, src + lo, hi - lo, false);
        }
        if (!cta_barrier(c, ++bar, 2 * j)) break;
        range(r, &lo, &hi);
        if (lo < hi) {
            const void* srcs[kMaxRanks];
            unsigned cg = 0;
            for (int q = 0; q < n; ++q) {
                if (q == r) {
                    srcs[q] = src + lo;
                } else {
                    srcs[q] = ts_inbox(c, r, half, q, cap) + s0;
                    cg |= 1u << q;
                }
            }
            cta_reduce_any(p.dtype, ts_result(c, r, half, cap) + s0, srcs, n, cg, hi - lo, p.op, n, p.scale);
        }
        if (!cta_barrier(c, ++bar, 2 * j + 1)) break;
        for (int q = 0; q < n; ++q) {
            range(q, &lo, &hi);
            if (lo < hi) cta_copy(dst + lo, ts_result(c, q, half, cap) + s0, hi - lo, true);
        }
    }
    finish_launch(c, (uint64_t)p.nrounds, 2ull * (uint64_t)p.nrounds, 0);
}

}  // namespace
}  // namespace dev

cudaError_t LaunchTwoShot(const DevComm& c, const void* src, void* dst, unsigned long long count, int dtype, int op,
                          float scale, unsigned long long shard_cap, int nctas, cudaStream_t stream) {
    if (nctas <= 0 || nctas > kMaxCtas || shard_cap == 0 || (shard_cap & 15) != 0) return cudaErrorInvalidValue;
    dev::TwoShotParams p;
    p.comm = c;
    p.src = src;
    p.dst = dst;
    p.bytes = count * (unsigned long long)dev::dtype_size(dtype);
    p.shard_cap = shard_cap;
    const unsigned long long chunk = shard_cap * (unsigned long long)c.nranks;
    p.nrounds = (int)((p.bytes + chunk - 1) / chunk);
    if (p.nrounds == 0) p.nrounds = 1;
    p.dtype = dtype;
    p.op = op;
    p.scale = scale;
    dev::twoshot_kernel<<<nctas, 512, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace bccl
