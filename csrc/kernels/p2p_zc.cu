// Zero-copy collectives over NVLink peer memory, for user buffers that every rank can address:
// buffers registered with Communicator::RegisterBuffer (CUDA IPC mappings of ordinary
// cudaMalloc memory, e.g. PyTorch tensors) and symmetric allocations. No staging buffer, no
// pipeline rounds, no multicast: each rank reads its share straight from the peers' inputs and
// writes results straight into the peers' outputs.
//
//   AllReduce (two-shot):  rank r owns shard r of the payload; it loads that shard from all N
//                          inputs (N-1 of them over NVLink), reduces in the accumulation type,
//                          applies AVG / scale, and stores the result into all N outputs.
//   ReduceScatter:         rank r loads block r from all N inputs, reduces, stores locally.
//   AllGather:             rank r loads its own input and stores it into block r of all N
//                          outputs.
// Each rank moves 2(N-1)/N of the payload in each NVLink direction for AllReduce, the two-shot
// optimum, in one kernel. CTA b of every rank works on chunk b of every shard, so the per-CTA
// cross-rank barrier (same CTA index on every rank) is the only synchronisation: the entry
// barrier proves that every peer's kernel has started (its inputs are written and its outputs
// are free, by stream order), the exit barrier, after the stores, that chunk b of this rank's
// output is complete and that no peer still reads chunk b of this rank's input.
//
// The reference moves the same data through CPU ring steps over per-edge transports
// (OriginCCL src/topology/topology_ring.cpp:231-290); its zero-copy RDMA transport registers
// user buffers in an MR cache (src/transport/transport_rdma_zc.cpp:198-212), which is what the
// registration here corresponds to.
#include "kernels/common.cuh"
#include "kernels/launch.h"

namespace bccl {
namespace dev {
namespace {

struct P2pZcParams {
    DevComm comm;
    const char* in[kMaxRanks];  // every rank's input as mapped here (AllGather: only in[rank] used)
    char* out[kMaxRanks];       // every rank's output as mapped here (ReduceScatter: only out[rank])
    unsigned long long bytes;   // AllReduce: payload; AllGather / ReduceScatter: per-rank block
    int func;                   // 0 AllReduce, 3 AllGather, 4 ReduceScatter (CollFunc values)
    int op;
    float scale;
};

static_assert(sizeof(P2pZcParams) <= 32764, "kernel parameter limit");

// Loads vectors [v0, v1) (16 bytes each, at byte offset src_off) from n sources, reduces them
// and stores the result at dst_off into nd destinations. NS bounds n; U vectors per thread are
// in flight (U * n loads): with every SM's 512 threads loading, that is megabytes in flight,
// well above NVLink's bandwidth-latency product, while staying within 128 registers.
template <int D, int O, int NS>
__device__ __forceinline__ void reduce_fanout(const char* const* src, int n, size_t src_off, char* const* dst, int nd,
                                              size_t dst_off, size_t v0, size_t v1, int nranks, float scale) {
    using V = Vec<D>;
    using Acc = typename Ty<D>::Acc;
    constexpr int E = V::E;
    constexpr int U = NS <= 4 ? 2 : 1;
    const bool post = (O == kAvg) || scale != 1.0f;
    const char* sp[NS];
    char* dp[NS];
#pragma unroll
    for (int p = 0; p < NS; ++p) {
        sp[p] = src[p < n ? p : 0] + src_off;
        dp[p] = dst[p < nd ? p : 0] + dst_off;
    }
    const size_t nt = blockDim.x;
    size_t i = v0 + threadIdx.x;
    for (; i + (U - 1) * nt < v1; i += U * nt) {
        uint4 w[U][NS];
#pragma unroll
        for (int u = 0; u < U; ++u) {
#pragma unroll
            for (int p = 0; p < NS; ++p) {
                if (p < n) w[u][p] = ld_cg(sp[p] + ((i + u * nt) << 4));
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            Acc acc[E], x[E];
            V::unpack(w[u][0], acc);
#pragma unroll
            for (int p = 1; p < NS; ++p) {
                if (p < n) {
                    V::unpack(w[u][p], x);
#pragma unroll
                    for (int e = 0; e < E; ++e) acc[e] = combine<Acc>(O, acc[e], x[e]);
                }
            }
            if (post) {
#pragma unroll
                for (int e = 0; e < E; ++e) acc[e] = epilogue<Acc>(O, acc[e], nranks, scale);
            }
            const uint4 r = V::pack(acc);
#pragma unroll
            for (int p = 0; p < NS; ++p) {
                if (p < nd) st_cg(dp[p] + ((i + u * nt) << 4), r);
            }
        }
    }
    for (; i < v1; i += nt) {
        Acc acc[E], x[E];
        V::unpack(ld_cg(sp[0] + (i << 4)), acc);
#pragma unroll
        for (int p = 1; p < NS; ++p) {
            if (p < n) {
                V::unpack(ld_cg(sp[p] + (i << 4)), x);
#pragma unroll
                for (int e = 0; e < E; ++e) acc[e] = combine<Acc>(O, acc[e], x[e]);
            }
        }
        if (post) {
#pragma unroll
            for (int e = 0; e < E; ++e) acc[e] = epilogue<Acc>(O, acc[e], nranks, scale);
        }
        const uint4 r = V::pack(acc);
#pragma unroll
        for (int p = 0; p < NS; ++p) {
            if (p < nd) st_cg(dp[p] + (i << 4), r);
        }
    }
}

// Copies vectors [v0, v1) of src into nd destinations (AllGather).
template <int NS>
__device__ __forceinline__ void copy_fanout(const char* src, char* const* dst, int nd, size_t dst_off, size_t v0,
                                            size_t v1) {
    constexpr int U = 4;
    char* dp[NS];
#pragma unroll
    for (int p = 0; p < NS; ++p) dp[p] = dst[p < nd ? p : 0] + dst_off;
    const size_t nt = blockDim.x;
    size_t i = v0 + threadIdx.x;
    for (; i + (U - 1) * nt < v1; i += U * nt) {
        uint4 w[U];
#pragma unroll
        for (int u = 0; u < U; ++u) w[u] = *reinterpret_cast<const uint4*>(src + ((i + u * nt) << 4));
#pragma unroll
        for (int u = 0; u < U; ++u) {
#pragma unroll
            for (int p = 0; p < NS; ++p) {
                if (p < nd) st_cg(dp[p] + ((i + u * nt) << 4), w[u]);
            }
        }
    }
    for (; i < v1; i += nt) {
        const uint4 w = *reinterpret_cast<const uint4*>(src + (i << 4));
#pragma unroll
        for (int p = 0; p < NS; ++p) {
            if (p < nd) st_cg(dp[p] + (i << 4), w);
        }
    }
}

template <int D, int O, int NS>
__global__ void __launch_bounds__(512, 1) p2p_zc_kernel(const __grid_constant__ P2pZcParams p) {
    const DevComm& c = p.comm;
    const int r = c.rank, n = c.nranks;
    const uint64_t bar = load_state_u64(&c.state->barrier_seq);
    if (threadIdx.x == 0) trace(c, 0, kTrBegin, (int)(bar & 0x7fffffffull));
    bool ok = cta_barrier(c, bar + 1, 0);
    if (ok) {
        const size_t nvec = p.bytes / 16;
        // The span this rank works on: its shard (AllReduce) or its whole block.
        const size_t per_rank = p.func == 0 ? (nvec + n - 1) / n : nvec;
        const size_t s0 = p.func == 0 ? min(nvec, (size_t)r * per_rank) : 0;
        const size_t s1 = min(nvec, s0 + per_rank);
        const size_t per_cta = (s1 - s0 + gridDim.x - 1) / gridDim.x;
        const size_t v0 = min(s1, s0 + (size_t)blockIdx.x * per_cta), v1 = min(s1, v0 + per_cta);
        if (p.func == 3) {  // AllGather: own input into block r of every output
            copy_fanout<NS>(p.in[r], p.out, n, (size_t)r * p.bytes, v0, v1);
        } else if (p.func == 4) {  // ReduceScatter: block r of every input into the own output
            reduce_fanout<D, O, NS>(p.in, n, (size_t)r * p.bytes, p.out + r, 1, 0, v0, v1, n, p.scale);
        } else {  // AllReduce: shard r of every input into shard r of every output
            reduce_fanout<D, O, NS>(p.in, n, 0, p.out, n, 0, v0, v1, n, p.scale);
        }
        ok = cta_barrier(c, bar + 2, 1);
    }
    if (threadIdx.x == 0) trace(c, 0, kTrEnd, 0);
    finish_launch(c, 0, 2, 0);
}

template <int D, int O>
cudaError_t launch(const P2pZcParams& p, int nctas, cudaStream_t s) {
    if (p.comm.nranks <= 4) {
        p2p_zc_kernel<D, O, 4><<<nctas, 512, 0, s>>>(p);
    } else {
        p2p_zc_kernel<D, O, kMaxRanks><<<nctas, 512, 0, s>>>(p);
    }
    return cudaGetLastError();
}

}  // namespace
}  // namespace dev

cudaError_t LaunchP2pZeroCopy(const DevComm& c, int func, const char* const* in, char* const* out,
                              unsigned long long count, int dtype, int op, float scale, int nctas, cudaStream_t stream) {
    using namespace dev;
    const unsigned long long bytes = count * (unsigned long long)dtype_size(dtype);
    if (nctas <= 0 || nctas > kMaxCtas || (bytes % 16) != 0 || c.nranks < 2 || c.nranks > kMaxRanks ||
        (func != 0 && func != 3 && func != 4)) {
        return cudaErrorInvalidValue;
    }
    P2pZcParams p;
    p.comm = c;
    uintptr_t mis = 0;
    for (int q = 0; q < kMaxRanks; ++q) {
        p.in[q] = q < c.nranks ? in[q] : nullptr;
        p.out[q] = q < c.nranks ? out[q] : nullptr;
        if (q < c.nranks) mis |= reinterpret_cast<uintptr_t>(p.in[q]) | reinterpret_cast<uintptr_t>(p.out[q]);
    }
    if ((mis & 15) != 0) return cudaErrorInvalidValue;
    p.bytes = bytes;
    p.func = func;
    p.op = op;
    p.scale = scale;
    if (func == 3) return launch<kF32, kSum>(p, nctas, stream);  // data movement only
#define P2P_CASE(D)                                                   \
    if (dtype == D) {                                                 \
        switch (op) {                                                 \
        case kSum: return launch<D, kSum>(p, nctas, stream);          \
        case kMax: return launch<D, kMax>(p, nctas, stream);          \
        case kMin: return launch<D, kMin>(p, nctas, stream);          \
        case kAvg: return launch<D, kAvg>(p, nctas, stream);          \
        default: return cudaErrorInvalidValue;                        \
        }                                                             \
    }
    P2P_CASE(kF32)
    P2P_CASE(kF64)
    P2P_CASE(kI32)
    P2P_CASE(kI64)
    P2P_CASE(kBF16)
    P2P_CASE(kF16)
#undef P2P_CASE
    return cudaErrorInvalidValue;
}

}  // namespace bccl
