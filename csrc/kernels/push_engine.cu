// Push engine: one kernel for every small/medium collective and for whole groups.
//
// The reference runs each collective as a CPU state machine over per-edge transports
// (OriginCCL src/topology/topology_ring.cpp:330-623, topology_tree.cpp:135-306) and its
// dynamic executor spreads a group's slices over channels with an in-band control
// broadcast (src/executor/dynamic_multi_thread_executor.cpp:176-230). On one NVSwitch
// node every GPU is one hop from every other, so here each rank stores its per-peer
// payload straight into the peer's inbox over NVLink, crosses one flag barrier per round
// and then consumes its inbox locally:
//   AllReduce / Reduce : push the input to every peer (to the root), reduce N slots
//   ReduceScatter      : push shard p to peer p, reduce N slots of the own shard
//   AllGather          : push the input to every peer, copy slots into the output
//   Broadcast          : the root pushes, the others copy their slot out
// A launch carries a list of WorkItems laid end to end in a per-peer byte stream; rounds
// cut the stream into inbox-sized pieces and CTA b always owns piece b of a round on
// every rank, so one per-CTA barrier per round is the only synchronisation (no grid-wide
// barrier, no host round trip). Inboxes are double-buffered by round parity; a rank only
// rewrites half h after the barrier of the following round has proven that every peer
// finished reading it.
#include "kernels/common.cuh"
#include "kernels/launch.h"

namespace bccl {
namespace dev {
namespace {

template <int MAXI>
struct PushParams {
    DevComm comm;
    int nitems;
    int nrounds;
    unsigned long long stream_bytes;
    unsigned long long slot_bytes;  // per-source inbox capacity of one half
    WorkItem items[MAXI];
};

__device__ __forceinline__ size_t payload_bytes(const WorkItem& it) {
    return (size_t)it.count * dtype_size(it.dtype);
}

__device__ __forceinline__ char* inbox(const DevComm& c, int owner, int half, int src, size_t slot) {
    return c.uc[owner] + kCtrlBytes + ((size_t)half * c.nranks + src) * slot;
}

// Loads once, stores to every destination in dsts[0..n).
__device__ __forceinline__ void cta_push_multi(char* const* dsts, int n, const char* src, size_t bytes) {
    const size_t t = threadIdx.x, nt = blockDim.x;
    uintptr_t mis = reinterpret_cast<uintptr_t>(src);
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p)
        if (p < n) mis |= reinterpret_cast<uintptr_t>(dsts[p]);
    const size_t nv = ((mis & 15) == 0) ? (bytes >> 4) : 0;
    size_t i = t;
    for (; i + 3 * nt < nv; i += 4 * nt) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = *reinterpret_cast<const uint4*>(src + ((i + u * nt) << 4));
#pragma unroll
        for (int p = 0; p < kMaxRanks; ++p) {
            if (p < n) {
#pragma unroll
                for (int u = 0; u < 4; ++u) st_cg(dsts[p] + ((i + u * nt) << 4), v[u]);
            }
        }
    }
    for (; i < nv; i += nt) {
        uint4 v = *reinterpret_cast<const uint4*>(src + (i << 4));
#pragma unroll
        for (int p = 0; p < kMaxRanks; ++p)
            if (p < n) st_cg(dsts[p] + (i << 4), v);
    }
    for (size_t j = (nv << 4) + t; j < bytes; j += nt) {
        char b = src[j];
#pragma unroll
        for (int p = 0; p < kMaxRanks; ++p)
            if (p < n) dsts[p][j] = b;
    }
}

// Phase 1 of a round: send this CTA's piece [ia, ib) of item `it` (inbox offset q).
__device__ void produce(const DevComm& c, const WorkItem& it, size_t ia, size_t ib, size_t q, int half,
                        size_t slot) {
    const int r = c.rank, n = c.nranks;
    const size_t len = ib - ia;
    const size_t es = dtype_size(it.dtype);
    const char* src = static_cast<const char*>(it.src);
    char* dsts[kMaxRanks];
    int nd = 0;
    switch (it.func) {
    case 0:  // AllReduce
    case 3:  // AllGather
        for (int p = 0; p < n; ++p)
            if (p != r) dsts[nd++] = inbox(c, p, half, r, slot) + q;
        if (nd > 0) cta_push_multi(dsts, nd, src + ia, len);
        break;
    case 1:  // Broadcast
        if (r == it.root) {
            for (int p = 0; p < n; ++p)
                if (p != r) dsts[nd++] = inbox(c, p, half, r, slot) + q;
            cta_push_multi(dsts, nd, src + ia, len);
        }
        break;
    case 2:  // Reduce
        if (r != it.root) {
            dsts[0] = inbox(c, it.root, half, r, slot) + q;
            cta_push_multi(dsts, 1, src + ia, len);
        }
        break;
    case 4:  // ReduceScatter: shard p goes to peer p
        for (int p = 0; p < n; ++p) {
            if (p == r) continue;
            dsts[0] = inbox(c, p, half, r, slot) + q;
            cta_push_multi(dsts, 1, src + (size_t)p * it.count * es + ia, len);
        }
        break;
    default: break;
    }
}

// Phase 2 of a round: consume the piece from the local inbox.
__device__ void consume(const DevComm& c, const WorkItem& it, size_t ia, size_t ib, size_t q, int half, size_t slot) {
    const int r = c.rank, n = c.nranks;
    const size_t len = ib - ia;
    const size_t es = dtype_size(it.dtype);
    const char* src = static_cast<const char*>(it.src);
    char* dst = static_cast<char*>(it.dst);
    const void* srcs[kMaxRanks];
    unsigned cg = 0;
    switch (it.func) {
    case 0:  // AllReduce
    case 2:  // Reduce
        if (it.func == 2 && r != it.root) break;
        for (int p = 0; p < n; ++p) {
            if (p == r) {
                srcs[p] = src + ia;
            } else {
                srcs[p] = inbox(c, r, half, p, slot) + q;
                cg |= 1u << p;
            }
        }
        cta_reduce_any(it.dtype, dst + ia, srcs, n, cg, len, it.op, n, it.scale);
        break;
    case 4:  // ReduceScatter
        for (int p = 0; p < n; ++p) {
            if (p == r) {
                srcs[p] = src + (size_t)r * it.count * es + ia;
            } else {
                srcs[p] = inbox(c, r, half, p, slot) + q;
                cg |= 1u << p;
            }
        }
        cta_reduce_any(it.dtype, dst + ia, srcs, n, cg, len, it.op, n, it.scale);
        break;
    case 3:  // AllGather
        for (int p = 0; p < n; ++p) {
            char* out = dst + (size_t)p * it.count * es + ia;
            if (p == r) {
                if (out != src + ia) cta_copy(out, src + ia, len, false);
            } else {
                cta_copy(out, inbox(c, r, half, p, slot) + q, len, true);
            }
        }
        break;
    case 1:  // Broadcast
        if (r == it.root) {
            if (dst != src) cta_copy(dst + ia, src + ia, len, false);
        } else {
            cta_copy(dst + ia, inbox(c, r, half, it.root, slot) + q, len, true);
        }
        break;
    default: break;
    }
}

template <int MAXI>
__global__ void __launch_bounds__(512, 1) push_engine_kernel(const __grid_constant__ PushParams<MAXI> p) {
    const DevComm& c = p.comm;
    const uint64_t round0 = load_state_u64(&c.state->round_seq);
    const uint64_t bar0 = load_state_u64(&c.state->barrier_seq);
    const size_t slot = p.slot_bytes;
    if (threadIdx.x == 0) trace(c, 0, kTrBegin, 0);
    bool ok = true;
    int first = 0;  // first item that can still overlap this CTA's pieces (items are sorted)
    for (int j = 0; j < p.nrounds && ok; ++j) {
        const int half = (int)((round0 + (uint64_t)j) & 1ull);
        const size_t rbeg = (size_t)j * slot;
        const size_t rend = min((size_t)p.stream_bytes, rbeg + slot);
        const size_t piece = round_up((rend - rbeg + gridDim.x - 1) / gridDim.x, 16);
        const size_t a = min(rend, rbeg + (size_t)blockIdx.x * piece);
        const size_t b = min(rend, a + piece);
        while (first < p.nitems && p.items[first].stream_off + payload_bytes(p.items[first]) <= a) ++first;
        for (int i = first; i < p.nitems && a < b; ++i) {
            const WorkItem& it = p.items[i];
            const size_t s0 = it.stream_off, s1 = s0 + payload_bytes(it);
            if (s0 >= b) break;
            const size_t lo = max(a, s0), hi = min(b, s1);
            if (lo < hi) produce(c, it, lo - s0, hi - s0, lo - rbeg, half, slot);
        }
        ok = cta_barrier(c, bar0 + (uint64_t)j + 1, j);
        if (!ok) break;
        if (threadIdx.x == 0) trace(c, 0, kTrBarrier, j);
        for (int i = first; i < p.nitems && a < b; ++i) {
            const WorkItem& it = p.items[i];
            const size_t s0 = it.stream_off, s1 = s0 + payload_bytes(it);
            if (s0 >= b) break;
            const size_t lo = max(a, s0), hi = min(b, s1);
            if (lo < hi) consume(c, it, lo - s0, hi - s0, lo - rbeg, half, slot);
        }
    }
    if (threadIdx.x == 0) trace(c, 0, kTrEnd, p.nrounds);
    finish_launch(c, (uint64_t)p.nrounds, (uint64_t)p.nrounds, 0);
}

template <int MAXI>
cudaError_t Launch(const DevComm& c, const WorkItem* items, int nitems, unsigned long long stream_bytes,
                   unsigned long long slot_bytes, int nctas, cudaStream_t s) {
    PushParams<MAXI> p;
    p.comm = c;
    p.nitems = nitems;
    p.stream_bytes = stream_bytes;
    p.slot_bytes = slot_bytes;
    p.nrounds = (int)((stream_bytes + slot_bytes - 1) / slot_bytes);
    if (p.nrounds == 0) p.nrounds = 1;
    for (int i = 0; i < nitems; ++i) p.items[i] = items[i];
    push_engine_kernel<MAXI><<<nctas, 512, 0, s>>>(p);
    return cudaGetLastError();
}

}  // namespace
}  // namespace dev

cudaError_t LaunchPushEngine(const DevComm& c, const WorkItem* items, int nitems, unsigned long long stream_bytes,
                             unsigned long long slot_bytes, int nctas, cudaStream_t stream) {
    if (nitems <= 0 || nctas <= 0 || nctas > kMaxCtas || slot_bytes == 0 || (slot_bytes & 15) != 0) {
        return cudaErrorInvalidValue;
    }
    if (nitems <= 4) return dev::Launch<4>(c, items, nitems, stream_bytes, slot_bytes, nctas, stream);
    if (nitems <= kPushMaxItems) {
        return dev::Launch<kPushMaxItems>(c, items, nitems, stream_bytes, slot_bytes, nctas, stream);
    }
    return cudaErrorInvalidValue;
}

}  // namespace bccl
