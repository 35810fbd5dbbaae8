// Device side of the push engine, shared by the kernel that takes its work list in launch
// parameters (push_engine.cu) and by variants that read it from global memory.
#pragma once

#include "kernels/common.cuh"

namespace bccl {
namespace dev {


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
__device__ __forceinline__ void produce(const DevComm& c, const WorkItem& it, size_t ia, size_t ib, size_t q, int half,
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
__device__ __forceinline__ void consume(const DevComm& c, const WorkItem& it, size_t ia, size_t ib, size_t q, int half, size_t slot) {
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

// The push engine's round loop over `nitems` work items (sorted by stream offset).
__device__ __forceinline__ void push_engine_body(const DevComm& c, const WorkItem* items, int nitems, int nrounds,
                                                 size_t stream_bytes, size_t slot) {
    const uint64_t round0 = load_state_u64(&c.state->round_seq);
    const uint64_t bar0 = load_state_u64(&c.state->barrier_seq);
    if (threadIdx.x == 0) trace(c, 0, kTrBegin, (int)(bar0 & 0x7fffffffull));  // round field: barrier base
    bool ok = true;
    int first = 0;  // first item that can still overlap this CTA's pieces (items are sorted)
    // CTA b owns the same bytes [b * piece, (b + 1) * piece) of every round's inbox slot, the last
    // (shorter) round included: the per-CTA barrier that frees a half only covers CTA b on the
    // peers, so a CTA must never write bytes of a half that another CTA may still be reading.
    const size_t full = min(stream_bytes, slot);
    const size_t piece = round_up((full + gridDim.x - 1) / gridDim.x, 16);
    for (int j = 0; j < nrounds && ok; ++j) {
        const int half = (int)((round0 + (uint64_t)j) & 1ull);
        const size_t rbeg = (size_t)j * slot;
        const size_t rend = min(stream_bytes, rbeg + slot);
        const size_t a = min(rend, rbeg + (size_t)blockIdx.x * piece);
        const size_t b = min(rend, a + piece);
        while (first < nitems && items[first].stream_off + payload_bytes(items[first]) <= a) ++first;
        for (int i = first; i < nitems && a < b; ++i) {
            const WorkItem& it = items[i];
            const size_t s0 = it.stream_off, s1 = s0 + payload_bytes(it);
            if (s0 >= b) break;
            const size_t lo = max(a, s0), hi = min(b, s1);
            if (lo < hi) produce(c, it, lo - s0, hi - s0, lo - rbeg, half, slot);
        }
        ok = cta_barrier(c, bar0 + (uint64_t)j + 1, j);
        if (!ok) break;
        if (threadIdx.x == 0) trace(c, 0, kTrBarrier, j);
        for (int i = first; i < nitems && a < b; ++i) {
            const WorkItem& it = items[i];
            const size_t s0 = it.stream_off, s1 = s0 + payload_bytes(it);
            if (s0 >= b) break;
            const size_t lo = max(a, s0), hi = min(b, s1);
            if (lo < hi) consume(c, it, lo - s0, hi - s0, lo - rbeg, half, slot);
        }
    }
    if (threadIdx.x == 0) trace(c, 0, kTrEnd, nrounds);
    finish_launch(c, (uint64_t)nrounds, (uint64_t)nrounds, 0);
}

}  // namespace dev
}  // namespace bccl
