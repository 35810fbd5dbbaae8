// Ring AllReduce: reduce-scatter then all-gather between ring neighbours only.
//
// Parity with the reference's ring (OriginCCL src/topology/topology_ring.cpp:255-290,370-431):
// the payload is cut into units of N blocks; in unit u, rank r first sends block r to rank r+1,
// then for steps s = 1 .. 2N-2 receives block (r - s) mod N from rank r-1, adds its own copy
// while s < N (the block is complete at s = N-1 and is written to the output with the AVG /
// scale epilogue), and forwards it unless it is the last step. On one NVSwitch node every GPU
// reaches every other at full bandwidth, so the one-shot / two-shot / NVLS kernels are the
// defaults; the ring is kept as the neighbour-only algorithm (BCCL_ALGO=ring).
//
// B200 mapping: a "channel" is one CTA, which owns units blockIdx.x, blockIdx.x + grid, ... A
// message is one block written with st.global into the successor's inbox (two slots per CTA,
// in the successor's peer-mapped data region), then announced by a posted counter in the
// successor's control region; the successor returns a consumed counter so the slot can be
// reused. Counters are message numbers offset by DevState::ring_seq, monotonic across
// launches. One system-scope fence per step orders the block (and the inbox reads) before the
// counters. All waits are bounded. The kernel ends with a barrier over every rank, so the next
// launch may reuse the inbox region.
#include <algorithm>

#include "kernels/common.cuh"
#include "kernels/launch.h"

namespace bccl {
namespace dev {
namespace {

struct RingParams {
    DevComm comm;
    const void* src;
    void* dst;
    unsigned long long bytes;
    unsigned long long block;  // bytes per block (multiple of 16)
    unsigned long long units;
    unsigned long long msgs_max;  // messages of the busiest CTA (advance of ring_seq)
    int op;
    float scale;
};

__device__ __forceinline__ uint64_t* ring_flag(char* uc_base, size_t off, int cta) {
    return reinterpret_cast<uint64_t*>(uc_base + off) + cta;
}

__device__ __forceinline__ char* ring_inbox(const DevComm& c, int owner, int cta, int slot, size_t block) {
    return c.uc[owner] + kCtrlBytes + (size_t)(c.data_bytes / 2) + ((size_t)cta * 2 + slot) * block;
}

// Copies `bytes` (ld.cg: the source was written by another GPU) to every destination in outs.
__device__ __forceinline__ void fwd_cg(char* const* outs, int no, const char* s, size_t bytes) {
    const size_t t = threadIdx.x, nt = blockDim.x;
    uintptr_t mis = reinterpret_cast<uintptr_t>(s);
    for (int q = 0; q < no; ++q) mis |= reinterpret_cast<uintptr_t>(outs[q]);
    const size_t nv = (mis & 15) ? 0 : (bytes >> 4);
    size_t i = t;
    for (; i + nt < nv; i += 2 * nt) {
        const uint4 a = ld_cg(s + (i << 4)), b = ld_cg(s + ((i + nt) << 4));
        for (int q = 0; q < no; ++q) {
            st_cg(outs[q] + (i << 4), a);
            st_cg(outs[q] + ((i + nt) << 4), b);
        }
    }
    for (; i < nv; i += nt) {
        const uint4 a = ld_cg(s + (i << 4));
        for (int q = 0; q < no; ++q) st_cg(outs[q] + (i << 4), a);
    }
    for (size_t j = (nv << 4) + t; j < bytes; j += nt) {
        const char b = (char)__ldcg(reinterpret_cast<const signed char*>(s + j));
        for (int q = 0; q < no; ++q) outs[q][j] = b;
    }
}

// outs[q][i] = epilogue(a[i] (+) b[i]); `a` is an inbox (ld.cg), `b` this rank's input.
template <int D, int O>
__device__ __forceinline__ void add2(char* const* outs, int no, const char* a, const char* b, size_t bytes,
                                     bool final_step, int nranks, float scale) {
    using V = Vec<D>;
    using Acc = typename Ty<D>::Acc;
    using Bits = typename Ty<D>::Bits;
    const size_t t = threadIdx.x, nt = blockDim.x;
    uintptr_t mis = reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b);
    for (int q = 0; q < no; ++q) mis |= reinterpret_cast<uintptr_t>(outs[q]);
    const size_t nv = (mis & 15) ? 0 : (bytes >> 4);
    // Partial sums travel without the epilogue; AVG divides once, at the final step.
    constexpr int OP = (O == kAvg) ? kSum : O;
    const bool post = final_step && (O == kAvg || scale != 1.0f);
    for (size_t i = t; i < nv; i += nt) {
        Acc x[V::E], y[V::E];
        V::unpack(ld_cg(a + (i << 4)), x);
        V::unpack(*reinterpret_cast<const uint4*>(b + (i << 4)), y);
#pragma unroll
        for (int e = 0; e < V::E; ++e) {
            x[e] = combine<Acc>(OP, x[e], y[e]);
            if (post) x[e] = epilogue<Acc>(O, x[e], nranks, scale);
        }
        const uint4 r = V::pack(x);
        for (int q = 0; q < no; ++q) st_cg(outs[q] + (i << 4), r);
    }
    for (size_t j = (nv << 4) + t * sizeof(Bits); j < bytes; j += nt * sizeof(Bits)) {
        Acc x = Ty<D>::load(__ldcg(reinterpret_cast<const Bits*>(a + j)));
        x = combine<Acc>(OP, x, Ty<D>::load(*reinterpret_cast<const Bits*>(b + j)));
        if (post) x = epilogue<Acc>(O, x, nranks, scale);
        for (int q = 0; q < no; ++q) *reinterpret_cast<Bits*>(outs[q] + j) = Ty<D>::store(x);
    }
}

template <int D, int O>
__global__ void __launch_bounds__(512, 1) ring_kernel(const __grid_constant__ RingParams p) {
    const DevComm& c = p.comm;
    const int r = c.rank, n = c.nranks;
    const int next = (r + 1) % n, prev = (r + n - 1) % n;
    const uint64_t B = load_state_u64(&c.state->ring_seq);
    const uint64_t bar0 = load_state_u64(&c.state->barrier_seq);
    const size_t blk = p.block, unit = (size_t)n * blk;
    const char* src = static_cast<const char*>(p.src);
    char* dst = static_cast<char*>(p.dst);
    uint64_t* posted_here = ring_flag(c.uc[r], kRingPostedOff, blockIdx.x);
    uint64_t* consumed_here = ring_flag(c.uc[r], kRingConsumedOff, blockIdx.x);
    uint64_t* posted_next = ring_flag(c.uc[next], kRingPostedOff, blockIdx.x);
    uint64_t* consumed_prev = ring_flag(c.uc[prev], kRingConsumedOff, blockIdx.x);
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        s_ok = 1;
        trace(c, 0, kTrBegin, (int)(B & 0x7fffffffull));
    }
    __syncthreads();
    uint64_t m = 0;  // messages this CTA sent (and received) in this launch
    for (uint64_t u = blockIdx.x; u < p.units && s_ok; u += gridDim.x) {
        const size_t base = (size_t)u * unit;
        const size_t ulen = min((size_t)p.bytes - base, unit);
        auto blen = [&](int k) -> size_t {
            const size_t lo = (size_t)k * blk;
            return lo >= ulen ? 0 : min(blk, ulen - lo);
        };
        const uint64_t mb = m;
        for (int s = 0; s <= 2 * n - 2 && s_ok; ++s) {
            // ---- receive (steps >= 1): message mb + s - 1 from prev, block (r - s) mod n
            const int kin = ((r - s) % n + n) % n;
            const uint64_t gin = B + mb + (uint64_t)s - 1;
            const char* inb = ring_inbox(c, r, blockIdx.x, (int)(gin & 1ull), blk);
            // ---- send (steps <= 2n-3): message mb + s to next
            const bool do_send = s <= 2 * n - 3;
            const uint64_t gout = B + mb + (uint64_t)s;
            char* outb = ring_inbox(c, next, blockIdx.x, (int)(gout & 1ull), blk);
            if (threadIdx.x == 0) {
                bool ok = true;
                if (s >= 1) ok = wait_flag_geq(c, posted_here, gin + 1, prev, s);
                // the successor consumed message gout-2 (same slot), unless it was sent in an
                // earlier launch (the end-of-launch barrier then covers it)
                if (ok && do_send && mb + (uint64_t)s >= 2) ok = wait_flag_geq(c, consumed_here, gout - 1, next, s);
                if (!ok) s_ok = 0;
            }
            __syncthreads();
            if (!s_ok) break;
            const size_t len = s == 0 ? blen(r) : blen(kin);
            const size_t off = base + (size_t)(s == 0 ? r : kin) * blk;
            char* outs[2];
            if (s == 0) {
                outs[0] = outb;
                cta_copy(outs[0], src + off, len, false);
            } else if (s < n - 1) {  // reduce-scatter hop: partial sum to the successor
                outs[0] = outb;
                add2<D, O>(outs, 1, inb, src + off, len, false, n, p.scale);
            } else if (s == n - 1) {  // block complete: output + first all-gather hop
                outs[0] = dst + off;
                outs[1] = outb;
                add2<D, O>(outs, do_send ? 2 : 1, inb, src + off, len, true, n, p.scale);
            } else {  // all-gather hop
                outs[0] = dst + off;
                outs[1] = outb;
                fwd_cg(outs, do_send ? 2 : 1, inb, len);
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                fence_acq_rel_sys();  // the block (and the inbox reads) before the counters
                if (do_send) st_relaxed_sys_flag(posted_next, gout + 1);
                if (s >= 1) st_relaxed_sys_flag(consumed_prev, gin + 1);
            }
        }
        m = mb + 2ull * (uint64_t)n - 2ull;
    }
    __syncthreads();
    if (threadIdx.x == 0) trace(c, 0, kTrEnd, (int)m);
    // Every rank is done with every inbox before any rank's next launch writes one.
    if (s_ok) cta_barrier(c, bar0 + 1, 0);
    finish_launch(c, 0, 1, 0, p.msgs_max);
}

template <int D, int O>
cudaError_t launch_t(const RingParams& p, int nctas, cudaStream_t s) {
    ring_kernel<D, O><<<nctas, 512, 0, s>>>(p);
    return cudaGetLastError();
}

template <int D>
cudaError_t launch_op(const RingParams& p, int nctas, cudaStream_t s) {
    switch (p.op) {
    case kSum: return launch_t<D, kSum>(p, nctas, s);
    case kAvg: return launch_t<D, kAvg>(p, nctas, s);
    case kMax: return launch_t<D, kMax>(p, nctas, s);
    case kMin: return launch_t<D, kMin>(p, nctas, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace
}  // namespace dev

cudaError_t LaunchRingAllReduce(const DevComm& c, const void* src, void* dst, unsigned long long count, int dtype,
                                int op, float scale, unsigned long long block, int max_ctas, cudaStream_t stream) {
    using namespace dev;
    const unsigned long long es = dtype_size(dtype);
    if (c.nranks < 2 || es == 0 || block == 0 || (block % 256) != 0 || max_ctas < 1) return cudaErrorInvalidValue;
    RingParams p;
    p.comm = c;
    p.src = src;
    p.dst = dst;
    p.bytes = count * es;
    p.block = block;
    const unsigned long long unit = (unsigned long long)c.nranks * block;
    p.units = (p.bytes + unit - 1) / unit;
    if (p.units == 0) p.units = 1;
    const int nctas = (int)std::min<unsigned long long>(p.units, (unsigned long long)std::min(max_ctas, kMaxCtas));
    if ((size_t)nctas * 2 * block > c.data_bytes / 2) return cudaErrorInvalidValue;
    p.msgs_max = ((p.units + nctas - 1) / nctas) * (2ull * c.nranks - 2ull);
    p.op = op;
    p.scale = scale;
    switch (dtype) {
    case kF32: return launch_op<kF32>(p, nctas, stream);
    case kF64: return launch_op<kF64>(p, nctas, stream);
    case kI32: return launch_op<kI32>(p, nctas, stream);
    case kI64: return launch_op<kI64>(p, nctas, stream);
    case kBF16: return launch_op<kBF16>(p, nctas, stream);
    case kF16: return launch_op<kF16>(p, nctas, stream);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace bccl
