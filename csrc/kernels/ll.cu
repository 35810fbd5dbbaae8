// Low-latency AllReduce, ReduceScatter and AllGather for small payloads: data and
// synchronisation travel in the same store.
//
// The push engine's small-message cost is its barrier: the NVLink data stores, a system-scope
// fence that waits for them, a flag store, then the peer's poll. Here every 8 bytes of payload
// travel in one 16-byte line {data.lo, epoch, data.hi, epoch} written with a single vector
// store into every peer's line buffer; the receiver polls the lines themselves and takes a line
// once both epoch words match the launch's epoch (a 16-byte store may reach the peer as two
// 8-byte halves, hence two epoch words). No fence, no flag, no barrier: one NVLink trip.
//
//   rank r, launch epoch e (LLEpoch(DevState::ll_seq), the same on every rank), parity e & 1:
//     for each of its lines i: store line(i, own payload, e) into buf[peer][parity][r][i]
//     then for each of them:   poll buf[r][parity][p][i] for every peer p until epoch == e
//                              out[i] = epilogue(reduce(own, peers in rank order))
//
// ReduceScatter sends line i of input block q to peer q and reduces line i of its own block;
// AllGather sends its block's lines to every peer and writes the peers' lines into their output
// blocks. Broadcast and Reduce are not run this way: their exchange is one-sided (the root only
// sends, or only receives), so a sender could run two launches ahead of a slow receiver.
//
// Buffers alternate by parity; a rank writes parity e & 1 again only in launch e + 2, which it
// can reach only after every peer has sent its launch e + 1 lines, i.e. after every peer's
// launch e (which read those buffers) has completed. Lines are owned by the same thread on
// every rank, so a thread's sends and receives need no synchronisation with other threads.
// The line buffers are zeroed at Init (epochs start at 1). Every wait is bounded.
// The reference's small-message path is its Tree (OriginCCL src/topology/topology_tree.cpp),
// whose role on one NVSwitch node is this one-hop exchange.
#include <algorithm>

#include "kernels/common.cuh"
#include "kernels/launch.h"
#include "kernels/ll_epoch.h"

namespace bccl {
namespace dev {
namespace {

struct LLParams {
    DevComm comm;
    const char* src;
    char* dst;
    unsigned long long bytes;
    int op;
    float scale;
};

__device__ __forceinline__ uint4* ll_line(const DevComm& c, int owner, int parity, int src, size_t i) {
    char* base = c.uc[owner] + c.ll_off;
    return reinterpret_cast<uint4*>(base) + ((size_t)parity * kMaxRanks + src) * kLLMaxLines + i;
}

__device__ __forceinline__ void st_line(uint4* p, uint4 v) {
    asm volatile("st.volatile.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ uint4 ld_line(const uint4* p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p)
                 : "memory");
    return v;
}

// 8 payload bytes <-> accumulators (per dtype), combined like cta_reduce does.
template <int D> struct Pack8;
template <> struct Pack8<kF32> {
    static constexpr int E = 2;
    using Acc = float;
    static __device__ __forceinline__ void unpack(uint2 w, Acc* a) { a[0] = __uint_as_float(w.x); a[1] = __uint_as_float(w.y); }
    static __device__ __forceinline__ uint2 pack(const Acc* a) { return make_uint2(__float_as_uint(a[0]), __float_as_uint(a[1])); }
};
template <> struct Pack8<kI32> {
    static constexpr int E = 2;
    using Acc = int32_t;
    static __device__ __forceinline__ void unpack(uint2 w, Acc* a) { a[0] = (int32_t)w.x; a[1] = (int32_t)w.y; }
    static __device__ __forceinline__ uint2 pack(const Acc* a) { return make_uint2((uint32_t)a[0], (uint32_t)a[1]); }
};
template <> struct Pack8<kF64> {
    static constexpr int E = 1;
    using Acc = double;
    static __device__ __forceinline__ void unpack(uint2 w, Acc* a) {
        a[0] = __longlong_as_double((long long)(((unsigned long long)w.y << 32) | w.x));
    }
    static __device__ __forceinline__ uint2 pack(const Acc* a) {
        const unsigned long long b = (unsigned long long)__double_as_longlong(a[0]);
        return make_uint2((uint32_t)b, (uint32_t)(b >> 32));
    }
};
template <> struct Pack8<kI64> {
    static constexpr int E = 1;
    using Acc = long long;
    static __device__ __forceinline__ void unpack(uint2 w, Acc* a) { a[0] = (long long)(((unsigned long long)w.y << 32) | w.x); }
    static __device__ __forceinline__ uint2 pack(const Acc* a) {
        return make_uint2((uint32_t)(unsigned long long)a[0], (uint32_t)((unsigned long long)a[0] >> 32));
    }
};
template <> struct Pack8<kBF16> {
    static constexpr int E = 4;
    using Acc = float;
    static __device__ __forceinline__ void unpack(uint2 w, Acc* a) {
        a[0] = __uint_as_float(w.x << 16); a[1] = __uint_as_float(w.x & 0xffff0000u);
        a[2] = __uint_as_float(w.y << 16); a[3] = __uint_as_float(w.y & 0xffff0000u);
    }
    static __device__ __forceinline__ uint2 pack(const Acc* a) {
        uint32_t b[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) b[e] = Ty<kBF16>::store(a[e]);
        return make_uint2(b[0] | (b[1] << 16), b[2] | (b[3] << 16));
    }
};
template <> struct Pack8<kF16> {
    static constexpr int E = 4;
    using Acc = float;
    static __device__ __forceinline__ void unpack(uint2 w, Acc* a) {
        a[0] = Ty<kF16>::load((unsigned short)(w.x & 0xffffu)); a[1] = Ty<kF16>::load((unsigned short)(w.x >> 16));
        a[2] = Ty<kF16>::load((unsigned short)(w.y & 0xffffu)); a[3] = Ty<kF16>::load((unsigned short)(w.y >> 16));
    }
    static __device__ __forceinline__ uint2 pack(const Acc* a) {
        uint32_t b[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) b[e] = Ty<kF16>::store(a[e]);
        return make_uint2(b[0] | (b[1] << 16), b[2] | (b[3] << 16));
    }
};

// 8 bytes at p (fewer at the payload's end; unaligned addresses byte by byte).
__device__ __forceinline__ uint2 load8(const char* p, size_t valid) {
    if (valid >= 8 && (reinterpret_cast<uintptr_t>(p) & 7) == 0) return *reinterpret_cast<const uint2*>(p);
    uint2 v = make_uint2(0, 0);
    char* b = reinterpret_cast<char*>(&v);
    for (size_t k = 0; k < 8 && k < valid; ++k) b[k] = p[k];
    return v;
}
__device__ __forceinline__ void store8(char* p, uint2 v, size_t valid) {
    if (valid >= 8 && (reinterpret_cast<uintptr_t>(p) & 7) == 0) {
        *reinterpret_cast<uint2*>(p) = v;
        return;
    }
    const char* b = reinterpret_cast<const char*>(&v);
    for (size_t k = 0; k < 8 && k < valid; ++k) p[k] = b[k];
}

// Waits (bounded) until line `src` carries `epoch` in both halves; returns its payload.
__device__ __forceinline__ bool ll_recv(const DevComm& c, const uint4* src, uint32_t epoch, int peer, uint2* out) {
    uint4 v = ld_line(src);
    if (v.y != epoch || v.w != epoch) {
        const uint64_t t0 = globaltimer();
        for (uint32_t it = 1;; ++it) {
            v = ld_line(src);
            if (v.y == epoch && v.w == epoch) break;
            if ((it & 255u) == 0) {
                const uint64_t waited = globaltimer() - t0;
                if ((waited > kAbortCheckAfterNs && *c.abort != 0) || waited > c.timeout_ns) {
                    record_error(c, *c.abort != 0 ? kDevAborted : kDevTimeout, peer, 0, epoch, waited);
                    return false;
                }
            }
        }
    }
    *out = make_uint2(v.x, v.z);
    return true;
}

// AllReduce (RS = false: every peer gets this rank's payload line) and ReduceScatter (RS = true:
// input = N blocks of p.bytes, peer q gets line i of block q); each thread then reduces line i
// of its own part from every rank's contribution, in rank order.
template <int D, int O, bool RS>
__global__ void __launch_bounds__(256) ll_reduce_kernel(const __grid_constant__ LLParams p) {
    const DevComm& c = p.comm;
    const int r = c.rank, n = c.nranks;
    const uint32_t epoch = LLEpoch(load_state_u64(&c.state->ll_seq));
    const int parity = (int)(epoch & 1u);
    const size_t lines = (p.bytes + 7) / 8;
    using P = Pack8<D>;
    using Acc = typename P::Acc;
    const size_t first = (size_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
    // Every line goes out before any is awaited, so a thread with several lines keeps one round
    // trip in flight for all of them.
    for (size_t i = first; i < lines; i += stride) {
        const size_t off = i * 8, valid = min((size_t)8, (size_t)p.bytes - off);
        const uint2 mine = load8(p.src + (RS ? (size_t)r * p.bytes : 0) + off, valid);
        for (int q = 0; q < n; ++q) {
            if (q == r) continue;
            const uint2 d = RS ? load8(p.src + (size_t)q * p.bytes + off, valid) : mine;
            st_line(ll_line(c, q, parity, r, i), make_uint4(d.x, epoch, d.y, epoch));
        }
    }
    bool ok = true;
    for (size_t i = first; i < lines && ok; i += stride) {
        const size_t off = i * 8, valid = min((size_t)8, (size_t)p.bytes - off);
        // Ranks in order, so every rank rounds the same way and gets bit-identical results; each
        // contribution is folded in as it arrives (no per-rank array in local memory).
        Acc acc[P::E], x[P::E];
        for (int q = 0; q < n; ++q) {
            uint2 w;
            if (q == r) {
                // Own part of the input, read again: only this thread writes these bytes of the
                // output, so an in-place call still sees its input here.
                w = load8(p.src + (RS ? (size_t)r * p.bytes : 0) + off, valid);
            } else if (!ll_recv(c, ll_line(c, r, parity, q, i), epoch, q, &w)) {
                ok = false;
                break;
            }
            P::unpack(w, q == 0 ? acc : x);
            if (q > 0) {
#pragma unroll
                for (int e = 0; e < P::E; ++e) acc[e] = combine<Acc>(O, acc[e], x[e]);
            }
        }
        if (!ok) break;
#pragma unroll
        for (int e = 0; e < P::E; ++e) acc[e] = epilogue<Acc>(O, acc[e], n, p.scale);
        store8(p.dst + off, P::pack(acc), valid);
    }
    finish_launch(c, 0, 0, 0, 0, 1);
}

// AllGather: every peer gets this rank's block line by line; the output's block q receives rank
// q's lines (this rank's own block is copied locally).
__global__ void __launch_bounds__(256) ll_allgather_kernel(const __grid_constant__ LLParams p) {
    const DevComm& c = p.comm;
    const int r = c.rank, n = c.nranks;
    const uint32_t epoch = LLEpoch(load_state_u64(&c.state->ll_seq));
    const int parity = (int)(epoch & 1u);
    const size_t lines = (p.bytes + 7) / 8;
    const size_t first = (size_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
    char* own = p.dst + (size_t)r * p.bytes;
    for (size_t i = first; i < lines; i += stride) {
        const size_t off = i * 8, valid = min((size_t)8, (size_t)p.bytes - off);
        const uint2 mine = load8(p.src + off, valid);
        const uint4 line = make_uint4(mine.x, epoch, mine.y, epoch);
        for (int q = 0; q < n; ++q)
            if (q != r) st_line(ll_line(c, q, parity, r, i), line);
        if (own != p.src) store8(own + off, mine, valid);
    }
    bool ok = true;
    for (size_t i = first; i < lines && ok; i += stride) {
        const size_t off = i * 8, valid = min((size_t)8, (size_t)p.bytes - off);
        for (int q = 0; q < n && ok; ++q) {
            if (q == r) continue;
            uint2 d;
            ok = ll_recv(c, ll_line(c, r, parity, q, i), epoch, q, &d);
            if (ok) store8(p.dst + (size_t)q * p.bytes + off, d, valid);
        }
    }
    finish_launch(c, 0, 0, 0, 0, 1);
}

template <int D, bool RS>
cudaError_t launch_op(const LLParams& p, int nctas, cudaStream_t s) {
    switch (p.op) {
    case kSum: ll_reduce_kernel<D, kSum, RS><<<nctas, 256, 0, s>>>(p); break;
    case kMax: ll_reduce_kernel<D, kMax, RS><<<nctas, 256, 0, s>>>(p); break;
    case kMin: ll_reduce_kernel<D, kMin, RS><<<nctas, 256, 0, s>>>(p); break;
    case kAvg: ll_reduce_kernel<D, kAvg, RS><<<nctas, 256, 0, s>>>(p); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

template <bool RS>
cudaError_t launch_dtype(const LLParams& p, int dtype, int nctas, cudaStream_t s) {
    switch (dtype) {
    case kF32: return launch_op<kF32, RS>(p, nctas, s);
    case kF64: return launch_op<kF64, RS>(p, nctas, s);
    case kI32: return launch_op<kI32, RS>(p, nctas, s);
    case kI64: return launch_op<kI64, RS>(p, nctas, s);
    case kBF16: return launch_op<kBF16, RS>(p, nctas, s);
    case kF16: return launch_op<kF16, RS>(p, nctas, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace
}  // namespace dev

cudaError_t LaunchCollectiveLL(const DevComm& c, int func, const void* src, void* dst, unsigned long long count,
                               int dtype, int op, float scale, cudaStream_t stream) {
    using namespace dev;
    const unsigned long long bytes = count * (unsigned long long)dtype_size(dtype);
    const unsigned long long lines = (bytes + 7) / 8;
    if (c.nranks < 2 || c.ll_off == 0 || bytes == 0 || lines > kLLMaxLines || (func != 0 && func != 3 && func != 4)) {
        return cudaErrorInvalidValue;
    }
    LLParams p;
    p.comm = c;
    p.src = static_cast<const char*>(src);
    p.dst = static_cast<char*>(dst);
    p.bytes = bytes;
    p.op = op;
    p.scale = scale;
    // One line per thread: 256-thread CTAs, as many as the lines need (up to two per SM; larger
    // payloads loop, each thread taking every (grid * 256)-th line).
    const int nctas = (int)std::min<unsigned long long>(296, (lines + 255) / 256);
    if (func == 3) {
        ll_allgather_kernel<<<nctas, 256, 0, stream>>>(p);
        return cudaGetLastError();
    }
    return func == 4 ? launch_dtype<true>(p, dtype, nctas, stream) : launch_dtype<false>(p, dtype, nctas, stream);
}

}  // namespace bccl
