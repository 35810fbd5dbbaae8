// NVSwitch multicast Broadcast, Reduce, AllGather and ReduceScatter on staged (unregistered)
// buffers.
//
// The reference moves every byte through per-edge transports and reduces on the CPU
// (OriginCCL src/topology/topology_ring.cpp:178-253). With NVLS:
//   Broadcast:     the root multimem.st's each chunk once (one egress copy; the switch fans it
//                  out to every GPU) -> barrier -> every rank copies the slot to its output.
//   Reduce:        every rank copies its chunk into its slot -> barrier -> the root
//                  multimem.ld_reduce's the slot (the switch reads and reduces all copies) into
//                  its output -> barrier.
//   AllGather:     every rank multimem.st's its block's chunk into sub-slot `rank` of every
//                  GPU's slot (one egress copy of the block instead of N-1) -> barrier -> every
//                  rank copies the N sub-slots to its output.
//   ReduceScatter: every rank copies the chunk of each of its N input blocks into sub-slot q of
//                  its slot -> barrier -> rank r multimem.ld_reduce's sub-slot r (the switch
//                  reduces the N copies) into its output. One barrier per round: with three or
//                  more slots, round j+1's copy-in lands in a slot no rank still reads.
// AllGather and ReduceScatter take `chunk` bytes of every rank's block per round, so a slot
// holds N chunks.
// Slots form the same ring (indexed by DevState::nvls_round_seq) as the pipelined AllReduce,
// so the two kinds of launch can follow each other.
// No fence.proxy.alias between the multicast and unicast views of a slot: the system-scope
// release/acquire of the barrier orders them (switch writes land in the owner's L2, and the
// copy-out reads with ld.global.cg), as in the pipelined AllReduce; the alias fence cost tens
// of microseconds per round with multicast traffic in flight.
#include "kernels/common.cuh"
#include "kernels/launch.h"

namespace bccl {
namespace dev {
namespace {

template <int D, int O> __device__ __forceinline__ uint4 red16(const void* p);
#define NV_V4(D, O, SPEC)                                                                        \
    template <> __device__ __forceinline__ uint4 red16<D, O>(const void* p) {                    \
        uint4 r;                                                                               \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " {%0,%1,%2,%3}, [%4];"     \
                     : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p) : "memory");        \
        return r;                                                                              \
    }
#define NV_S32(D, O, SPEC)                                                                       \
    template <> __device__ __forceinline__ uint4 red16<D, O>(const void* p) {                    \
        uint4 r;                                                                               \
        const char* c = static_cast<const char*>(p);                                           \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " %0, [%1];" : "=r"(r.x) : "l"(c) : "memory");      \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " %0, [%1];" : "=r"(r.y) : "l"(c + 4) : "memory");  \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " %0, [%1];" : "=r"(r.z) : "l"(c + 8) : "memory");  \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " %0, [%1];" : "=r"(r.w) : "l"(c + 12) : "memory"); \
        return r;                                                                              \
    }
#define NV_S64(D, O, SPEC)                                                                       \
    template <> __device__ __forceinline__ uint4 red16<D, O>(const void* p) {                    \
        unsigned long long a, b;                                                               \
        const char* c = static_cast<const char*>(p);                                           \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " %0, [%1];" : "=l"(a) : "l"(c) : "memory");     \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " %0, [%1];" : "=l"(b) : "l"(c + 8) : "memory"); \
        return make_uint4((unsigned)a, (unsigned)(a >> 32), (unsigned)b, (unsigned)(b >> 32));                      \
    }
NV_V4(kF32, kSum, "add.v4.f32")
NV_V4(kBF16, kSum, "add.acc::f32.v4.bf16x2")
NV_V4(kBF16, kMax, "max.v4.bf16x2")
NV_V4(kBF16, kMin, "min.v4.bf16x2")
NV_V4(kF16, kSum, "add.acc::f32.v4.f16x2")
NV_V4(kF16, kMax, "max.v4.f16x2")
NV_V4(kF16, kMin, "min.v4.f16x2")
NV_S32(kI32, kSum, "add.u32")
NV_S32(kI32, kMax, "max.s32")
NV_S32(kI32, kMin, "min.s32")
NV_S64(kI64, kSum, "add.u64")
NV_S64(kI64, kMax, "max.s64")
NV_S64(kI64, kMin, "min.s64")
NV_S64(kF64, kSum, "add.f64")

__device__ __forceinline__ void mm_st(void* p, const uint4& v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

// 16 bytes from a possibly short or unaligned tail (never reads past `valid`).
__device__ __forceinline__ uint4 load_partial(const char* p, size_t valid) {
    if (valid >= 16 && (reinterpret_cast<uintptr_t>(p) & 15) == 0) return *reinterpret_cast<const uint4*>(p);
    uint4 v = make_uint4(0, 0, 0, 0);
    char* b = reinterpret_cast<char*>(&v);
    for (size_t i = 0; i < 16 && i < valid; ++i) b[i] = p[i];
    return v;
}

struct NvlsParams {
    DevComm comm;
    const void* src;
    void* dst;
    unsigned long long bytes;
    unsigned long long chunk;       // bytes per round
    unsigned long long slot_bytes;  // >= chunk, multiple of 16
    int nslots;
    int nrounds;
    int func;  // 1 Broadcast, 2 Reduce, 3 AllGather, 4 ReduceScatter (CollFunc values)
    int op;
    int root;
    float scale;
};

// Multicast stores of [lo, hi) of `src` to `mc` (four 16-byte loads in flight per thread).
__device__ __forceinline__ void mcast_range(char* mc, const char* src, size_t lo, size_t hi) {
    const size_t t = threadIdx.x, nt = blockDim.x;
    size_t off = lo + t * 16;
    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        for (; off + 3 * nt * 16 + 16 <= hi; off += 4 * nt * 16) {
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = *reinterpret_cast<const uint4*>(src + off + u * nt * 16);
#pragma unroll
            for (int u = 0; u < 4; ++u) mm_st(mc + off + u * nt * 16, v[u]);
        }
    }
    for (; off < hi; off += nt * 16) mm_st(mc + off, load_partial(src + off, hi - off));
}

// dst[lo, hi) = epilogue(multimem.ld_reduce of mc[lo, hi)); four switch reductions in flight
// per thread (each is a round trip through the switch to every GPU), then their stores.
template <int D, int O>
__device__ __forceinline__ void reduce_range(char* dst, const char* mc, size_t lo, size_t hi, int op, int n,
                                             float scale) {
    constexpr int E = 16 / sizeof(typename Ty<D>::Bits);
    const bool post = op == kAvg || scale != 1.0f;
    const size_t t = threadIdx.x, nt = blockDim.x;
    size_t off = lo + t * 16;
    if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        for (; off + 3 * nt * 16 + 16 <= hi; off += 4 * nt * 16) {
            V16<D> v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u].u = red16<D, O>(mc + off + u * nt * 16);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (post) {
#pragma unroll
                    for (int e = 0; e < E; ++e)
                        v[u].b[e] = Ty<D>::store(epilogue<typename Ty<D>::Acc>(op, Ty<D>::load(v[u].b[e]), n, scale));
                }
                *reinterpret_cast<uint4*>(dst + off + u * nt * 16) = v[u].u;
            }
        }
    }
    for (; off < hi; off += nt * 16) {
        V16<D> v;
        v.u = red16<D, O>(mc + off);
        if (post) {
#pragma unroll
            for (int e = 0; e < E; ++e)
                v.b[e] = Ty<D>::store(epilogue<typename Ty<D>::Acc>(op, Ty<D>::load(v.b[e]), n, scale));
        }
        const size_t valid = min((size_t)16, hi - off);
        char* d = dst + off;
        if (valid == 16 && (reinterpret_cast<uintptr_t>(d) & 15) == 0) {
            *reinterpret_cast<uint4*>(d) = v.u;
        } else {
            for (size_t i = 0; i < valid; ++i) d[i] = reinterpret_cast<const char*>(&v.u)[i];
        }
    }
}

template <int D, int O>
__global__ void __launch_bounds__(512, 1) nvls_kernel(const __grid_constant__ NvlsParams p) {
    const DevComm& c = p.comm;
    const int r = c.rank, n = c.nranks;
    const uint64_t round0 = load_state_u64(&c.state->nvls_round_seq);
    uint64_t bar = load_state_u64(&c.state->barrier_seq);
    if (threadIdx.x == 0) trace(c, 0, kTrBegin, (int)(bar & 0x7fffffffull));
    const int per_round = (p.func == 2) ? 2 : 1;
    const char* sbase = static_cast<const char*>(p.src);
    char* dbase = static_cast<char*>(p.dst);
    // CTA b owns the same bytes of a slot in every round (the last, shorter one included): a slot
    // is reused every nslots rounds and the per-CTA barrier only covers CTA b on the other ranks.
    const size_t piece = round_up((min((size_t)p.bytes, (size_t)p.chunk) + gridDim.x - 1) / gridDim.x, 16);
    for (int j = 0; j < p.nrounds; ++j) {
        const size_t cbeg = (size_t)j * p.chunk;
        const size_t clen = min((size_t)p.bytes - cbeg, (size_t)p.chunk);
        const size_t lo = min(clen, (size_t)blockIdx.x * piece), hi = min(clen, lo + piece);
        const size_t slot = (size_t)((round0 + (uint64_t)j) % (uint64_t)p.nslots);
        char* uc = c.nvls_uc + slot * p.slot_bytes;
        char* mc = c.nvls_mc + slot * p.slot_bytes;
        if (p.func == 1) {  // Broadcast
            const char* src = sbase + cbeg;
            char* dst = dbase + cbeg;
            if (r == p.root) mcast_range(mc, src, lo, hi);
            if (!cta_barrier(c, ++bar, j)) break;
            if (lo < hi && r != p.root) cta_copy(dst + lo, uc + lo, hi - lo, true);
            if (lo < hi && r == p.root && dst != src) cta_copy(dst + lo, src + lo, hi - lo, false);
        } else if (p.func == 2) {  // Reduce
            const char* src = sbase + cbeg;
            if (lo < hi) cta_copy(uc + lo, src + lo, hi - lo, false);
            if (!cta_barrier(c, ++bar, 2 * j)) break;
            if (r == p.root) reduce_range<D, O>(dbase + cbeg, mc, lo, hi, p.op, n, p.scale);
            if (!cta_barrier(c, ++bar, 2 * j + 1)) break;
        } else if (p.func == 3) {  // AllGather: src = this rank's block, dst = [n][bytes]
            mcast_range(mc + (size_t)r * p.chunk, sbase + cbeg, lo, hi);
            if (!cta_barrier(c, ++bar, j)) break;
            if (lo < hi) {
                for (int q = 0; q < n; ++q) {
                    char* out = dbase + (size_t)q * p.bytes + cbeg;
                    if (q == r) {
                        if (out != sbase + cbeg) cta_copy(out + lo, sbase + cbeg + lo, hi - lo, false);
                    } else {
                        cta_copy(out + lo, uc + (size_t)q * p.chunk + lo, hi - lo, true);
                    }
                }
            }
        } else {  // ReduceScatter: src = [n][bytes], dst = this rank's block
            if (lo < hi) {
                for (int q = 0; q < n; ++q)
                    cta_copy(uc + (size_t)q * p.chunk + lo, sbase + (size_t)q * p.bytes + cbeg + lo, hi - lo, false);
            }
            if (!cta_barrier(c, ++bar, j)) break;
            reduce_range<D, O>(dbase + cbeg, mc + (size_t)r * p.chunk, lo, hi, p.op, n, p.scale);
        }
    }
    if (threadIdx.x == 0) trace(c, 0, kTrEnd, p.nrounds);
    finish_launch(c, 0, (uint64_t)per_round * (uint64_t)p.nrounds, (uint64_t)p.nrounds);
}

// Zero-copy collectives on buffers bound to the multicast object (symmetric user buffers), no
// staging:
//   AllReduce:     rank r reduces its shard of every 16-byte vector straight from all ranks' send
//                  buffers (multimem.ld_reduce on the send buffer's multicast address) and stores
//                  it into every rank's receive buffer (multimem.st on its multicast address);
//   ReduceScatter: rank r reduces its own block from all ranks' send buffers into its output;
//   AllGather:     rank r stores its input block into every rank's receive buffer at block r.
// An entry barrier makes every rank's input (and free output) ready before any rank touches
// them; the exit barrier (system-scope release after the multicast stores) makes every output
// complete, and every input read, before any rank's later work. Symmetric buffers sit at the
// same offset on every rank.
struct ZcParams {
    DevComm comm;
    const char* send;   // AllReduce, ReduceScatter: the send buffer's multicast address; AllGather: local input
    char* recv;         // AllReduce, AllGather: the receive buffer's multicast address; ReduceScatter: local output
    unsigned long long bytes;  // AllReduce: payload; AllGather / ReduceScatter: per-rank block; multiple of 16
    int func;           // 0 AllReduce, 3 AllGather, 4 ReduceScatter (CollFunc values)
    int op;
    float scale;
};

template <int D, int O>
__global__ void __launch_bounds__(512, 1) nvls_zc_kernel(const __grid_constant__ ZcParams p) {
    const DevComm& c = p.comm;
    const int r = c.rank, n = c.nranks;
    const uint64_t bar = load_state_u64(&c.state->barrier_seq);
    if (threadIdx.x == 0) trace(c, 0, kTrBegin, (int)(bar & 0x7fffffffull));
    bool ok = cta_barrier(c, bar + 1, 0);
    if (ok && p.func == 3) {  // AllGather: this rank's block into every rank's output
        const size_t nvec = p.bytes / 16;
        const size_t per_cta = (nvec + gridDim.x - 1) / gridDim.x;
        const size_t c0 = min(nvec, (size_t)blockIdx.x * per_cta), c1 = min(nvec, c0 + per_cta);
        char* out = p.recv + (size_t)r * p.bytes;
        size_t i = c0 + threadIdx.x;
        for (; i + 3 * blockDim.x < c1; i += 4 * blockDim.x) {
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = *reinterpret_cast<const uint4*>(p.send + (i + u * blockDim.x) * 16);
#pragma unroll
            for (int u = 0; u < 4; ++u) mm_st(out + (i + u * blockDim.x) * 16, v[u]);
        }
        for (; i < c1; i += blockDim.x) mm_st(out + i * 16, *reinterpret_cast<const uint4*>(p.send + i * 16));
        ok = cta_barrier(c, bar + 2, 1);
    } else if (ok) {
        constexpr int E = 16 / sizeof(typename Ty<D>::Bits);
        const bool post = p.op == kAvg || p.scale != 1.0f;
        const bool rs = p.func == 4;  // ReduceScatter: reduce this rank's block into local memory
        const size_t nvec = p.bytes / 16;
        const size_t per_rank = rs ? nvec : (nvec + n - 1) / n;
        const size_t r0 = rs ? 0 : min(nvec, (size_t)r * per_rank), r1 = min(nvec, r0 + per_rank);
        const char* in = rs ? p.send + (size_t)r * p.bytes : p.send;
        const size_t per_cta = (r1 - r0 + gridDim.x - 1) / gridDim.x;
        const size_t c0 = min(r1, r0 + (size_t)blockIdx.x * per_cta), c1 = min(r1, c0 + per_cta);
        const size_t t = threadIdx.x, nt = blockDim.x;
        // AllReduce: multicast store of the reduced vector to every rank; ReduceScatter: plain
        // store to this rank's output.
        auto put = [&](size_t idx, const uint4& val) {
            if (rs) *reinterpret_cast<uint4*>(p.recv + idx * 16) = val;
            else mm_st(p.recv + idx * 16, val);
        };
        size_t i = c0 + t;
        for (; i + 3 * nt < c1; i += 4 * nt) {  // four reductions in flight per thread
            V16<D> v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u].u = red16<D, O>(in + (i + u * nt) * 16);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (post) {
#pragma unroll
                    for (int e = 0; e < E; ++e)
                        v[u].b[e] = Ty<D>::store(epilogue<typename Ty<D>::Acc>(p.op, Ty<D>::load(v[u].b[e]), n, p.scale));
                }
                put(i + u * nt, v[u].u);
            }
        }
        for (; i < c1; i += nt) {
            V16<D> v;
            v.u = red16<D, O>(in + i * 16);
            if (post) {
#pragma unroll
                for (int e = 0; e < E; ++e)
                    v.b[e] = Ty<D>::store(epilogue<typename Ty<D>::Acc>(p.op, Ty<D>::load(v.b[e]), n, p.scale));
            }
            put(i, v.u);
        }
        ok = cta_barrier(c, bar + 2, 1);
    }
    if (threadIdx.x == 0) trace(c, 0, kTrEnd, 0);
    finish_launch(c, 0, 2, 0);
}

template <int D, int O>
cudaError_t launch_zc(const ZcParams& p, int nctas, cudaStream_t s) {
    nvls_zc_kernel<D, O><<<nctas, 512, 0, s>>>(p);
    return cudaGetLastError();
}

template <int D, int O>
cudaError_t launch_t(const NvlsParams& p, int nctas, cudaStream_t s) {
    nvls_kernel<D, O><<<nctas, 512, 0, s>>>(p);
    return cudaGetLastError();
}

}  // namespace
}  // namespace dev

cudaError_t LaunchNvlsZeroCopy(const DevComm& c, int func, const void* send, void* recv, unsigned long long count,
                               int dtype, int op, float scale, int nctas, cudaStream_t stream) {
    using namespace dev;
    const unsigned long long bytes = count * (unsigned long long)dtype_size(dtype);
    if (nctas <= 0 || nctas > kMaxCtas || (bytes % 16) != 0 ||
        ((reinterpret_cast<uintptr_t>(send) | reinterpret_cast<uintptr_t>(recv)) & 15) != 0 ||
        (func != 0 && func != 3 && func != 4) || (func != 3 && !NvlsSupports(dtype, op))) {
        return cudaErrorInvalidValue;
    }
    ZcParams p;
    p.comm = c;
    p.send = static_cast<const char*>(send);
    p.recv = static_cast<char*>(recv);
    p.bytes = bytes;
    p.func = func;
    p.op = op;
    p.scale = scale;
    if (func == 3) return launch_zc<kF32, kSum>(p, nctas, stream);  // data movement only
    const int o = (op == kAvg) ? kSum : op;
#define ZC_CASE(D, O) \
    if (dtype == D && o == O) return launch_zc<D, O>(p, nctas, stream);
    ZC_CASE(kF32, kSum)
    ZC_CASE(kF64, kSum)
    ZC_CASE(kBF16, kSum)
    ZC_CASE(kBF16, kMax)
    ZC_CASE(kBF16, kMin)
    ZC_CASE(kF16, kSum)
    ZC_CASE(kF16, kMax)
    ZC_CASE(kF16, kMin)
    ZC_CASE(kI32, kSum)
    ZC_CASE(kI32, kMax)
    ZC_CASE(kI32, kMin)
    ZC_CASE(kI64, kSum)
    ZC_CASE(kI64, kMax)
    ZC_CASE(kI64, kMin)
#undef ZC_CASE
    return cudaErrorNotSupported;
}

bool NvlsSupports(int dtype, int op) {
    using namespace dev;
    if (op == kAvg) op = kSum;
    switch (dtype) {
    case kF32:
    case kF64: return op == kSum;
    case kBF16:
    case kF16:
    case kI32:
    case kI64: return op == kSum || op == kMax || op == kMin;
    default: return false;
    }
}

cudaError_t LaunchNvls(const DevComm& c, int func, const void* src, void* dst, unsigned long long count, int dtype,
                       int op, int root, float scale, unsigned long long chunk, unsigned long long slot_bytes,
                       int nslots, int nctas, cudaStream_t stream) {
    using namespace dev;
    const bool per_rank = func == 3 || func == 4;  // a slot holds one chunk of every rank's block
    if (c.nvls_mc == nullptr || nctas <= 0 || nctas > kMaxCtas || nslots < (func == 4 ? 3 : 2) || chunk == 0 ||
        (chunk & 15) != 0 || (per_rank ? chunk * (unsigned long long)c.nranks : chunk) > slot_bytes ||
        (slot_bytes & 15) != 0 || (size_t)nslots * slot_bytes > c.nvls_bytes || func < 1 || func > 4) {
        return cudaErrorInvalidValue;
    }
    if ((func == 2 || func == 4) && !NvlsSupports(dtype, op)) return cudaErrorNotSupported;
    NvlsParams p;
    p.comm = c;
    p.src = src;
    p.dst = dst;
    p.bytes = count * (unsigned long long)dtype_size(dtype);
    p.chunk = chunk;
    p.slot_bytes = slot_bytes;
    p.nslots = nslots;
    p.nrounds = (int)((p.bytes + chunk - 1) / chunk);
    if (p.nrounds == 0) p.nrounds = 1;
    p.func = func;
    p.op = op;
    p.root = root;
    p.scale = scale;
    if (func == 1 || func == 3) return launch_t<kF32, kSum>(p, nctas, stream);  // data movement only
    const int o = (op == kAvg) ? kSum : op;
#define NV_CASE(D, O) \
    if (dtype == D && o == O) return launch_t<D, O>(p, nctas, stream);
    NV_CASE(kF32, kSum)
    NV_CASE(kF64, kSum)
    NV_CASE(kBF16, kSum)
    NV_CASE(kBF16, kMax)
    NV_CASE(kBF16, kMin)
    NV_CASE(kF16, kSum)
    NV_CASE(kF16, kMax)
    NV_CASE(kF16, kMin)
    NV_CASE(kI32, kSum)
    NV_CASE(kI32, kMax)
    NV_CASE(kI32, kMin)
    NV_CASE(kI64, kSum)
    NV_CASE(kI64, kMax)
    NV_CASE(kI64, kMin)
#undef NV_CASE
    return cudaErrorNotSupported;
}

}  // namespace bccl
