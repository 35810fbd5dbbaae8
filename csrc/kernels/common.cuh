// Device primitives shared by the collective kernels (sm_100a only).
//
//  * cross-GPU ordering: st.release.sys / ld.acquire.sys on flags in peer-mapped memory;
//  * bounded waits: every spin reads %globaltimer and gives up after DevComm::timeout_ns
//    (or when the host raises the abort word), records who waited on whom in the
//    host-mapped ErrorRecord and returns false. Nothing here traps or spins forever;
//  * dtype traits: bf16/fp16 are reduced in fp32 and rounded once; integer SUM wraps like
//    two's complement; AVG divides the final value by the rank count (integer division
//    for integer types), matching the reference's ApplyAverage
//    (OriginCCL src/utils.cpp:372-410).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "device/dev_types.h"

namespace bccl {
namespace dev {

enum DT : int { kF32 = 0, kF64 = 1, kI32 = 2, kI64 = 3, kBF16 = 4, kF16 = 5 };
enum OP : int { kSum = 0, kMax = 1, kMin = 2, kAvg = 3 };

// ---------------------------------------------------------------- PTX wrappers

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void st_relaxed_sys_flag(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint64_t ld_relaxed_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Acquire fence at system scope (turns a preceding relaxed read into an acquire pattern).
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Orders accesses made through different virtual aliases of the same memory (the
// multicast and the unicast view of an NVLS buffer).
__device__ __forceinline__ void fence_proxy_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

__device__ __forceinline__ uint4 ld_cg(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ uint4 ld_nc(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ void st_cg(void* p, const uint4& v) { __stcg(reinterpret_cast<uint4*>(p), v); }

// ---------------------------------------------------------------- tracing

// Appends one record when tracing is on (one thread per call site).
__device__ __forceinline__ void trace(const DevComm& c, int group, int event, int round) {
    if (c.trace == nullptr) return;
    unsigned int i = atomicAdd(c.trace_count, 1u);
    if (i >= c.trace_cap) return;
    TraceRecord r;
    r.t_ns = globaltimer();
    r.cta = blockIdx.x;
    r.group = (unsigned short)group;
    r.event = (unsigned short)event;
    r.round = (unsigned int)round;
    r.kernel = c.kernel_serial;
    c.trace[i] = r;
}

// ---------------------------------------------------------------- flags, waits, barriers

__device__ __forceinline__ uint64_t* barrier_flag(char* uc_base, int cta, int src) {
    return reinterpret_cast<uint64_t*>(uc_base + kBarrierFlagsOff) + (size_t)cta * kMaxRanks + src;
}

__device__ __forceinline__ void record_error(const DevComm& c, int code, int peer, int phase, uint64_t seq,
                                             uint64_t waited) {
    if (atomicCAS(&c.err->code, 0, code) == 0) {
        c.err->rank = c.rank;
        c.err->cta = blockIdx.x;
        c.err->peer = peer;
        c.err->phase = phase;
        c.err->seq = seq;
        c.err->waited_ns = waited;
        __threadfence_system();
    }
}

constexpr uint64_t kAbortCheckAfterNs = 1000000ull;

// Spin until *flag >= target. Returns false (and records the error) on timeout or abort.
// Polling uses relaxed loads with a short sleep between them (an acquire load per poll
// invalidates the SM's L1 and stalls its memory pipeline, which slows every other warp of
// the CTA); a single acquire fence follows the successful read.
__device__ __forceinline__ bool wait_flag_geq(const DevComm& c, const uint64_t* flag, uint64_t target, int peer,
                                              int phase) {
    if (ld_relaxed_sys(flag) >= target) {
        fence_acq_rel_sys();
        return true;
    }
    const uint64_t t0 = globaltimer();
    uint32_t iter = 0;
    for (;;) {
        if (!c.spin_wait) __nanosleep(iter < 64 ? 32 : 256);
        if (ld_relaxed_sys(flag) >= target) {
            fence_acq_rel_sys();
            return true;
        }
        if ((++iter & 63u) == 0) {
            const uint64_t waited = globaltimer() - t0;
            // The abort word is host memory: a read crosses PCIe, and when the link has gone
            // idle its wake-up stalls the reading thread for hundreds of microseconds. Only
            // waits that already took over 1 ms look at it.
            if (waited > kAbortCheckAfterNs && *c.abort != 0) {
                record_error(c, kDevAborted, peer, phase, target, waited);
                return false;
            }
            if (waited > c.timeout_ns) {
                record_error(c, kDevTimeout, peer, phase, target, waited);
                return false;
            }
        }
    }
}

// All-to-all barrier between CTA `blockIdx.x` of every rank, value `seq` (monotonic).
// Every thread's prior global writes (local and remote) are ordered before the flags by
// bar.sync + the releasing thread's system-scope fence; the acquiring threads' bar.sync
// orders the flags before every thread's later reads.
__device__ __forceinline__ bool cta_barrier(const DevComm& c, uint64_t seq, int phase) {
    __syncthreads();
    const int t = threadIdx.x;
    bool ok = true;
    if (t < c.nranks && t != c.rank) {
        st_release_sys(barrier_flag(c.uc[t], blockIdx.x, c.rank), seq);
        ok = wait_flag_geq(c, barrier_flag(c.uc[c.rank], blockIdx.x, t), seq, t, phase);
    }
    return __syncthreads_and(ok) != 0;
}

// Called by every CTA once at the end of a launch: the last CTA advances the device-side
// counters so the next launch (possibly a CUDA-graph replay) starts from fresh values.
__device__ __forceinline__ void finish_launch(const DevComm& c, uint64_t rounds, uint64_t barriers,
                                              uint64_t nvls_rounds, uint64_t ring_msgs = 0, uint64_t ll = 0) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        unsigned prev = atomicAdd(&c.state->done_ctas, 1u);
        if (prev == gridDim.x - 1) {
            c.state->round_seq += rounds;
            c.state->barrier_seq += barriers;
            c.state->nvls_round_seq += nvls_rounds;
            c.state->ring_seq += ring_msgs;
            c.state->ll_seq += ll;
            c.state->done_ctas = 0;
            __threadfence();
        }
    }
}

__device__ __forceinline__ uint64_t load_state_u64(const unsigned long long* p) {
    return *reinterpret_cast<const volatile unsigned long long*>(p);
}

// ---------------------------------------------------------------- dtype traits

template <int D> struct Ty;
template <> struct Ty<kF32> {
    using Bits = uint32_t;
    using Acc = float;
    static __device__ __forceinline__ Acc load(Bits b) { return __uint_as_float(b); }
    static __device__ __forceinline__ Bits store(Acc a) { return __float_as_uint(a); }
};
template <> struct Ty<kF64> {
    using Bits = unsigned long long;
    using Acc = double;
    static __device__ __forceinline__ Acc load(Bits b) { return __longlong_as_double((long long)b); }
    static __device__ __forceinline__ Bits store(Acc a) { return (Bits)__double_as_longlong(a); }
};
template <> struct Ty<kI32> {
    using Bits = uint32_t;
    using Acc = int32_t;
    static __device__ __forceinline__ Acc load(Bits b) { return (int32_t)b; }
    static __device__ __forceinline__ Bits store(Acc a) { return (uint32_t)a; }
};
template <> struct Ty<kI64> {
    using Bits = unsigned long long;
    using Acc = long long;
    static __device__ __forceinline__ Acc load(Bits b) { return (long long)b; }
    static __device__ __forceinline__ Bits store(Acc a) { return (Bits)a; }
};
template <> struct Ty<kBF16> {
    using Bits = unsigned short;
    using Acc = float;
    static __device__ __forceinline__ Acc load(Bits b) { return __uint_as_float(((uint32_t)b) << 16); }
    static __device__ __forceinline__ Bits store(Acc a) { return __bfloat16_as_ushort(__float2bfloat16_rn(a)); }
};
template <> struct Ty<kF16> {
    using Bits = unsigned short;
    using Acc = float;
    static __device__ __forceinline__ Acc load(Bits b) { return __half2float(__ushort_as_half(b)); }
    static __device__ __forceinline__ Bits store(Acc a) { return __half_as_ushort(__float2half_rn(a)); }
};

template <typename Acc>
__device__ __forceinline__ Acc combine(int op, Acc a, Acc b) {
    if (op == kMax) return a < b ? b : a;
    if (op == kMin) return b < a ? b : a;
    return a + b;
}
template <>
__device__ __forceinline__ int32_t combine<int32_t>(int op, int32_t a, int32_t b) {
    if (op == kMax) return a < b ? b : a;
    if (op == kMin) return b < a ? b : a;
    return (int32_t)((uint32_t)a + (uint32_t)b);
}
template <>
__device__ __forceinline__ long long combine<long long>(int op, long long a, long long b) {
    if (op == kMax) return a < b ? b : a;
    if (op == kMin) return b < a ? b : a;
    return (long long)((unsigned long long)a + (unsigned long long)b);
}

// Final transform: AVG divides by the rank count, then the fused scale (floating only).
template <typename Acc>
__device__ __forceinline__ Acc epilogue(int op, Acc a, int nranks, float scale) {
    if (op == kAvg) a = a / (Acc)nranks;
    if (scale != 1.0f) a = a * (Acc)scale;
    return a;
}
template <>
__device__ __forceinline__ int32_t epilogue<int32_t>(int op, int32_t a, int nranks, float) {
    return op == kAvg ? a / nranks : a;
}
template <>
__device__ __forceinline__ long long epilogue<long long>(int op, long long a, int nranks, float) {
    return op == kAvg ? a / (long long)nranks : a;
}

template <int D>
union V16 {
    uint4 u;
    typename Ty<D>::Bits b[16 / sizeof(typename Ty<D>::Bits)];
};

// 16 bytes <-> E accumulators, written per type with word operations so that the values
// stay in registers.
template <int D> struct Vec;
template <> struct Vec<kF32> {
    static constexpr int E = 4;
    static __device__ __forceinline__ void unpack(const uint4& u, float (&a)[4]) {
        a[0] = __uint_as_float(u.x); a[1] = __uint_as_float(u.y); a[2] = __uint_as_float(u.z); a[3] = __uint_as_float(u.w);
    }
    static __device__ __forceinline__ uint4 pack(const float (&a)[4]) {
        return make_uint4(__float_as_uint(a[0]), __float_as_uint(a[1]), __float_as_uint(a[2]), __float_as_uint(a[3]));
    }
};
template <> struct Vec<kI32> {
    static constexpr int E = 4;
    static __device__ __forceinline__ void unpack(const uint4& u, int32_t (&a)[4]) {
        a[0] = (int32_t)u.x; a[1] = (int32_t)u.y; a[2] = (int32_t)u.z; a[3] = (int32_t)u.w;
    }
    static __device__ __forceinline__ uint4 pack(const int32_t (&a)[4]) {
        return make_uint4((uint32_t)a[0], (uint32_t)a[1], (uint32_t)a[2], (uint32_t)a[3]);
    }
};
template <> struct Vec<kF64> {
    static constexpr int E = 2;
    static __device__ __forceinline__ void unpack(const uint4& u, double (&a)[2]) {
        a[0] = __hiloint2double((int)u.y, (int)u.x); a[1] = __hiloint2double((int)u.w, (int)u.z);
    }
    static __device__ __forceinline__ uint4 pack(const double (&a)[2]) {
        return make_uint4((uint32_t)__double2loint(a[0]), (uint32_t)__double2hiint(a[0]),
                          (uint32_t)__double2loint(a[1]), (uint32_t)__double2hiint(a[1]));
    }
};
template <> struct Vec<kI64> {
    static constexpr int E = 2;
    static __device__ __forceinline__ void unpack(const uint4& u, long long (&a)[2]) {
        a[0] = (long long)(((unsigned long long)u.y << 32) | u.x);
        a[1] = (long long)(((unsigned long long)u.w << 32) | u.z);
    }
    static __device__ __forceinline__ uint4 pack(const long long (&a)[2]) {
        return make_uint4((uint32_t)a[0], (uint32_t)((unsigned long long)a[0] >> 32), (uint32_t)a[1],
                          (uint32_t)((unsigned long long)a[1] >> 32));
    }
};
template <> struct Vec<kBF16> {
    static constexpr int E = 8;
    static __device__ __forceinline__ void unpack(const uint4& u, float (&a)[8]) {
        a[0] = __uint_as_float(u.x << 16); a[1] = __uint_as_float(u.x & 0xffff0000u);
        a[2] = __uint_as_float(u.y << 16); a[3] = __uint_as_float(u.y & 0xffff0000u);
        a[4] = __uint_as_float(u.z << 16); a[5] = __uint_as_float(u.z & 0xffff0000u);
        a[6] = __uint_as_float(u.w << 16); a[7] = __uint_as_float(u.w & 0xffff0000u);
    }
    static __device__ __forceinline__ uint32_t pk(float lo, float hi) {
        __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    static __device__ __forceinline__ uint4 pack(const float (&a)[8]) {
        return make_uint4(pk(a[0], a[1]), pk(a[2], a[3]), pk(a[4], a[5]), pk(a[6], a[7]));
    }
};
template <> struct Vec<kF16> {
    static constexpr int E = 8;
    static __device__ __forceinline__ float2 up(uint32_t w) {
        __half2 h = *reinterpret_cast<__half2*>(&w);
        return __half22float2(h);
    }
    static __device__ __forceinline__ void unpack(const uint4& u, float (&a)[8]) {
        float2 f;
        f = up(u.x); a[0] = f.x; a[1] = f.y;
        f = up(u.y); a[2] = f.x; a[3] = f.y;
        f = up(u.z); a[4] = f.x; a[5] = f.y;
        f = up(u.w); a[6] = f.x; a[7] = f.y;
    }
    static __device__ __forceinline__ uint32_t pk(float lo, float hi) {
        __half2 h = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    static __device__ __forceinline__ uint4 pack(const float (&a)[8]) {
        return make_uint4(pk(a[0], a[1]), pk(a[2], a[3]), pk(a[4], a[5]), pk(a[6], a[7]));
    }
};

// ---------------------------------------------------------------- cooperative copy / reduce

// Copies `bytes` from src to dst with the whole CTA. 16-byte vectors when both pointers
// are aligned, bytes otherwise. `cg_src` reads bypass L1 (data written by another GPU).
__device__ __forceinline__ void cta_copy(void* dst, const void* src, size_t bytes, bool cg_src) {
    const size_t t = threadIdx.x, nt = blockDim.x;
    char* d = static_cast<char*>(dst);
    const char* s = static_cast<const char*>(src);
    if (((reinterpret_cast<uintptr_t>(d) | reinterpret_cast<uintptr_t>(s)) & 15) == 0) {
        const size_t nv = bytes >> 4;
        size_t i = t;
        for (; i + 3 * nt < nv; i += 4 * nt) {
            uint4 v0 = cg_src ? ld_cg(s + (i << 4)) : *reinterpret_cast<const uint4*>(s + (i << 4));
            uint4 v1 = cg_src ? ld_cg(s + ((i + nt) << 4)) : *reinterpret_cast<const uint4*>(s + ((i + nt) << 4));
            uint4 v2 = cg_src ? ld_cg(s + ((i + 2 * nt) << 4)) : *reinterpret_cast<const uint4*>(s + ((i + 2 * nt) << 4));
            uint4 v3 = cg_src ? ld_cg(s + ((i + 3 * nt) << 4)) : *reinterpret_cast<const uint4*>(s + ((i + 3 * nt) << 4));
            st_cg(d + (i << 4), v0);
            st_cg(d + ((i + nt) << 4), v1);
            st_cg(d + ((i + 2 * nt) << 4), v2);
            st_cg(d + ((i + 3 * nt) << 4), v3);
        }
        for (; i < nv; i += nt) st_cg(d + (i << 4), cg_src ? ld_cg(s + (i << 4)) : *reinterpret_cast<const uint4*>(s + (i << 4)));
        for (size_t j = (nv << 4) + t; j < bytes; j += nt) d[j] = cg_src ? (char)__ldcg(reinterpret_cast<const signed char*>(s + j)) : s[j];
    } else {
        for (size_t j = t; j < bytes; j += nt) d[j] = cg_src ? (char)__ldcg(reinterpret_cast<const signed char*>(s + j)) : s[j];
    }
}

// dst[i] = epilogue(reduce_p srcs[p][i]) over `bytes` bytes, p in [0, n) in rank order
// (identical order on every rank, so every rank produces bit-identical results).
// srcs[p] with (cg_mask >> p) & 1 are read with ld.cg (written by another GPU).
// NS bounds n (the register arrays' size); with NS <= 4 every thread keeps two vectors' loads
// in flight (2n loads), which a CTA needs to approach its share of memory bandwidth when n is
// small, while NS = 8 keeps one (8 loads) to stay within the register budget.
template <int D, int O, int NS>
__device__ __noinline__ void cta_reduce(void* dst, const void* const* srcs, int n, unsigned cg_mask, size_t bytes,
                                        int nranks, float scale) {
    using T = Ty<D>;
    using Bits = typename T::Bits;
    using Acc = typename T::Acc;
    using V = Vec<D>;
    constexpr int E = V::E;
    constexpr int U = NS <= 4 ? 2 : 1;
    const size_t t = threadIdx.x, nt = blockDim.x;
    // Source pointers into registers (static indices below); unused slots alias source 0.
    const char* sp[NS];
#pragma unroll
    for (int p = 0; p < NS; ++p) sp[p] = static_cast<const char*>(srcs[p < n ? p : 0]);
    uintptr_t mis = reinterpret_cast<uintptr_t>(dst);
#pragma unroll
    for (int p = 0; p < NS; ++p) mis |= reinterpret_cast<uintptr_t>(sp[p]);
    const size_t nv = ((mis & 15) == 0) ? (bytes >> 4) : 0;
    const bool post = (O == kAvg) || scale != 1.0f;
    size_t i = t;
    for (; i + (U - 1) * nt < nv; i += U * nt) {
        uint4 w[U][NS];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const size_t off = (i + u * nt) << 4;
#pragma unroll
            for (int p = 0; p < NS; ++p) {
                if (p < n)
                    w[u][p] = ((cg_mask >> p) & 1) ? ld_cg(sp[p] + off) : *reinterpret_cast<const uint4*>(sp[p] + off);
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
            st_cg(static_cast<char*>(dst) + ((i + u * nt) << 4), V::pack(acc));
        }
    }
    for (; i < nv; i += nt) {  // at most one vector per thread left
        const size_t off = i << 4;
        Acc acc[E], x[E];
        V::unpack(((cg_mask & 1u) ? ld_cg(sp[0] + off) : *reinterpret_cast<const uint4*>(sp[0] + off)), acc);
#pragma unroll
        for (int p = 1; p < NS; ++p) {
            if (p < n) {
                V::unpack(((cg_mask >> p) & 1) ? ld_cg(sp[p] + off) : *reinterpret_cast<const uint4*>(sp[p] + off), x);
#pragma unroll
                for (int e = 0; e < E; ++e) acc[e] = combine<Acc>(O, acc[e], x[e]);
            }
        }
        if (post) {
#pragma unroll
            for (int e = 0; e < E; ++e) acc[e] = epilogue<Acc>(O, acc[e], nranks, scale);
        }
        st_cg(static_cast<char*>(dst) + off, V::pack(acc));
    }
    // Ragged tail (or a misaligned buffer): one element at a time.
    const size_t done = nv << 4;
    const size_t nelem = (bytes - done) / sizeof(Bits);
    for (size_t j = t; j < nelem; j += nt) {
        const size_t off = done + j * sizeof(Bits);
        Acc acc = Acc(0);
#pragma unroll
        for (int p = 0; p < NS; ++p) {
            if (p < n) {
                const Bits* e = reinterpret_cast<const Bits*>(sp[p] + off);
                Bits b = ((cg_mask >> p) & 1) ? __ldcg(e) : *e;
                acc = (p == 0) ? T::load(b) : combine<Acc>(O, acc, T::load(b));
            }
        }
        *reinterpret_cast<Bits*>(static_cast<char*>(dst) + off) = T::store(epilogue<Acc>(O, acc, nranks, scale));
    }
}

template <int D, int O>
__device__ __forceinline__ void cta_reduce_n(void* dst, const void* const* srcs, int n, unsigned cg_mask, size_t bytes,
                                             int nranks, float scale) {
    if (n <= 4) cta_reduce<D, O, 4>(dst, srcs, n, cg_mask, bytes, nranks, scale);
    else cta_reduce<D, O, kMaxRanks>(dst, srcs, n, cg_mask, bytes, nranks, scale);
}

template <int D>
__device__ __forceinline__ void cta_reduce_op(int op, void* dst, const void* const* srcs, int n, unsigned cg_mask,
                                              size_t bytes, int nranks, float scale) {
    switch (op) {
    case kSum: cta_reduce_n<D, kSum>(dst, srcs, n, cg_mask, bytes, nranks, scale); break;
    case kMax: cta_reduce_n<D, kMax>(dst, srcs, n, cg_mask, bytes, nranks, scale); break;
    case kMin: cta_reduce_n<D, kMin>(dst, srcs, n, cg_mask, bytes, nranks, scale); break;
    case kAvg: cta_reduce_n<D, kAvg>(dst, srcs, n, cg_mask, bytes, nranks, scale); break;
    default: break;
    }
}

// Runtime dtype/op dispatch.
__device__ __forceinline__ void cta_reduce_any(int dtype, void* dst, const void* const* srcs, int n, unsigned cg_mask,
                                               size_t bytes, int op, int nranks, float scale) {
    switch (dtype) {
    case kF32: cta_reduce_op<kF32>(op, dst, srcs, n, cg_mask, bytes, nranks, scale); break;
    case kF64: cta_reduce_op<kF64>(op, dst, srcs, n, cg_mask, bytes, nranks, scale); break;
    case kI32: cta_reduce_op<kI32>(op, dst, srcs, n, cg_mask, bytes, nranks, scale); break;
    case kI64: cta_reduce_op<kI64>(op, dst, srcs, n, cg_mask, bytes, nranks, scale); break;
    case kBF16: cta_reduce_op<kBF16>(op, dst, srcs, n, cg_mask, bytes, nranks, scale); break;
    case kF16: cta_reduce_op<kF16>(op, dst, srcs, n, cg_mask, bytes, nranks, scale); break;
    default: break;
    }
}

__host__ __device__ __forceinline__ int dtype_size(int dtype) {
    return (dtype == kF64 || dtype == kI64) ? 8 : (dtype == kBF16 || dtype == kF16) ? 2 : 4;
}

__host__ __device__ __forceinline__ size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace dev
}  // namespace bccl
