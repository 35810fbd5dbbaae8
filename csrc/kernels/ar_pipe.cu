// Software-pipelined AllReduce for large payloads.
//
// All CTAs run the same phase; CTA b owns piece b of every round on every rank, and one
// per-CTA barrier (flags in peer memory) closes each iteration. Iteration t does
//   ONESHOT: A = push round t's piece to every peer's inbox slot
//            B = reduce round t-1: own input + N-1 inbox slots -> output
//   TWOSHOT: A = push shard q of round t to peer q's inbox slot
//            B = reduce own shard of round t-1 -> own output, and push it into every peer's
//                gather slot
//            C = copy round t-2's peer shards out of the local gather slot
//   NVLS:    A = copy round t's piece into the local NVLS slot
//            B = multimem.ld_reduce + multimem.st of the own shard of round t-1
//            C = copy round t-2 out of the local NVLS slot
// then fence + signal + wait (barrier t). The phase that crosses NVLink runs on one warp
// group while the local phases run on the other, so copies overlap link traffic; both
// groups finish before the single fence of the iteration. B(t-1) only needs A(t-1) from every rank and C(t-2)
// only needs B(t-2) from every rank, both proven by barrier t-1. NVLink writes are issued
// first in an iteration, so by the time the CTA fences (after its local work) they have
// mostly drained: a system-scope fence costs little when it is not waiting on fresh
// traffic, and a lot when it is (measured: a pipeline that fenced right behind its own
// NVLink stream ran 5-10x slower).
// Slots form a ring of S >= 3 per kind, indexed by a device-side round counter; a slot is
// rewritten at least two barriers after its last reader finished, and a completed launch
// implies every rank finished all its work (the last iteration's work precedes the last
// barrier), so launches of any kind can follow each other.
#include "kernels/common.cuh"
#include "kernels/launch.h"

namespace bccl {
namespace dev {
namespace {

constexpr int kThreads = 512;
constexpr int kUnroll = 4;

struct PipeParams {
    DevComm comm;
    const void* src;
    void* dst;
    unsigned long long bytes;
    unsigned long long chunk;       // bytes per round (multiple of 16 * nranks)
    unsigned long long slot_bytes;  // NVLS: bytes per slot (>= chunk); TWOSHOT: per-source inbox slot (>= shard)
    int nrounds;
    int nslots;
    int dtype;
    int op;
    float scale;
    int nvls;   // PipeKind
    int lag;    // barrier lag L (1 or 2): iteration t waits for barrier t-L; needs nslots >= 2L+1
    // Hybrid launch (hyb_ctas > 0): CTAs [0, hyb_ctas) run NVLS on bytes [0, hyb_bytes) in
    // hyb_rounds rounds of hyb_chunk (NVLS slots of hyb_slot bytes), the remaining CTAs run
    // `nvls` (two-shot) on [hyb_bytes, bytes) with chunk / slot_bytes / nrounds above. The two
    // parts share nothing but the launch: their staging buffers, round counters and per-CTA
    // barriers are disjoint.
    int hyb_ctas;
    int hyb_rounds;
    unsigned long long hyb_bytes;
    unsigned long long hyb_chunk;
    unsigned long long hyb_slot;
};


// Group copy, `kUnroll` 16-byte vectors in flight per thread.
__device__ __forceinline__ void grp_copy(char* d, const char* s, size_t bytes, int tid, int nt, bool cg) {
    if (((reinterpret_cast<uintptr_t>(d) | reinterpret_cast<uintptr_t>(s)) & 15) == 0) {
        const size_t nv = bytes >> 4;
        size_t i = tid;
        for (; i + (kUnroll - 1) * (size_t)nt < nv; i += kUnroll * (size_t)nt) {
            uint4 v[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const char* p = s + ((i + u * (size_t)nt) << 4);
                v[u] = cg ? ld_cg(p) : *reinterpret_cast<const uint4*>(p);
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) st_cg(d + ((i + u * (size_t)nt) << 4), v[u]);
        }
        for (; i < nv; i += nt) {
            const char* p = s + (i << 4);
            st_cg(d + (i << 4), cg ? ld_cg(p) : *reinterpret_cast<const uint4*>(p));
        }
        for (size_t j = (nv << 4) + tid; j < bytes; j += nt) d[j] = s[j];
    } else {
        for (size_t j = tid; j < bytes; j += nt) d[j] = cg ? (char)__ldcg(reinterpret_cast<const signed char*>(s + j)) : s[j];
    }
}

// Loads each 16-byte vector once and stores it to every destination in outs[0..no).
__device__ __forceinline__ void grp_push_multi(char* const* outs, int no, const char* src, size_t bytes, int tid,
                                               int nt) {
    char* op[kMaxRanks];
#pragma unroll
    for (int q = 0; q < kMaxRanks; ++q) op[q] = outs[q < no ? q : 0];
    uintptr_t mis = reinterpret_cast<uintptr_t>(src);
#pragma unroll
    for (int q = 0; q < kMaxRanks; ++q) mis |= reinterpret_cast<uintptr_t>(op[q]);
    const size_t nv = (mis & 15) ? 0 : (bytes >> 4);
    size_t i = tid;
    for (; i + (kUnroll - 1) * (size_t)nt < nv; i += kUnroll * (size_t)nt) {
        uint4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) v[u] = *reinterpret_cast<const uint4*>(src + ((i + u * (size_t)nt) << 4));
#pragma unroll
        for (int q = 0; q < kMaxRanks; ++q) {
            if (q < no) {
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) st_cg(op[q] + ((i + u * (size_t)nt) << 4), v[u]);
            }
        }
    }
    for (; i < nv; i += nt) {
        const uint4 v = *reinterpret_cast<const uint4*>(src + (i << 4));
        for (int q = 0; q < no; ++q) st_cg(op[q] + (i << 4), v);
    }
    for (size_t j = (nv << 4) + tid; j < bytes; j += nt) {
        const char b = src[j];
        for (int q = 0; q < no; ++q) op[q][j] = b;
    }
}

// ---- multimem (16-byte) -------------------------------------------------------------------
// (dtype, op) pairs with a multimem.ld_reduce form on sm_100a (checked against ptxas):
// f32 and f64 add only; bf16/f16 add (fp32 accumulation), max, min; integers add/max/min.
template <int D, int O>
struct NvlsOk {
    static constexpr bool value = (O == kSum) || (O == kAvg) ? true : (D != kF32 && D != kF64);
};
template <int D, int O> __device__ __forceinline__ uint4 mm_ld_reduce(const void* p);
#define PIPE_MM_V4(D, O, SPEC)                                                                  \
    template <> __device__ __forceinline__ uint4 mm_ld_reduce<D, O>(const void* p) {            \
        uint4 r;                                                                              \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " {%0,%1,%2,%3}, [%4];"    \
                     : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p) : "memory");       \
        return r;                                                                             \
    }
#define PIPE_MM_S32(D, O, SPEC)                                                                 \
    template <> __device__ __forceinline__ uint4 mm_ld_reduce<D, O>(const void* p) {            \
        uint4 r;                                                                              \
        const char* c = static_cast<const char*>(p);                                          \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " %0, [%1];" : "=r"(r.x) : "l"(c) : "memory");      \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " %0, [%1];" : "=r"(r.y) : "l"(c + 4) : "memory");  \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " %0, [%1];" : "=r"(r.z) : "l"(c + 8) : "memory");  \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " %0, [%1];" : "=r"(r.w) : "l"(c + 12) : "memory"); \
        return r;                                                                             \
    }
#define PIPE_MM_S64(D, O, SPEC)                                                                 \
    template <> __device__ __forceinline__ uint4 mm_ld_reduce<D, O>(const void* p) {            \
        unsigned long long a, b;                                                              \
        const char* c = static_cast<const char*>(p);                                          \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " %0, [%1];" : "=l"(a) : "l"(c) : "memory");     \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " %0, [%1];" : "=l"(b) : "l"(c + 8) : "memory"); \
        return make_uint4((unsigned)a, (unsigned)(a >> 32), (unsigned)b, (unsigned)(b >> 32));                      \
    }
PIPE_MM_V4(kF32, kSum, "add.v4.f32")
PIPE_MM_V4(kBF16, kSum, "add.acc::f32.v4.bf16x2")
PIPE_MM_V4(kBF16, kMax, "max.v4.bf16x2")
PIPE_MM_V4(kBF16, kMin, "min.v4.bf16x2")
PIPE_MM_V4(kF16, kSum, "add.acc::f32.v4.f16x2")
PIPE_MM_V4(kF16, kMax, "max.v4.f16x2")
PIPE_MM_V4(kF16, kMin, "min.v4.f16x2")
PIPE_MM_S32(kI32, kSum, "add.u32")
PIPE_MM_S32(kI32, kMax, "max.s32")
PIPE_MM_S32(kI32, kMin, "min.s32")
PIPE_MM_S64(kI64, kSum, "add.u64")
PIPE_MM_S64(kI64, kMax, "max.s64")
PIPE_MM_S64(kI64, kMin, "min.s64")
PIPE_MM_S64(kF64, kSum, "add.f64")

__device__ __forceinline__ void mm_st(void* p, const uint4& v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

template <int D>
__device__ __forceinline__ uint4 post16(uint4 u, int op, int nranks, float scale) {
    if (op != kAvg && scale == 1.0f) return u;
    using V = Vec<D>;
    typename Ty<D>::Acc a[V::E];
    V::unpack(u, a);
#pragma unroll
    for (int e = 0; e < V::E; ++e) a[e] = epilogue<typename Ty<D>::Acc>(op, a[e], nranks, scale);
    return V::pack(a);
}

// G2 body (NVLS): reduce+broadcast [lo, hi) of the slot through the multicast address.
template <int D, int O>
__device__ __forceinline__ void nvls_reduce_bcast(char* mc, size_t lo, size_t hi, int tid, int nt, int op, int nranks,
                                                  float scale) {
    constexpr int U = 8;  // the switch round trip is long: keep 8 reductions in flight per thread
    const size_t nv = (hi - lo) >> 4;  // [lo, hi) is 16-byte aligned and padded
    size_t i = tid;
    for (; i + (U - 1) * (size_t)nt < nv; i += U * (size_t)nt) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) v[u] = mm_ld_reduce<D, O>(mc + lo + ((i + u * (size_t)nt) << 4));
#pragma unroll
        for (int u = 0; u < U; ++u) mm_st(mc + lo + ((i + u * (size_t)nt) << 4), post16<D>(v[u], op, nranks, scale));
    }
    for (; i < nv; i += nt) {
        char* p = mc + lo + (i << 4);
        mm_st(p, post16<D>(mm_ld_reduce<D, O>(p), op, nranks, scale));
    }
}

// G2 body (TWOSHOT): dst = reduce(srcs[0..n)) over `bytes`, srcs[p] for p != own read with ld.cg.
template <int D, int O>
__device__ __forceinline__ void grp_reduce(char* dst, const char* const* srcs, int n, int own, size_t bytes, int tid,
                                           int nt, int nranks, float scale) {
    using V = Vec<D>;
    using Acc = typename Ty<D>::Acc;
    using Bits = typename Ty<D>::Bits;
    const char* sp[kMaxRanks];
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p) sp[p] = srcs[p < n ? p : 0];
    uintptr_t mis = reinterpret_cast<uintptr_t>(dst);
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p) mis |= reinterpret_cast<uintptr_t>(sp[p]);
    const size_t nv = (mis & 15) ? 0 : (bytes >> 4);
    const bool post = O == kAvg || scale != 1.0f;
    for (size_t i = tid; i < nv; i += nt) {
        const size_t off = i << 4;
        uint4 w[kMaxRanks];
#pragma unroll
        for (int p = 0; p < kMaxRanks; ++p)
            if (p < n) w[p] = (p == own) ? *reinterpret_cast<const uint4*>(sp[p] + off) : ld_cg(sp[p] + off);
        Acc acc[V::E], x[V::E];
        V::unpack(w[0], acc);
#pragma unroll
        for (int p = 1; p < kMaxRanks; ++p) {
            if (p < n) {
                V::unpack(w[p], x);
#pragma unroll
                for (int e = 0; e < V::E; ++e) acc[e] = combine<Acc>(O, acc[e], x[e]);
            }
        }
        if (post) {
#pragma unroll
            for (int e = 0; e < V::E; ++e) acc[e] = epilogue<Acc>(O, acc[e], nranks, scale);
        }
        st_cg(dst + off, V::pack(acc));
    }
    const size_t done = nv << 4;
    for (size_t j = done + (size_t)tid * sizeof(Bits); j < bytes; j += (size_t)nt * sizeof(Bits)) {
        Acc acc = Acc(0);
#pragma unroll
        for (int p = 0; p < kMaxRanks; ++p) {
            if (p < n) {
                const Bits* e = reinterpret_cast<const Bits*>(sp[p] + j);
                const Bits b = (p == own) ? *e : __ldcg(e);
                acc = (p == 0) ? Ty<D>::load(b) : combine<Acc>(O, acc, Ty<D>::load(b));
            }
        }
        *reinterpret_cast<Bits*>(dst + j) = Ty<D>::store(epilogue<Acc>(O, acc, nranks, scale));
    }
}

// dst_p = reduce(srcs) for every output pointer (one local, the rest in peers' memory).
template <int D, int O>
__device__ __forceinline__ void grp_reduce_multi(char* const* outs, int no, const char* const* srcs, int n, int own,
                                                 size_t bytes, int tid, int nt, int nranks, float scale) {
    using V = Vec<D>;
    using Acc = typename Ty<D>::Acc;
    using Bits = typename Ty<D>::Bits;
    const char* sp[kMaxRanks];
    char* op[kMaxRanks];
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p) {
        sp[p] = srcs[p < n ? p : 0];
        op[p] = outs[p < no ? p : 0];
    }
    uintptr_t mis = 0;
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p) mis |= reinterpret_cast<uintptr_t>(sp[p]) | reinterpret_cast<uintptr_t>(op[p]);
    const size_t nv = (mis & 15) ? 0 : (bytes >> 4);
    const bool post = O == kAvg || scale != 1.0f;
    for (size_t i = tid; i < nv; i += nt) {
        const size_t off = i << 4;
        uint4 w[kMaxRanks];
#pragma unroll
        for (int p = 0; p < kMaxRanks; ++p)
            if (p < n) w[p] = (p == own) ? *reinterpret_cast<const uint4*>(sp[p] + off) : ld_cg(sp[p] + off);
        Acc acc[V::E], x[V::E];
        V::unpack(w[0], acc);
#pragma unroll
        for (int p = 1; p < kMaxRanks; ++p) {
            if (p < n) {
                V::unpack(w[p], x);
#pragma unroll
                for (int e = 0; e < V::E; ++e) acc[e] = combine<Acc>(O, acc[e], x[e]);
            }
        }
        if (post) {
#pragma unroll
            for (int e = 0; e < V::E; ++e) acc[e] = epilogue<Acc>(O, acc[e], nranks, scale);
        }
        const uint4 res = V::pack(acc);
#pragma unroll
        for (int p = 0; p < kMaxRanks; ++p)
            if (p < no) st_cg(op[p] + off, res);
    }
    const size_t done = nv << 4;
    for (size_t j = done + (size_t)tid * sizeof(Bits); j < bytes; j += (size_t)nt * sizeof(Bits)) {
        Acc acc = Acc(0);
#pragma unroll
        for (int p = 0; p < kMaxRanks; ++p) {
            if (p < n) {
                const Bits* e = reinterpret_cast<const Bits*>(sp[p] + j);
                const Bits b = (p == own) ? *e : __ldcg(e);
                acc = (p == 0) ? Ty<D>::load(b) : combine<Acc>(O, acc, Ty<D>::load(b));
            }
        }
        const Bits out = Ty<D>::store(epilogue<Acc>(O, acc, nranks, scale));
        for (int p = 0; p < no; ++p) *reinterpret_cast<Bits*>(op[p] + j) = out;
    }
}

// TWOSHOT data region (second half of the UC data region, disjoint from the push engine):
//   inbox  [nslots][nranks][slot_bytes]   pieces pushed by the peers' stage CTAs
//   gather [nslots][nranks][slot_bytes]   reduced shards pushed by the peers' reduce CTAs
__device__ __forceinline__ char* ts_region(const DevComm& c, int owner) {
    return c.uc[owner] + kCtrlBytes + (size_t)(c.data_bytes / 2);
}

template <int D, int O>
__global__ void __launch_bounds__(kThreads, 1) ar_sched_kernel(const __grid_constant__ PipeParams p) {
    const DevComm& c = p.comm;
    const int r = c.rank, n = c.nranks;
    // This CTA's part of the launch (the whole payload unless the launch is a hybrid).
    const bool hyb_nvls = p.hyb_ctas > 0 && (int)blockIdx.x < p.hyb_ctas;
    const int kind = hyb_nvls ? kPipeNvls : p.nvls;  // kPipeTwoShot / kPipeNvls / kPipeOneShot
    const size_t part_off = (p.hyb_ctas > 0 && !hyb_nvls) ? (size_t)p.hyb_bytes : 0;
    const size_t part_bytes = hyb_nvls ? (size_t)p.hyb_bytes : (size_t)p.bytes - part_off;
    const size_t part_chunk = hyb_nvls ? (size_t)p.hyb_chunk : (size_t)p.chunk;
    const int nrounds = hyb_nvls ? p.hyb_rounds : p.nrounds;
    const int cta = (p.hyb_ctas > 0 && !hyb_nvls) ? (int)blockIdx.x - p.hyb_ctas : (int)blockIdx.x;
    const int nct = p.hyb_ctas > 0 ? (hyb_nvls ? p.hyb_ctas : (int)gridDim.x - p.hyb_ctas) : (int)gridDim.x;
    // Warp groups run their phases concurrently for NVLS (two local copies against one switch
    // phase); for the push kinds a single group measured faster.
    const bool split = kind == kPipeNvls;
    const uint64_t bar0 = load_state_u64(&c.state->barrier_seq);
    const uint64_t round0 = kind == kPipeNvls ? load_state_u64(&c.state->nvls_round_seq)
                                              : load_state_u64(&c.state->round_seq);
    const int S = p.nslots;
    const size_t sb = hyb_nvls ? (size_t)p.hyb_slot : (size_t)p.slot_bytes;
    const char* src = static_cast<const char*>(p.src) + part_off;
    char* dst = static_cast<char*>(p.dst) + part_off;
    const int depth = (kind == kPipeOneShot) ? 1 : 2;
    const int L = p.lag;
    const int iters = nrounds + depth * L;
    // Two warp groups: "net" (warps 0-7) runs the phase that crosses NVLink, "local" (warps
    // 8-15) the phases that stay in this GPU's memory; without the split both do everything.
    const int half = blockDim.x / 2;
    const bool is_net = threadIdx.x < half;
    const int gtid = split ? (is_net ? threadIdx.x : threadIdx.x - half) : threadIdx.x;
    const int gnt = split ? half : blockDim.x;
    const bool do_net = !split || is_net, do_local = !split || !is_net;
    if (threadIdx.x == 0) trace(c, 0, kTrBegin, (int)(bar0 & 0x7fffffffull));  // round field: barrier base

    // Shards and CTA pieces follow the full chunk in every round, the last (shorter) one included,
    // so CTA b owns the same bytes of a slot in every round: a slot is reused every S rounds, and
    // the per-CTA barrier that frees it only covers CTA b on the other ranks.
    const size_t full_chunk = min(part_bytes, part_chunk);
    const size_t full_shard = (kind == kPipeOneShot) ? full_chunk : round_up((full_chunk + n - 1) / n, 16);
    const size_t piece = round_up((full_shard + nct - 1) / nct, 16);
    auto geom = [&](int j, size_t* cbeg, size_t* clen, size_t* shard, size_t* s0, size_t* s1) {
        *cbeg = (size_t)j * part_chunk;
        *clen = min(part_bytes - *cbeg, part_chunk);
        *shard = full_shard;
        // One-shot: the piece is a range of the chunk itself, cut at its end; the other kinds cut
        // rank q's range q * shard + [s0, s1) at the chunk's end where they use it.
        const size_t lim = (kind == kPipeOneShot) ? *clen : full_shard;
        *s0 = min(lim, (size_t)cta * piece);
        *s1 = min(lim, *s0 + piece);
    };
    // ---- phase bodies (tid/nt are group-relative)
    auto phase_a = [&](int j, int tid, int nt) {  // stage round j
        size_t cbeg, clen, shard, s0, s1;
        geom(j, &cbeg, &clen, &shard, &s0, &s1);
        const int slot = (int)((round0 + (uint64_t)j) % (uint64_t)S);
        if (kind == kPipeOneShot) {
            if (s0 < s1) {
                char* outs[kMaxRanks];
                int no = 0;
                for (int q = 0; q < n; ++q)
                    if (q != r) outs[no++] = ts_region(c, q) + ((size_t)slot * n + r) * sb + s0;
                if (no > 0) grp_push_multi(outs, no, src + cbeg + s0, s1 - s0, tid, nt);
            }
        } else if (kind == kPipeTwoShot) {
            for (int q = 0; q < n; ++q) {
                if (q == r) continue;
                const size_t lo = min(clen, q * shard + s0), hi = min(clen, q * shard + s1);
                char* inb = ts_region(c, q) + ((size_t)slot * n + r) * sb;
                if (lo < hi) grp_copy(inb + s0, src + cbeg + lo, hi - lo, tid, nt, false);
            }
        } else {
            char* slotp = c.nvls_uc + (size_t)slot * sb;
            for (int q = 0; q < n; ++q) {
                const size_t lo = min(clen, q * shard + s0), hi = min(clen, q * shard + s1);
                if (lo < hi) grp_copy(slotp + lo, src + cbeg + lo, hi - lo, tid, nt, false);
            }
        }
    };
    auto phase_b = [&](int j, int tid, int nt) {  // reduce round j
        size_t cbeg, clen, shard, s0, s1;
        geom(j, &cbeg, &clen, &shard, &s0, &s1);
        const int slot = (int)((round0 + (uint64_t)j) % (uint64_t)S);
        if (kind == kPipeOneShot) {
            if (s0 < s1) {
                const char* srcs[kMaxRanks];
                char* mine = ts_region(c, r);
                for (int q = 0; q < n; ++q) {
                    srcs[q] = (q == r) ? src + cbeg + s0 : mine + ((size_t)slot * n + q) * sb + s0;
                }
                char* outs[1] = {dst + cbeg + s0};
                grp_reduce_multi<D, O>(outs, 1, srcs, n, r, s1 - s0, tid, nt, n, p.scale);
            }
        } else if (kind == kPipeTwoShot) {
            const size_t lo = min(clen, r * shard + s0), hi = min(clen, r * shard + s1);
            if (lo < hi) {
                const char* srcs[kMaxRanks];
                char* mine = ts_region(c, r);
                for (int q = 0; q < n; ++q)
                    srcs[q] = (q == r) ? src + cbeg + lo : mine + ((size_t)slot * n + q) * sb + s0;
                char* outs[kMaxRanks];
                int no = 0;
                outs[no++] = dst + cbeg + lo;
                for (int q = 0; q < n; ++q)
                    if (q != r) outs[no++] = ts_region(c, q) + (size_t)S * n * sb + ((size_t)slot * n + r) * sb + s0;
                grp_reduce_multi<D, O>(outs, no, srcs, n, r, hi - lo, tid, nt, n, p.scale);
            }
        } else {
            if constexpr (NvlsOk<D, O>::value) {
                const size_t padded = round_up(clen, 16);
                const size_t lo = min(padded, r * shard + s0), hi = min(padded, r * shard + s1);
                if (lo < hi) {
                    nvls_reduce_bcast<D, (O == kAvg ? kSum : O)>(c.nvls_mc + (size_t)slot * sb, lo, hi, tid, nt, p.op,
                                                                 n, p.scale);
                }
            }
        }
    };
    auto phase_c = [&](int j, int tid, int nt) {  // finish round j
        size_t cbeg, clen, shard, s0, s1;
        geom(j, &cbeg, &clen, &shard, &s0, &s1);
        const int slot = (int)((round0 + (uint64_t)j) % (uint64_t)S);
        if (kind == kPipeTwoShot) {
            const char* gather = ts_region(c, r) + (size_t)S * n * sb + (size_t)slot * n * sb;
            for (int q = 0; q < n; ++q) {
                if (q == r) continue;
                const size_t lo = min(clen, q * shard + s0), hi = min(clen, q * shard + s1);
                if (lo < hi) grp_copy(dst + cbeg + lo, gather + (size_t)q * sb + s0, hi - lo, tid, nt, true);
            }
        } else {
            const char* slotp = c.nvls_uc + (size_t)slot * sb;
            for (int q = 0; q < n; ++q) {
                const size_t lo = min(clen, q * shard + s0), hi = min(clen, q * shard + s1);
                if (lo < hi) grp_copy(dst + cbeg + lo, slotp + lo, hi - lo, tid, nt, true);
            }
        }
    };
    // Barrier k closes iteration k on every rank. Iteration t starts only once barrier t-L has
    // closed: L = 1 is the lock-step schedule; L = 2 lets a CTA run one iteration ahead of the
    // slowest CTA with its index on the other GPUs, which hides the barrier's latency behind
    // the next iteration's work (the slot ring is then 2L+1 deep, so no slot is rewritten
    // while a rank may still read it).
    auto wait_barrier = [&](int k) {
        bool w = true;
        if (threadIdx.x < n && threadIdx.x != r) {
            w = wait_flag_geq(c, barrier_flag(c.uc[r], blockIdx.x, threadIdx.x), bar0 + (uint64_t)k + 1,
                              threadIdx.x, k);
        }
        w = __syncthreads_and(w) != 0;
        if (threadIdx.x == 0) trace(c, 0, kTrBarrier, k);
        return w;
    };
    bool ok = true;
    for (int t = 0; t < iters && ok; ++t) {
        if (t >= L && !(ok = wait_barrier(t - L))) break;
        const bool has_a = t < nrounds, has_b = t >= L && t - L < nrounds;
        const bool has_c = depth == 2 && t >= 2 * L && t - 2 * L < nrounds;
        // Which group runs what: NVLS crosses NVLink in B (multimem); two-shot and one-shot
        // cross it in A (pushes). The other phases run on the local group.
        if (kind == kPipeNvls) {
            if (do_net && has_b) phase_b(t - L, gtid, gnt);
            if (do_local && has_a) phase_a(t, gtid, gnt);
            if (do_local && has_c) phase_c(t - 2 * L, gtid, gnt);
        } else {
            if (do_net && has_a) phase_a(t, gtid, gnt);
            if (do_local && has_b) phase_b(t - L, gtid, gnt);
            if (do_local && has_c) phase_c(t - 2 * L, gtid, gnt);
        }
        // ---- barrier t: both groups' writes are issued; fence + signal (the wait comes L
        // iterations later).
        __syncthreads();
        if (threadIdx.x == 0) trace(c, 0, kTrStaged, t);  // this CTA's phases of iteration t are issued
        if (threadIdx.x < n && threadIdx.x != r) {
            fence_acq_rel_sys();
            st_relaxed_sys_flag(barrier_flag(c.uc[threadIdx.x], blockIdx.x, r), bar0 + (uint64_t)t + 1);
        }
    }
    // The launch ends with every rank's last iteration closed: a completed launch implies every
    // rank finished all its phases, whatever kind of launch comes next.
    if (ok) ok = wait_barrier(iters - 1);
    if (threadIdx.x == 0) trace(c, 0, kTrEnd, iters);
    // Every CTA passes the launch-wide totals (the last one to finish applies them).
    if (p.hyb_ctas > 0) {
        finish_launch(c, (uint64_t)p.nrounds, (uint64_t)max(p.nrounds, p.hyb_rounds) + 2 * p.lag, (uint64_t)p.hyb_rounds);
    } else if (p.nvls == kPipeNvls) {
        finish_launch(c, 0, (uint64_t)p.nrounds + 2 * p.lag, (uint64_t)p.nrounds);
    } else {
        finish_launch(c, (uint64_t)p.nrounds, (uint64_t)p.nrounds + (p.nvls == kPipeOneShot ? 1 : 2) * p.lag, 0);
    }
}

template <int D, int O>
cudaError_t launch_t(const PipeParams& p, int nctas, cudaStream_t s) {
    ar_sched_kernel<D, O><<<nctas, kThreads, 0, s>>>(p);
    return cudaGetLastError();
}

template <int D>
cudaError_t launch_op(const PipeParams& p, int nctas, cudaStream_t s) {
    switch (p.op) {
    case kSum: return launch_t<D, kSum>(p, nctas, s);
    case kAvg: return launch_t<D, kAvg>(p, nctas, s);  // AVG = SUM, then divide in the epilogue
    case kMax: return launch_t<D, kMax>(p, nctas, s);
    case kMin: return launch_t<D, kMin>(p, nctas, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace
}  // namespace dev

cudaError_t LaunchAllReducePipe(const DevComm& c, int kind, const void* src, void* dst, unsigned long long count,
                                int dtype, int op, float scale, unsigned long long chunk, unsigned long long slot_bytes,
                                int nslots, int nctas, cudaStream_t stream, int lag) {
    using namespace dev;
    const bool nvls = kind == kPipeNvls;
    if (nctas < 1 || nctas > kMaxCtas || lag < 1 || lag > 2 || nslots < 2 * lag + 1 || chunk == 0 ||
        (chunk % (16ull * c.nranks)) != 0) {
        return cudaErrorInvalidValue;
    }
    if (kind == kPipeOneShot && ((size_t)nslots * c.nranks * slot_bytes > c.data_bytes / 2 || slot_bytes < chunk)) {
        return cudaErrorInvalidValue;
    }
    if (nvls && (c.nvls_mc == nullptr || !NvlsSupports(dtype, op) || (size_t)nslots * slot_bytes > c.nvls_bytes ||
                 slot_bytes < chunk)) {
        return cudaErrorInvalidValue;
    }
    if (kind == kPipeTwoShot && ((size_t)nslots * 2 * c.nranks * slot_bytes > c.data_bytes / 2 || slot_bytes * c.nranks < chunk)) {
        return cudaErrorInvalidValue;
    }
    PipeParams p;
    p.comm = c;
    p.src = src;
    p.dst = dst;
    p.bytes = count * (unsigned long long)dtype_size(dtype);
    p.chunk = chunk;
    p.slot_bytes = slot_bytes;
    p.nrounds = (int)((p.bytes + chunk - 1) / chunk);
    if (p.nrounds == 0) p.nrounds = 1;
    p.nslots = nslots;
    p.dtype = dtype;
    p.op = op;
    p.scale = scale;
    p.nvls = kind == kPipeNvls ? 1 : (kind == kPipeOneShot ? 2 : 0);
    p.lag = lag;
    p.hyb_ctas = 0;
    p.hyb_rounds = 0;
    p.hyb_bytes = p.hyb_chunk = p.hyb_slot = 0;
    // f32 MAX/MIN and f64 MAX/MIN have no multimem form; they only reach here for TWOSHOT.
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

cudaError_t LaunchAllReduceHybrid(const DevComm& c, const void* src, void* dst, unsigned long long count, int dtype,
                                  int op, float scale, unsigned long long nvls_bytes, unsigned long long nvls_chunk,
                                  unsigned long long nvls_slot, int nvls_ctas, unsigned long long ts_chunk,
                                  unsigned long long ts_slot, int ts_ctas, int nslots, cudaStream_t stream, int lag) {
    using namespace dev;
    const unsigned long long bytes = count * (unsigned long long)dtype_size(dtype);
    const unsigned long long q = 16ull * c.nranks;
    if (nvls_ctas < 1 || ts_ctas < 1 || nvls_ctas + ts_ctas > kMaxCtas || lag < 1 || lag > 2 ||
        nslots < 2 * lag + 1 || nvls_bytes == 0 ||
        nvls_bytes >= bytes || (nvls_bytes % q) != 0 || nvls_chunk == 0 || (nvls_chunk % q) != 0 || ts_chunk == 0 ||
        (ts_chunk % q) != 0 || c.nvls_mc == nullptr || !NvlsSupports(dtype, op) ||
        (size_t)nslots * nvls_slot > c.nvls_bytes || nvls_slot < nvls_chunk ||
        (size_t)nslots * 2 * c.nranks * ts_slot > c.data_bytes / 2 || ts_slot * c.nranks < ts_chunk) {
        return cudaErrorInvalidValue;
    }
    PipeParams p;
    p.comm = c;
    p.src = src;
    p.dst = dst;
    p.bytes = bytes;
    p.chunk = ts_chunk;
    p.slot_bytes = ts_slot;
    p.nrounds = (int)((bytes - nvls_bytes + ts_chunk - 1) / ts_chunk);
    p.nslots = nslots;
    p.dtype = dtype;
    p.op = op;
    p.scale = scale;
    p.nvls = kPipeTwoShot;
    p.lag = lag;
    p.hyb_ctas = nvls_ctas;
    p.hyb_bytes = nvls_bytes;
    p.hyb_chunk = nvls_chunk;
    p.hyb_slot = nvls_slot;
    p.hyb_rounds = (int)((nvls_bytes + nvls_chunk - 1) / nvls_chunk);
    const int nctas = nvls_ctas + ts_ctas;
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
