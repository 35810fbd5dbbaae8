// NVSwitch multicast (NVLS) collectives.
//
// The reference reduces on the CPU after moving every byte through transports
// (OriginCCL src/utils.cpp:312-370, src/topology/topology_ring.cpp:255-290). On an
// NVSwitch node the switch itself can reduce: multimem.ld_reduce on the multicast address
// returns the element-wise reduction of every rank's copy, multimem.st writes one value to
// every rank's copy. Per round:
//   AllReduce: copy-in the chunk -> barrier -> each rank ld_reduce+st its 1/N shard ->
//              barrier -> copy-out. Per-direction NVLink bytes ~ S*(1+1/N) instead of the
//              2*S*(N-1)/N of any point-to-point algorithm.
//   Broadcast: the root multimem.st's its chunk (one egress copy) -> barrier -> copy-out.
//   Reduce:    copy-in -> barrier -> the root ld_reduce's into its output -> barrier.
// zero_copy: src/dst are already the NVLS buffer (symmetric allocation), so copy-in and
// copy-out are skipped.
// CTA b owns piece b of every shard on every rank, so the barriers are per-CTA only.
#include "kernels/common.cuh"
#include "kernels/launch.h"

namespace bccl {
namespace dev {
namespace {

// ---- multimem wrappers (16 bytes). Supported (dtype, op) pairs were checked against ptxas
// for sm_100a: f32 has add only; bf16/f16 add (fp32 accumulation), max, min; integers
// add/max/min through scalar 32/64-bit forms; f64 add.
template <int D, int O>
__device__ __forceinline__ uint4 mm_ld_reduce(const void* p);

#define BCCL_MM_V4(D, O, SPEC)                                                                       \
    template <>                                                                                    \
    __device__ __forceinline__ uint4 mm_ld_reduce<D, O>(const void* p) {                           \
        uint4 r;                                                                                   \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " {%0,%1,%2,%3}, [%4];"         \
                     : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)                                  \
                     : "l"(p)                                                                      \
                     : "memory");                                                                  \
        return r;                                                                                  \
    }
#define BCCL_MM_S32(D, O, SPEC)                                                                      \
    template <>                                                                                    \
    __device__ __forceinline__ uint4 mm_ld_reduce<D, O>(const void* p) {                           \
        uint4 r;                                                                                   \
        const char* c = static_cast<const char*>(p);                                               \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " %0, [%1];" : "=r"(r.x) : "l"(c) : "memory");      \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " %0, [%1];" : "=r"(r.y) : "l"(c + 4) : "memory");  \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " %0, [%1];" : "=r"(r.z) : "l"(c + 8) : "memory");  \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " %0, [%1];" : "=r"(r.w) : "l"(c + 12) : "memory"); \
        return r;                                                                                  \
    }
#define BCCL_MM_S64(D, O, SPEC)                                                                      \
    template <>                                                                                    \
    __device__ __forceinline__ uint4 mm_ld_reduce<D, O>(const void* p) {                           \
        unsigned long long a, b;                                                                   \
        const char* c = static_cast<const char*>(p);                                               \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " %0, [%1];" : "=l"(a) : "l"(c) : "memory");        \
        asm volatile("multimem.ld_reduce.relaxed.sys.global." SPEC " %0, [%1];" : "=l"(b) : "l"(c + 8) : "memory");    \
        return make_uint4((unsigned)a, (unsigned)(a >> 32), (unsigned)b, (unsigned)(b >> 32));     \
    }

BCCL_MM_V4(kF32, kSum, "add.v4.f32")
BCCL_MM_V4(kBF16, kSum, "add.acc::f32.v4.bf16x2")
BCCL_MM_V4(kBF16, kMax, "max.v4.bf16x2")
BCCL_MM_V4(kBF16, kMin, "min.v4.bf16x2")
BCCL_MM_V4(kF16, kSum, "add.acc::f32.v4.f16x2")
BCCL_MM_V4(kF16, kMax, "max.v4.f16x2")
BCCL_MM_V4(kF16, kMin, "min.v4.f16x2")
BCCL_MM_S32(kI32, kSum, "add.u32")
BCCL_MM_S32(kI32, kMax, "max.s32")
BCCL_MM_S32(kI32, kMin, "min.s32")
BCCL_MM_S64(kI64, kSum, "add.u64")
BCCL_MM_S64(kI64, kMax, "max.s64")
BCCL_MM_S64(kI64, kMin, "min.s64")
BCCL_MM_S64(kF64, kSum, "add.f64")

__device__ __forceinline__ void mm_st(void* p, const uint4& v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

// AVG and the fused scale on a reduced 16-byte vector.
template <int D>
__device__ __forceinline__ uint4 apply_epilogue(uint4 u, int op, int nranks, float scale) {
    if (op != kAvg && scale == 1.0f) return u;
    using T = Ty<D>;
    V16<D> v;
    v.u = u;
    constexpr int E = 16 / sizeof(typename T::Bits);
#pragma unroll
    for (int e = 0; e < E; ++e) v.b[e] = T::store(epilogue<typename T::Acc>(op, T::load(v.b[e]), nranks, scale));
    return v.u;
}

// 16 bytes from a possibly short, possibly unaligned tail (never reads past `valid`).
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
    unsigned long long chunk;  // bytes per round (multiple of 16 * nranks)
    int nrounds;
    int func;
    int dtype;
    int op;
    int root;
    float scale;
    int zero_copy;
};

// [lo, hi) of shard q, piece b, clipped to [0, limit).
__device__ __forceinline__ void shard_piece(size_t shard, size_t piece, int q, size_t limit, size_t* lo, size_t* hi) {
    size_t s0 = (size_t)q * shard, s1 = min(limit, s0 + shard);
    size_t a = s0 + (size_t)blockIdx.x * piece;
    *lo = min(a, s1);
    *hi = min(a + piece, s1);
}

template <int D, int O>
__device__ void reduce_range(const NvlsParams& p, char* mc, char* out_uc, size_t lo, size_t hi, bool to_mc) {
    const int nr = p.comm.nranks;
    for (size_t off = lo + (size_t)threadIdx.x * 16; off < hi; off += (size_t)blockDim.x * 16) {
        uint4 v = apply_epilogue<D>(mm_ld_reduce<D, O>(mc + off), p.op, nr, p.scale);
        if (to_mc) {
            mm_st(mc + off, v);
        } else {
            // Reduce: the root writes its own output; clip the final partial vector.
            size_t valid = min((size_t)16, hi - off);
            char* d = out_uc + off;
            if (valid == 16 && (reinterpret_cast<uintptr_t>(d) & 15) == 0) {
                *reinterpret_cast<uint4*>(d) = v;
            } else {
                const char* b = reinterpret_cast<const char*>(&v);
                for (size_t i = 0; i < valid; ++i) d[i] = b[i];
            }
        }
    }
}

template <int D, int O>
__device__ bool nvls_round(const NvlsParams& p, int j, uint64_t half, uint64_t& bar) {
    const DevComm& c = p.comm;
    const int r = c.rank, n = c.nranks;
    const size_t cap = p.chunk;
    const size_t cbeg = (size_t)j * p.chunk;
    const size_t clen = min((size_t)p.bytes - cbeg, (size_t)p.chunk);
    const size_t padded = round_up(clen, 16);
    char* buf_uc = p.zero_copy ? (char*)p.dst + cbeg : c.nvls_uc + half * cap;
    char* buf_mc = p.zero_copy ? c.nvls_mc + ((char*)p.dst - c.nvls_uc) + cbeg : c.nvls_mc + half * cap;
    const char* src = static_cast<const char*>(p.src) + cbeg;
    char* dst = static_cast<char*>(p.dst) + cbeg;

    if (p.func == 0) {  // AllReduce
        const size_t shard = round_up((clen + n - 1) / n, 16);
        const size_t piece = round_up((shard + gridDim.x - 1) / gridDim.x, 16);
        size_t lo, hi;
        if (!p.zero_copy) {
            for (int q = 0; q < n; ++q) {
                shard_piece(shard, piece, q, clen, &lo, &hi);
                if (lo < hi) cta_copy(buf_uc + lo, src + lo, hi - lo, false);
            }
        }
        fence_proxy_alias();
        if (!cta_barrier(c, ++bar, 2 * j)) return false;
        fence_proxy_alias();
        shard_piece(shard, piece, r, padded, &lo, &hi);
        reduce_range<D, O>(p, buf_mc, nullptr, lo, hi, true);
        fence_proxy_alias();
        if (!cta_barrier(c, ++bar, 2 * j + 1)) return false;
        fence_proxy_alias();
        if (!p.zero_copy) {
            for (int q = 0; q < n; ++q) {
                shard_piece(shard, piece, q, clen, &lo, &hi);
                if (lo < hi) cta_copy(dst + lo, buf_uc + lo, hi - lo, true);
            }
        }
        return true;
    }
    const size_t piece = round_up((clen + gridDim.x - 1) / gridDim.x, 16);
    size_t lo, hi;
    shard_piece(clen, piece, 0, clen, &lo, &hi);
    if (p.func == 1) {  // Broadcast
        if (r == p.root) {
            for (size_t off = lo + (size_t)threadIdx.x * 16; off < hi; off += (size_t)blockDim.x * 16)
                mm_st(buf_mc + off, load_partial(src + off, hi - off));
        }
        fence_proxy_alias();
        if (!cta_barrier(c, ++bar, 2 * j)) return false;
        fence_proxy_alias();
        if (lo < hi && (r != p.root ? true : dst != src)) {
            cta_copy(dst + lo, r == p.root ? src + lo : buf_uc + lo, hi - lo, r != p.root);
        }
        return true;
    }
    // Reduce
    if (!p.zero_copy && lo < hi) cta_copy(buf_uc + lo, src + lo, hi - lo, false);
    fence_proxy_alias();
    if (!cta_barrier(c, ++bar, 2 * j)) return false;
    fence_proxy_alias();
    if (r == p.root) reduce_range<D, O>(p, buf_mc, dst, lo, hi, false);
    if (!cta_barrier(c, ++bar, 2 * j + 1)) return false;
    return true;
}

template <int D, int O>
__global__ void __launch_bounds__(512, 1) nvls_kernel(const __grid_constant__ NvlsParams p) {
    const DevComm& c = p.comm;
    const uint64_t round0 = load_state_u64(&c.state->nvls_round_seq);
    uint64_t bar = load_state_u64(&c.state->barrier_seq);
    const uint64_t bar0 = bar;
    for (int j = 0; j < p.nrounds; ++j) {
        if (!nvls_round<D, O>(p, j, (round0 + (uint64_t)j) & 1ull, bar)) break;
    }
    const uint64_t per_round = (p.func == 1) ? 1 : 2;
    (void)bar0;
    finish_launch(c, 0, per_round * (uint64_t)p.nrounds, (uint64_t)p.nrounds);
}

template <int D, int O>
cudaError_t launch_t(const NvlsParams& p, int nctas, cudaStream_t s) {
    nvls_kernel<D, O><<<nctas, 512, 0, s>>>(p);
    return cudaGetLastError();
}

cudaError_t dispatch(const NvlsParams& p, int nctas, cudaStream_t s) {
    // Broadcast never reduces; any supported instantiation serves it.
    const int op = (p.func == 1) ? kSum : (p.op == kAvg ? kSum : p.op);
    const int dt = (p.func == 1) ? kF32 : p.dtype;
#define BCCL_CASE(D, O) \
    if (dt == D && op == O) return launch_t<D, O>(p, nctas, s);
    BCCL_CASE(kF32, kSum)
    BCCL_CASE(kBF16, kSum)
    BCCL_CASE(kBF16, kMax)
    BCCL_CASE(kBF16, kMin)
    BCCL_CASE(kF16, kSum)
    BCCL_CASE(kF16, kMax)
    BCCL_CASE(kF16, kMin)
    BCCL_CASE(kI32, kSum)
    BCCL_CASE(kI32, kMax)
    BCCL_CASE(kI32, kMin)
    BCCL_CASE(kI64, kSum)
    BCCL_CASE(kI64, kMax)
    BCCL_CASE(kI64, kMin)
    BCCL_CASE(kF64, kSum)
#undef BCCL_CASE
    return cudaErrorNotSupported;
}

}  // namespace
}  // namespace dev

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
                       int op, int root, float scale, unsigned long long chunk_cap, int nctas, bool zero_copy,
                       cudaStream_t stream) {
    if (c.nvls_mc == nullptr || nctas <= 0 || nctas > kMaxCtas || chunk_cap == 0 || (chunk_cap % (16ull * c.nranks)) != 0) {
        return cudaErrorInvalidValue;
    }
    if (func != 1 && !NvlsSupports(dtype, op)) return cudaErrorNotSupported;
    dev::NvlsParams p;
    p.comm = c;
    p.src = src;
    p.dst = dst;
    p.bytes = count * (unsigned long long)dev::dtype_size(dtype);
    p.chunk = zero_copy ? p.bytes : chunk_cap;
    if (zero_copy) p.chunk = dev::round_up(p.bytes, 16ull * c.nranks);
    p.nrounds = (int)((p.bytes + p.chunk - 1) / p.chunk);
    if (p.nrounds == 0) p.nrounds = 1;
    p.func = func;
    p.dtype = dtype;
    p.op = op;
    p.root = root;
    p.scale = scale;
    p.zero_copy = zero_copy ? 1 : 0;
    return dev::dispatch(p, nctas, stream);
}

}  // namespace bccl
