// One-rank collectives of 1 MiB and more: every collective on a single rank is dst = src, times
// the AllReduce scale for floating-point types (AVG over one rank is the identity). The batched
// push kernel handles that too, but it is built for N sources (128 registers, one CTA per SM,
// two vectors in flight per thread) and reached ~40% of the HBM copy bandwidth; this kernel is a
// plain streaming copy: 256 threads, several CTAs per SM, four 16-byte loads in flight per
// thread before their stores.
#include "kernels/common.cuh"
#include "kernels/launch.h"

namespace bccl {
namespace dev {
namespace {

constexpr int kCopyThreads = 256;
constexpr int kCopyUnroll = 4;

template <int D>
__device__ __forceinline__ uint4 scale16(const uint4& v, float s) {
    using V = Vec<D>;
    using Acc = typename Ty<D>::Acc;
    Acc a[V::E];
    V::unpack(v, a);
#pragma unroll
    for (int e = 0; e < V::E; ++e) a[e] = a[e] * static_cast<Acc>(s);
    return V::pack(a);
}

// D < 0: plain copy; otherwise multiply by `scale` in type D.
template <int D>
__global__ void __launch_bounds__(kCopyThreads, 4) local_copy_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                                     size_t nvec, float scale) {
    const size_t stride = static_cast<size_t>(gridDim.x) * kCopyThreads;
    size_t i = static_cast<size_t>(blockIdx.x) * kCopyThreads + threadIdx.x;
    for (; i + (kCopyUnroll - 1) * stride < nvec; i += kCopyUnroll * stride) {
        uint4 v[kCopyUnroll];
#pragma unroll
        for (int u = 0; u < kCopyUnroll; ++u) v[u] = __ldcs(src + i + u * stride);
#pragma unroll
        for (int u = 0; u < kCopyUnroll; ++u) {
            if constexpr (D >= 0) v[u] = scale16<D>(v[u], scale);
            __stcs(dst + i + u * stride, v[u]);
        }
    }
    for (; i < nvec; i += stride) {
        uint4 v = __ldcs(src + i);
        if constexpr (D >= 0) v = scale16<D>(v, scale);
        __stcs(dst + i, v);
    }
}

template <int D>
cudaError_t launch(const void* src, void* dst, size_t nvec, float scale, int sms, cudaStream_t s) {
    const size_t want = (nvec + static_cast<size_t>(kCopyThreads) * kCopyUnroll - 1) /
                        (static_cast<size_t>(kCopyThreads) * kCopyUnroll);
    const int grid = static_cast<int>(std::max<size_t>(1, std::min<size_t>(want, static_cast<size_t>(sms) * 4)));
    local_copy_kernel<D><<<grid, kCopyThreads, 0, s>>>(static_cast<const uint4*>(src), static_cast<uint4*>(dst), nvec,
                                                       scale);
    return cudaGetLastError();
}

}  // namespace
}  // namespace dev

cudaError_t LaunchLocalCopy(const void* src, void* dst, unsigned long long bytes, int dtype, float scale, int sms,
                            cudaStream_t stream) {
    using namespace dev;
    if ((bytes % 16) != 0 || ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) != 0 ||
        sms <= 0) {
        return cudaErrorInvalidValue;
    }
    const size_t nvec = bytes / 16;
    if (nvec == 0) return cudaSuccess;
    const bool scaled = scale != 1.0f && (dtype == kF32 || dtype == kF64 || dtype == kBF16 || dtype == kF16);
    if (!scaled) return launch<-1>(src, dst, nvec, 1.0f, sms, stream);
    switch (dtype) {
    case kF32: return launch<kF32>(src, dst, nvec, scale, sms, stream);
    case kF64: return launch<kF64>(src, dst, nvec, scale, sms, stream);
    case kBF16: return launch<kBF16>(src, dst, nvec, scale, sms, stream);
    default: return launch<kF16>(src, dst, nvec, scale, sms, stream);
    }
}

}  // namespace bccl
