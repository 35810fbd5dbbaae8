// Self-test of the bounded wait: one thread waits on a flag that nothing ever sets (the
// rank's own slot of the last CTA row, which peers never write) and must give up after the
// given time, record kDevTimeout in the host-mapped error record and return. Used by the
// failure-detection tests; it cannot fault or hang the GPU.
#include "kernels/common.cuh"
#include "kernels/launch.h"

namespace bccl {
namespace dev {
namespace {

__global__ void wait_probe_kernel(DevComm c, unsigned long long timeout_ns) {
    c.timeout_ns = timeout_ns;
    if (threadIdx.x == 0) {
        const uint64_t* f = barrier_flag(c.uc[c.rank], kMaxCtas - 1, c.rank);
        wait_flag_geq(c, f, ~0ull >> 1, c.rank, -1);
    }
}

// Bandwidth probe: grid-strided 16-byte copy, 4 vectors in flight per thread. With dst or
// src in a peer's memory this measures NVLink write or read bandwidth; with dst in the
// multicast view (mode 3) it measures multimem.st.
__global__ void __launch_bounds__(512, 1) bw_probe_kernel(char* dst, const char* src, size_t bytes, int multicast) {
    const size_t nv = bytes >> 4;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < nv; i += 4 * stride) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = ld_cg(src + ((i + u * stride) << 4));
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            char* d = dst + ((i + u * stride) << 4);
            if (multicast) {
                asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(d), "r"(v[u].x),
                             "r"(v[u].y), "r"(v[u].z), "r"(v[u].w) : "memory");
            } else {
                st_cg(d, v[u]);
            }
        }
    }
    for (; i < nv; i += stride) st_cg(dst + (i << 4), ld_cg(src + (i << 4)));
}

}  // namespace
}  // namespace dev

cudaError_t LaunchBandwidthProbe(void* dst, const void* src, unsigned long long bytes, bool multicast, int nctas,
                                 cudaStream_t stream) {
    dev::bw_probe_kernel<<<nctas, 512, 0, stream>>>(static_cast<char*>(dst), static_cast<const char*>(src), bytes,
                                                    multicast ? 1 : 0);
    return cudaGetLastError();
}

cudaError_t LaunchWaitProbe(const DevComm& c, unsigned long long timeout_ns, cudaStream_t stream) {
    dev::wait_probe_kernel<<<1, 32, 0, stream>>>(c, timeout_ns);
    return cudaGetLastError();
}

}  // namespace bccl
