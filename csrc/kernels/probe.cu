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

}  // namespace
}  // namespace dev

cudaError_t LaunchWaitProbe(const DevComm& c, unsigned long long timeout_ns, cudaStream_t stream) {
    dev::wait_probe_kernel<<<1, 32, 0, stream>>>(c, timeout_ns);
    return cudaGetLastError();
}

}  // namespace bccl
