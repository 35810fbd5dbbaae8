// Allocation-free variant of the push-engine kernel (see bccl/noalloc.h; no counterpart in
// the reference library). The kernel is the push engine's round loop run by a one-rank
// communicator; what differs is where its scratch memory lives: a file-scope device array.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "bccl/noalloc.h"
#include "bccl/types.h"
#include "core/logger.h"
#include "device/cuda_driver.h"
#include "kernels/push_engine.cuh"

namespace bccl {
namespace {

// Scratch layout: [DevState | ErrorRecord | abort word] in the first 2 KiB, then the
// work list (BCCL_NOALLOC_MAX_ITEMS WorkItems).
constexpr size_t kHeaderBytes = 2048;
static_assert(sizeof(DevState) + sizeof(ErrorRecord) + sizeof(int) <= kHeaderBytes, "scratch header too small");
static_assert(kHeaderBytes + sizeof(WorkItem) * BCCL_NOALLOC_MAX_ITEMS <= BCCL_NOALLOC_SCRATCH_BYTES,
              "scratch array too small for the work list");

static __device__ __align__(256) unsigned char g_noalloc_scratch[BCCL_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
// Device address of g_noalloc_scratch per device, and the context it was looked up in: a
// cudaDeviceReset destroys the primary context and reloads the module at another address, so a
// different current context means the cached address is stale.
void* g_scratch_addr[kMaxDevices] = {};
CUcontext g_scratch_ctx[kMaxDevices] = {};

// Once per device (and again after a context change), with that device current: the array's
// name in host code is only a host-side stand-in, so the device address comes from
// cudaGetSymbolAddress.
void* ScratchFor(int device) {
    std::lock_guard<std::mutex> lk(g_mu);
    CUcontext ctx = nullptr;
    const DriverApi* drv = Driver();
    if (drv != nullptr && drv->cuCtxGetCurrent != nullptr) drv->cuCtxGetCurrent(&ctx);
    if (g_scratch_addr[device] == nullptr || ctx != g_scratch_ctx[device]) {
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || ptr == nullptr) {
            LOG_ERROR("noalloc: cudaGetSymbolAddress failed on device %d: %s", device, cudaGetErrorString(e));
            return nullptr;
        }
        // The runtime makes the primary context current in that call; record that one.
        if (drv != nullptr && drv->cuCtxGetCurrent != nullptr) drv->cuCtxGetCurrent(&ctx);
        g_scratch_addr[device] = ptr;
        g_scratch_ctx[device] = ctx;
    }
    return g_scratch_addr[device];
}

__global__ void __launch_bounds__(512, 1) push_engine_scratch_kernel(DevComm c, int nitems, int nrounds,
                                                                     unsigned long long stream_bytes,
                                                                     unsigned long long slot) {
    // The work list sits in the scratch array right after the header.
    const WorkItem* items = reinterpret_cast<const WorkItem*>(reinterpret_cast<const char*>(c.state) + kHeaderBytes);
    dev::push_engine_body(c, items, nitems, nrounds, stream_bytes, slot);
}

}  // namespace
}  // namespace bccl

extern "C" int bcclLocalAllReduceNoAlloc(const void* const* srcs, void* const* dsts, const size_t* counts, int n,
                                         int dtype, int op, float scale, void* stream_ptr) {
    using namespace bccl;
    if (n < 0 || n > BCCL_NOALLOC_MAX_ITEMS) {
        LOG_ERROR("bcclLocalAllReduceNoAlloc: %d tensors requested, at most %d fit the fixed %d-byte scratch array",
                  n, BCCL_NOALLOC_MAX_ITEMS, BCCL_NOALLOC_SCRATCH_BYTES);
        return 1;
    }
    if (dtype < 0 || dtype > static_cast<int>(DataType::FP16) || op < 0 || op > static_cast<int>(ReduceOp::AVG)) {
        LOG_ERROR("bcclLocalAllReduceNoAlloc: invalid dtype %d or op %d", dtype, op);
        return 1;
    }
    if (n == 0) return 0;
    if (srcs == nullptr || dsts == nullptr || counts == nullptr) {
        LOG_ERROR("bcclLocalAllReduceNoAlloc: null argument array");
        return 1;
    }
    int device = -1;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) {
        LOG_ERROR("bcclLocalAllReduceNoAlloc: no usable current device");
        return 1;
    }
    char* scratch = static_cast<char*>(ScratchFor(device));
    if (scratch == nullptr) return 1;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);

    // Work list: items laid end to end in 16-byte padded slots of the per-peer stream.
    WorkItem items[BCCL_NOALLOC_MAX_ITEMS];
    const size_t es = DataTypeSize(static_cast<DataType>(dtype));
    unsigned long long off = 0;
    int m = 0;
    for (int i = 0; i < n; ++i) {
        if (counts[i] == 0) continue;
        if (srcs[i] == nullptr || dsts[i] == nullptr) {
            LOG_ERROR("bcclLocalAllReduceNoAlloc: tensor %d has a null pointer", i);
            return 1;
        }
        WorkItem& w = items[m++];
        memset(&w, 0, sizeof(w));
        w.src = srcs[i];
        w.dst = dsts[i];
        w.count = counts[i];
        w.stream_off = off;
        w.func = static_cast<unsigned char>(CollFunc::AllReduce);
        w.dtype = static_cast<unsigned char>(dtype);
        w.op = static_cast<unsigned char>(op);
        w.scale = scale;
        off += (counts[i] * es + 15) / 16 * 16;
    }
    if (m == 0) return 0;

    // The counters, the error record and the abort word must start at zero on every call
    // (the array keeps the previous call's contents); the work list is copied behind them. The
    // list is built in host memory on this stack frame; an asynchronous copy from pageable
    // memory takes its bytes into the driver's staging memory before it returns.
    cudaError_t e = cudaMemsetAsync(scratch, 0, kHeaderBytes, stream);
    if (e == cudaSuccess) {
        e = cudaMemcpyAsync(scratch + kHeaderBytes, items, sizeof(WorkItem) * static_cast<size_t>(m),
                            cudaMemcpyHostToDevice, stream);
    }
    if (e != cudaSuccess) {
        LOG_ERROR("bcclLocalAllReduceNoAlloc: staging the work list failed: %s", cudaGetErrorString(e));
        return 1;
    }
    DevComm c;
    memset(&c, 0, sizeof(c));
    c.rank = 0;
    c.nranks = 1;
    c.uc[0] = scratch;  // one rank: no inbox traffic, no peer flags
    c.state = reinterpret_cast<DevState*>(scratch);
    c.err = reinterpret_cast<ErrorRecord*>(scratch + sizeof(DevState));
    c.abort = reinterpret_cast<const volatile int*>(scratch + sizeof(DevState) + sizeof(ErrorRecord));
    c.timeout_ns = 10ull * 1000 * 1000 * 1000;
    // One round covering the whole stream; CTAs as for a push-engine launch of this size.
    const unsigned long long stream_bytes = off;
    const unsigned long long slot = (stream_bytes + 15) / 16 * 16;
    int ctas = 1;
    if (stream_bytes > (16u << 10)) ctas = 2;
    if (stream_bytes > (64u << 10)) ctas = 4;
    if (stream_bytes > (256u << 10)) ctas = 8;
    if (stream_bytes > (1u << 20)) ctas = static_cast<int>(std::min<unsigned long long>(148, std::max<unsigned long long>(16, stream_bytes / (128u << 10))));
    push_engine_scratch_kernel<<<ctas, 512, 0, stream>>>(c, m, 1, stream_bytes, slot);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
        LOG_ERROR("bcclLocalAllReduceNoAlloc: launch failed: %s", cudaGetErrorString(e));
        return 1;
    }
    return 0;
}
