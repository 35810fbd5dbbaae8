// Host-callable launchers of the collective kernels (implemented in the .cu files).
// Every launcher only enqueues work on `stream`; errors in the kernel surface through the
// communicator's ErrorRecord after the stream synchronises.
#pragma once

#include <cuda_runtime.h>

#include "device/dev_types.h"

namespace bccl {

constexpr int kPushMaxItems = 256;  // WorkItems carried in one push-engine launch's parameters

cudaError_t LaunchPushEngine(const DevComm& c, const WorkItem* items, int nitems, unsigned long long stream_bytes,
                             unsigned long long slot_bytes, int nctas, cudaStream_t stream);

// AllReduce by reduce-scatter (push) + all-gather (pull) through the UC data region.
cudaError_t LaunchTwoShot(const DevComm& c, const void* src, void* dst, unsigned long long count, int dtype, int op,
                          float scale, unsigned long long shard_cap, int nctas, cudaStream_t stream);

// NVSwitch multicast collectives: func is AllReduce, Broadcast or Reduce.
cudaError_t LaunchNvls(const DevComm& c, int func, const void* src, void* dst, unsigned long long count, int dtype,
                       int op, int root, float scale, unsigned long long chunk_cap, int nctas, bool zero_copy,
                       cudaStream_t stream);
// Bounded-wait self-test: waits on a flag nothing sets; must time out and report.
cudaError_t LaunchWaitProbe(const DevComm& c, unsigned long long timeout_ns, cudaStream_t stream);

// Whether multimem.ld_reduce exists for (dtype, op) on this build.
bool NvlsSupports(int dtype, int op);

}  // namespace bccl
