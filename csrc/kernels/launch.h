// Host-callable launchers of the collective kernels (implemented in the .cu files).
// Every launcher only enqueues work on `stream`; errors in the kernel surface through the
// communicator's ErrorRecord after the stream synchronises.
#pragma once

#include <cuda_runtime.h>

#include "device/dev_types.h"
#include "kernels/p2p_sched.h"

namespace bccl {

constexpr int kPushMaxItems = 256;  // WorkItems carried in one push-engine launch's parameters

cudaError_t LaunchPushEngine(const DevComm& c, const WorkItem* items, int nitems, unsigned long long stream_bytes,
                             unsigned long long slot_bytes, int nctas, cudaStream_t stream);

// Pipelined AllReduce (kernels/ar_pipe.cu): NVSwitch multicast, two-shot (push reduce-scatter
// + push all-gather) or one-shot (push everything, reduce locally) through the second half of
// the UC data region.
enum PipeKind : int { kPipeTwoShot = 0, kPipeNvls = 1, kPipeOneShot = 2 };
cudaError_t LaunchAllReducePipe(const DevComm& c, int kind, const void* src, void* dst, unsigned long long count,
                                int dtype, int op, float scale, unsigned long long chunk, unsigned long long slot_bytes,
                                int nslots, int nctas, cudaStream_t stream, int lag = 1);
// One launch of the pipelined AllReduce split in two parts that run side by side: nvls_ctas
// CTAs reduce bytes [0, nvls_bytes) through the switch (NVLS kind), ts_ctas CTAs the rest over
// peer memory (two-shot kind). nvls_bytes and both chunks are multiples of 16 * nranks.
cudaError_t LaunchAllReduceHybrid(const DevComm& c, const void* src, void* dst, unsigned long long count, int dtype,
                                  int op, float scale, unsigned long long nvls_bytes, unsigned long long nvls_chunk,
                                  unsigned long long nvls_slot, int nvls_ctas, unsigned long long ts_chunk,
                                  unsigned long long ts_slot, int ts_ctas, int nslots, cudaStream_t stream,
                                  int lag = 1);

// NVSwitch multicast Broadcast (func 1), Reduce (2), AllGather (3) and ReduceScatter (4) over
// the NVLS slot ring. count is the payload (Broadcast, Reduce) or the per-rank block
// (AllGather, ReduceScatter) in elements; for the latter `chunk` is bytes of each rank's block
// per round (a multiple of 16, nranks * chunk <= slot_bytes) and ReduceScatter needs 3+ slots.
cudaError_t LaunchNvls(const DevComm& c, int func, const void* src, void* dst, unsigned long long count, int dtype,
                       int op, int root, float scale, unsigned long long chunk, unsigned long long slot_bytes,
                       int nslots, int nctas, cudaStream_t stream);

// Low-latency AllReduce (func 0), AllGather (3) or ReduceScatter (4) of up to kLLMaxLines * 8
// payload bytes per rank (ll.cu; count = elements of the payload or of one rank's block): no
// barrier, one NVLink trip.
cudaError_t LaunchCollectiveLL(const DevComm& c, int func, const void* src, void* dst, unsigned long long count,
                               int dtype, int op, float scale, cudaStream_t stream);

// Bounded-wait self-test: waits on a flag nothing sets; must time out and report.
cudaError_t LaunchWaitProbe(const DevComm& c, unsigned long long timeout_ns, cudaStream_t stream);

// Copy-bandwidth probe over local, peer or multicast addresses.
cudaError_t LaunchBandwidthProbe(void* dst, const void* src, unsigned long long bytes, bool multicast, int nctas,
                                 cudaStream_t stream);

// Ring AllReduce between neighbours (reduce-scatter then all-gather), `block` bytes per message
// (multiple of 256), at most max_ctas channels.
cudaError_t LaunchRingAllReduce(const DevComm& c, const void* src, void* dst, unsigned long long count, int dtype,
                                int op, float scale, unsigned long long block, int max_ctas, cudaStream_t stream);

// Zero-copy collectives on multicast-bound symmetric buffers (func 0 AllReduce: send and recv
// are multicast addresses; 3 AllGather: send local, recv multicast; 4 ReduceScatter: send
// multicast, recv local). count is the payload (AllReduce) or per-rank block (AllGather,
// ReduceScatter) in elements; its bytes must be a multiple of 16.
cudaError_t LaunchNvlsZeroCopy(const DevComm& c, int func, const void* send, void* recv, unsigned long long count,
                               int dtype, int op, float scale, int nctas, cudaStream_t stream);

// Zero-copy collectives over peer memory (func 0 AllReduce, 3 AllGather, 4 ReduceScatter):
// in[q] / out[q] are rank q's input / output as mapped on this GPU (AllGather reads only
// in[rank], ReduceScatter writes only out[rank]); count as for LaunchNvlsZeroCopy; bytes and
// every pointer 16-byte aligned.
cudaError_t LaunchP2pZeroCopy(const DevComm& c, int func, const char* const* in, char* const* out,
                              unsigned long long count, int dtype, int op, float scale, int nctas, cudaStream_t stream);

// Native Send/Recv of one group: one CTA per role (a channel of a directed pair), the pairs'
// operations in ops (p2p_sched.h); at most kP2pMaxRoles roles and kP2pMaxOps operations.
cudaError_t LaunchP2pNative(const DevComm& c, const P2pNativeOp* ops, int nops, const P2pNativeRole* roles,
                            int nroles, cudaStream_t stream);

// One-rank collective: dst = src, times `scale` for floating-point dtypes (1 = plain copy);
// bytes and both pointers 16-byte aligned; grid sized for `sms` SMs.
cudaError_t LaunchLocalCopy(const void* src, void* dst, unsigned long long bytes, int dtype, float scale, int sms,
                            cudaStream_t stream);

// Whether multimem.ld_reduce exists for (dtype, op) on this build.
bool NvlsSupports(int dtype, int op);

}  // namespace bccl
