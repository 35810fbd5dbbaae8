// Push engine: one kernel for every small/medium collective and for whole groups.
//
// The reference runs each collective as a CPU state machine over per-edge transports
// (OriginCCL src/topology/topology_ring.cpp:330-623, topology_tree.cpp:135-306) and its
// dynamic executor spreads a group's slices over channels with an in-band control
// broadcast (src/executor/dynamic_multi_thread_executor.cpp:176-230). On one NVSwitch
// node every GPU is one hop from every other, so here each rank stores its per-peer
// payload straight into the peer's inbox over NVLink, crosses one flag barrier per round
// and then consumes its inbox locally:
//   AllReduce / Reduce : push the input to every peer (to the root), reduce N slots
//   ReduceScatter      : push shard p to peer p, reduce N slots of the own shard
//   AllGather          : push the input to every peer, copy slots into the output
//   Broadcast          : the root pushes, the others copy their slot out
// A launch carries a list of WorkItems laid end to end in a per-peer byte stream; rounds
// cut the stream into inbox-sized pieces and CTA b always owns piece b of a round on
// every rank, so one per-CTA barrier per round is the only synchronisation (no grid-wide
// barrier, no host round trip). Inboxes are double-buffered by round parity; a rank only
// rewrites half h after the barrier of the following round has proven that every peer
// finished reading it.
#include "kernels/push_engine.cuh"
#include "kernels/launch.h"

namespace bccl {
namespace dev {
namespace {

template <int MAXI>
struct PushParams {
    DevComm comm;
    int nitems;
    int nrounds;
    unsigned long long stream_bytes;
    unsigned long long slot_bytes;  // per-source inbox capacity of one half
    WorkItem items[MAXI];
};

// Kernel parameters are limited to 32764 bytes (CUDA 12.1+ on sm_70 and later).
static_assert(sizeof(PushParams<kPushMaxItems>) <= 32764, "push-engine work list exceeds the kernel parameter limit");

template <int MAXI>
__global__ void __launch_bounds__(512, 1) push_engine_kernel(const __grid_constant__ PushParams<MAXI> p) {
    push_engine_body(p.comm, p.items, p.nitems, p.nrounds, p.stream_bytes, p.slot_bytes);
}

template <int MAXI>
cudaError_t Launch(const DevComm& c, const WorkItem* items, int nitems, unsigned long long stream_bytes,
                   unsigned long long slot_bytes, int nctas, cudaStream_t s) {
    PushParams<MAXI> p;
    p.comm = c;
    p.nitems = nitems;
    p.stream_bytes = stream_bytes;
    p.slot_bytes = slot_bytes;
    p.nrounds = (int)((stream_bytes + slot_bytes - 1) / slot_bytes);
    if (p.nrounds == 0) p.nrounds = 1;
    for (int i = 0; i < nitems; ++i) p.items[i] = items[i];
    push_engine_kernel<MAXI><<<nctas, 512, 0, s>>>(p);
    return cudaGetLastError();
}

}  // namespace
}  // namespace dev

cudaError_t LaunchPushEngine(const DevComm& c, const WorkItem* items, int nitems, unsigned long long stream_bytes,
                             unsigned long long slot_bytes, int nctas, cudaStream_t stream) {
    if (nitems <= 0 || nctas <= 0 || nctas > kMaxCtas || slot_bytes == 0 || (slot_bytes & 15) != 0) {
        return cudaErrorInvalidValue;
    }
    if (nitems <= 4) return dev::Launch<4>(c, items, nitems, stream_bytes, slot_bytes, nctas, stream);
    if (nitems <= kPushMaxItems) {
        return dev::Launch<kPushMaxItems>(c, items, nitems, stream_bytes, slot_bytes, nctas, stream);
    }
    return cudaErrorInvalidValue;
}

}  // namespace bccl
