// Point-to-point Send/Recv of the device communicator over NCCL.
//
// The reference runs Send/Recv over its own transports with lazily built connections
// (OriginCCL src/planner.cpp:210-513, src/topology/topology_p2p.cpp:46-66). Here NCCL
// p2p carries them: the NCCL communicator is created at Init from an ncclUniqueId that
// travels over this library's bootstrap, and a batch's Send/Recv are issued inside one
// ncclGroupStart/ncclGroupEnd on the communicator's stream, after its collectives.
// libnccl.so.2 is opened at run time (the copy PyTorch ships when loaded from Python),
// so the library itself has no link dependency on NCCL.
#pragma once

#include <cuda_runtime.h>

#include <vector>

#include "bccl/types.h"

namespace bccl {

class Bootstrap;

class NcclP2p {
public:
    bool Init(int rank, int nranks, Bootstrap* bs);
    void Destroy();
    bool ready() const { return comm_ != nullptr; }
    // Issues the P2P tasks (already in round order) as one NCCL group on `stream`.
    bool Run(const std::vector<CollTask>& tasks, cudaStream_t stream);
    const char* version() const { return version_; }

private:
    void* lib_ = nullptr;
    void* comm_ = nullptr;
    char version_[32] = {0};
};

}  // namespace bccl
