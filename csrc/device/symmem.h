// Symmetric device memory: one same-size allocation per rank, mapped by every rank.
//
// This replaces the reference's byte movers (SHM ring, TCP, RDMA; OriginCCL
// src/transport/*) on an NVSwitch node. Each rank creates physical memory with
// cuMemCreate, exports it as a POSIX fd, passes the fd to every local peer over AF_UNIX
// (SCM_RIGHTS), imports the peers' fds and maps all of them into one contiguous virtual
// range, so a kernel reaches rank p's copy at ptr[p] with ordinary loads and stores over
// NVLink. With multicast, rank 0 also creates an NVLS multicast object, every rank adds its
// device, binds its physical memory and maps the multicast address (mc) on which
// multimem.* instructions operate.
// Alloc/Free are collective over the communicator (same order and sizes on every rank).
// Any failure on any rank is agreed through the bootstrap so that no rank proceeds with a
// half-built mapping.
#pragma once

#include <cuda.h>

#include <cstddef>
#include <cstdint>

#include "device/dev_types.h"

namespace bccl {

class Bootstrap;
class FdPasser;

struct SymBuffer {
    size_t bytes = 0;                     // per rank (rounded to the granularity)
    char* ptr[kMaxRanks] = {};            // rank r's copy, mapped here
    char* base = nullptr;                 // start of the contiguous reservation
    CUmemGenericAllocationHandle local = 0;
    CUmemGenericAllocationHandle imported[kMaxRanks] = {};
    CUmemGenericAllocationHandle mc_handle = 0;
    char* mc = nullptr;                   // multicast address, or null
    bool valid = false;
};

class SymmetricMemory {
public:
    bool Init(int device, int rank, int nranks, Bootstrap* bs, FdPasser* fp, int timeout_ms, bool want_multicast);
    bool Alloc(size_t bytes, bool with_multicast, SymBuffer* out);
    void Free(SymBuffer* buf);
    bool multicast_supported() const { return mc_supported_; }
    size_t granularity() const { return gran_; }

private:
    bool SetupMulticast(SymBuffer* buf, uint32_t tag_base);
    bool AgreeAll(bool mine);  // true iff every rank passed `true`

    int device_ = -1;
    CUdevice cudev_ = 0;
    int rank_ = 0;
    int nranks_ = 1;
    Bootstrap* bs_ = nullptr;
    FdPasser* fp_ = nullptr;
    int timeout_ms_ = 30000;
    size_t gran_ = 2u << 20;
    size_t mc_gran_ = 2u << 20;
    bool mc_supported_ = false;
    uint32_t seq_ = 0;
};

}  // namespace bccl
