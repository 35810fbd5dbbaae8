// Passing file descriptors between the processes of one machine (AF_UNIX + SCM_RIGHTS).
//
// The GPU path exports cuMem allocations and NVLS multicast objects as POSIX file
// descriptors and the host path shares a memfd segment; both travel through this class.
// Parity: the reference's SHM transport passes its memfd ring and eventfds the same way
// (OriginCCL src/transport/transport_shm.cpp:204-278); here it is a standalone service
// keyed by (tag, source rank) so several exchanges can be in flight in any order.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <utility>

namespace bccl {

class FdPasser {
public:
    FdPasser() = default;
    ~FdPasser() { Close(); }
    FdPasser(const FdPasser&) = delete;
    FdPasser& operator=(const FdPasser&) = delete;

    // Binds the abstract socket "bccl.<ns>.<rank>". Must run before the bootstrap so peers
    // can never connect to an unbound name.
    bool Listen(const std::string& ns, int rank);
    // Sends a duplicate of `fd` to `peer` under `tag`.
    bool SendFd(int peer, uint32_t tag, int fd, int timeout_ms);
    // Receives the fd that `src` sent under `tag` (other arrivals are stashed).
    bool RecvFd(int src, uint32_t tag, int* fd, int timeout_ms);
    void Close();

private:
    std::string Name(int rank) const;

    std::string ns_;
    int rank_ = -1;
    int listen_fd_ = -1;
    std::map<std::pair<uint32_t, int>, int> stash_;
};

}  // namespace bccl
