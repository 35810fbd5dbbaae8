// Init-time control plane: a TCP star through rank 0.
//
// Parity: OriginCCL src/bootstrap.cpp:12-193 exchanges NodeInfo through rank 0 (the master
// accepts N-1 workers, gathers their NodeInfo and broadcasts the table). This version keeps
// that shape and keeps the sockets open after the exchange so the same star carries the
// later control traffic: AllGather of opaque bytes (NCCL unique id, memory-handle
// metadata), Broadcast and Barrier. No collective payload ever travels here.
// Every receive is bounded by a timeout; a rank that never joins, joins late past the bound
// or sends a malformed hello makes Run() return false on every rank that can observe it.
#pragma once

#include <cstdint>
#include <vector>

#include "bccl/types.h"
#include "core/net.h"

namespace bccl {

class Bootstrap {
public:
    Bootstrap() = default;
    ~Bootstrap() { Close(); }
    Bootstrap(const Bootstrap&) = delete;
    Bootstrap& operator=(const Bootstrap&) = delete;

    // listen_fd is the socket GetUniqueId bound on rank 0 (borrowed, not closed here).
    bool Run(const CommConfig& cfg, const NodeInfo& local, int listen_fd, std::vector<NodeInfo>* all_nodes);
    bool AllGather(const std::vector<uint8_t>& mine, std::vector<std::vector<uint8_t>>* all);
    bool Broadcast(int root, std::vector<uint8_t>* data);
    bool Barrier();
    void Close();

    int timeout_ms() const { return timeout_ms_; }
    bool ready() const { return ready_; }

    static std::vector<uint8_t> EncodeNode(const NodeInfo& n);
    static bool DecodeNode(net::Reader* r, NodeInfo* n);

private:
    bool RunMaster(const NodeInfo& local, int listen_fd, std::vector<NodeInfo>* all_nodes);
    bool RunWorker(const CommConfig& cfg, const NodeInfo& local, std::vector<NodeInfo>* all_nodes);

    int rank_ = 0;
    int world_ = 1;
    int timeout_ms_ = 30000;
    bool ready_ = false;
    std::vector<int> worker_fds_;  // master only: fd per rank (index 0 unused)
    int master_fd_ = -1;           // workers only
};

}  // namespace bccl
