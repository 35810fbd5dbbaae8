#include "core/bootstrap.h"

#include <chrono>
#include <thread>
#include <unistd.h>

#include "core/env.h"
#include "core/logger.h"
#include "core/net.h"

namespace bccl {
namespace {

constexpr uint32_t kHelloMagic = 0xBCC10A01u;
constexpr uint32_t kTableMagic = 0xBCC10A02u;
constexpr uint32_t kGatherMagic = 0xBCC10A03u;

}  // namespace

std::vector<uint8_t> Bootstrap::EncodeNode(const NodeInfo& n) {
    net::Writer w;
    w.I32(n.rank);
    w.Str(n.ip_addr);
    w.U16(n.data_port);
    w.Str(n.hostname);
    w.U64(n.boot_id_hash);
    w.I32(n.device);
    w.I32(n.pid);
    return w.bytes();
}

bool Bootstrap::DecodeNode(net::Reader* r, NodeInfo* n) {
    int32_t rank = 0, dev = 0, pid = 0;
    if (!r->I32(&rank) || !r->Str(&n->ip_addr) || !r->U16(&n->data_port) || !r->Str(&n->hostname) ||
        !r->U64(&n->boot_id_hash) || !r->I32(&dev) || !r->I32(&pid)) {
        return false;
    }
    n->rank = rank;
    n->device = dev;
    n->pid = pid;
    return true;
}

bool Bootstrap::Run(const CommConfig& cfg, const NodeInfo& local, int listen_fd, std::vector<NodeInfo>* all_nodes) {
    rank_ = cfg.rank;
    world_ = cfg.world_size;
    timeout_ms_ = static_cast<int>(EnvInt("BCCL_BOOTSTRAP_TIMEOUT_MS", 30000));
    all_nodes->assign(world_, NodeInfo());
    if (world_ == 1) {
        (*all_nodes)[0] = local;
        ready_ = true;
        return true;
    }
    bool ok = (rank_ == 0) ? RunMaster(local, listen_fd, all_nodes) : RunWorker(cfg, local, all_nodes);
    ready_ = ok;
    if (!ok) Close();
    return ok;
}

bool Bootstrap::RunMaster(const NodeInfo& local, int listen_fd, std::vector<NodeInfo>* all_nodes) {
    if (listen_fd < 0) {
        LOG_ERROR("bootstrap: rank 0 has no listening socket (call GetUniqueId on rank 0 first)");
        return false;
    }
    worker_fds_.assign(world_, -1);
    (*all_nodes)[0] = local;
    auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms_);
    int joined = 1;
    while (joined < world_) {
        int left = static_cast<int>(std::chrono::duration_cast<std::chrono::milliseconds>(
                                        deadline - std::chrono::steady_clock::now())
                                        .count());
        if (left <= 0) {
            LOG_ERROR("bootstrap: only %d of %d ranks joined within %d ms", joined, world_, timeout_ms_);
            return false;
        }
        int fd = net::Accept(listen_fd, left);
        if (fd < 0) continue;
        std::vector<uint8_t> hello;
        if (!net::RecvFrame(fd, &hello, timeout_ms_, 1 << 20)) {
            LOG_ERROR("bootstrap: failed to receive a hello frame");
            close(fd);
            return false;
        }
        net::Reader r(hello);
        uint32_t magic = 0;
        int32_t world = 0;
        NodeInfo node;
        if (!r.U32(&magic) || magic != kHelloMagic || !r.I32(&world) || !DecodeNode(&r, &node)) {
            LOG_ERROR("bootstrap: malformed hello (magic 0x%08x)", magic);
            close(fd);
            return false;
        }
        if (world != world_ || node.rank <= 0 || node.rank >= world_ || worker_fds_[node.rank] >= 0) {
            LOG_ERROR("bootstrap: rejected hello from rank %d (world %d, expected %d)", node.rank, world, world_);
            close(fd);
            return false;
        }
        worker_fds_[node.rank] = fd;
        (*all_nodes)[node.rank] = node;
        ++joined;
    }
    net::Writer w;
    w.U32(kTableMagic);
    w.I32(world_);
    for (const NodeInfo& n : *all_nodes) w.Raw(EncodeNode(n).data(), EncodeNode(n).size());
    for (int r = 1; r < world_; ++r) {
        if (!net::SendFrame(worker_fds_[r], w.bytes(), timeout_ms_)) {
            LOG_ERROR("bootstrap: failed to send the node table to rank %d", r);
            return false;
        }
    }
    return true;
}

bool Bootstrap::RunWorker(const CommConfig& cfg, const NodeInfo& local, std::vector<NodeInfo>* all_nodes) {
    long arg = 0;
    if (FaultActive("bootstrap_skip", rank_, &arg)) {
        LOG_ERROR("bootstrap: rank %d skips the bootstrap (fault injection)", rank_);
        return false;
    }
    if (FaultActive("bootstrap_delay", rank_, &arg)) {
        std::this_thread::sleep_for(std::chrono::milliseconds(arg));
    }
    master_fd_ = net::Connect(cfg.unique_id.ip_addr, cfg.unique_id.port, timeout_ms_);
    if (master_fd_ < 0) {
        LOG_ERROR("bootstrap: rank %d could not reach rank 0 at %s:%u", rank_, cfg.unique_id.ip_addr,
                  cfg.unique_id.port);
        return false;
    }
    net::Writer w;
    w.U32(FaultActive("bootstrap_corrupt", rank_) ? 0xDEADBEEFu : kHelloMagic);
    w.I32(world_);
    auto enc = EncodeNode(local);
    w.Raw(enc.data(), enc.size());
    if (!net::SendFrame(master_fd_, w.bytes(), timeout_ms_)) {
        LOG_ERROR("bootstrap: rank %d failed to send its hello", rank_);
        return false;
    }
    std::vector<uint8_t> table;
    if (!net::RecvFrame(master_fd_, &table, timeout_ms_)) {
        LOG_ERROR("bootstrap: rank %d did not receive the node table", rank_);
        return false;
    }
    net::Reader r(table);
    uint32_t magic = 0;
    int32_t world = 0;
    if (!r.U32(&magic) || magic != kTableMagic || !r.I32(&world) || world != world_) {
        LOG_ERROR("bootstrap: rank %d received a malformed node table", rank_);
        return false;
    }
    for (int i = 0; i < world_; ++i) {
        if (!DecodeNode(&r, &(*all_nodes)[i]) || (*all_nodes)[i].rank != i) {
            LOG_ERROR("bootstrap: rank %d could not decode node %d", rank_, i);
            return false;
        }
    }
    return true;
}

bool Bootstrap::AllGather(const std::vector<uint8_t>& mine, std::vector<std::vector<uint8_t>>* all) {
    all->assign(world_, {});
    (*all)[rank_] = mine;
    if (world_ == 1) return true;
    if (!ready_) {
        LOG_ERROR("bootstrap: AllGather before a successful Run");
        return false;
    }
    if (rank_ == 0) {
        for (int r = 1; r < world_; ++r) {
            std::vector<uint8_t> frame;
            if (!net::RecvFrame(worker_fds_[r], &frame, timeout_ms_)) {
                LOG_ERROR("bootstrap: AllGather lost rank %d", r);
                return false;
            }
            net::Reader rd(frame);
            uint32_t magic = 0;
            if (!rd.U32(&magic) || magic != kGatherMagic) {
                LOG_ERROR("bootstrap: AllGather got a malformed frame from rank %d", r);
                return false;
            }
            (*all)[r].assign(frame.begin() + 4, frame.end());
        }
        net::Writer w;
        for (int r = 0; r < world_; ++r) {
            w.U64((*all)[r].size());
            w.Raw((*all)[r].data(), (*all)[r].size());
        }
        for (int r = 1; r < world_; ++r) {
            if (!net::SendFrame(worker_fds_[r], w.bytes(), timeout_ms_)) {
                LOG_ERROR("bootstrap: AllGather could not reach rank %d", r);
                return false;
            }
        }
        return true;
    }
    net::Writer w;
    w.U32(kGatherMagic);
    w.Raw(mine.data(), mine.size());
    if (!net::SendFrame(master_fd_, w.bytes(), timeout_ms_)) {
        LOG_ERROR("bootstrap: AllGather send failed on rank %d", rank_);
        return false;
    }
    std::vector<uint8_t> frame;
    if (!net::RecvFrame(master_fd_, &frame, timeout_ms_)) {
        LOG_ERROR("bootstrap: AllGather receive failed on rank %d", rank_);
        return false;
    }
    net::Reader rd(frame);
    for (int r = 0; r < world_; ++r) {
        uint64_t n = 0;
        if (!rd.U64(&n) || n > frame.size()) return false;
        (*all)[r].resize(n);
        if (!rd.Raw((*all)[r].data(), n)) return false;
    }
    return true;
}

bool Bootstrap::Broadcast(int root, std::vector<uint8_t>* data) {
    std::vector<std::vector<uint8_t>> all;
    std::vector<uint8_t> mine = (rank_ == root) ? *data : std::vector<uint8_t>();
    if (!AllGather(mine, &all)) return false;
    *data = all[root];
    return true;
}

bool Bootstrap::Barrier() {
    std::vector<std::vector<uint8_t>> all;
    return AllGather({}, &all);
}

void Bootstrap::Close() {
    for (int& fd : worker_fds_) net::CloseFd(&fd);
    worker_fds_.clear();
    net::CloseFd(&master_fd_);
    ready_ = false;
}

}  // namespace bccl
