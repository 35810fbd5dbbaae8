#include "bccl/communicator.h"

#include <cstdio>

#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <map>

#include "core/bootstrap.h"
#include "core/env.h"
#include "core/fdpass.h"
#include "core/logger.h"
#include "core/nvtx.h"
#include "core/net.h"
#include "core/planner.h"
#include "core/watchdog.h"
#include "device/device_engine.h"
#include "host/host_engine.h"

namespace bccl {

std::string DefaultHostname() { return net::Hostname(); }

size_t DataTypeSize(DataType dtype) {
    switch (dtype) {
    case DataType::FLOAT32: return 4;
    case DataType::FLOAT64: return 8;
    case DataType::INT32: return 4;
    case DataType::INT64: return 8;
    case DataType::BF16: return 2;
    case DataType::FP16: return 2;
    }
    return 0;
}

const char* DataTypeName(DataType dtype) {
    switch (dtype) {
    case DataType::FLOAT32: return "float32";
    case DataType::FLOAT64: return "float64";
    case DataType::INT32: return "int32";
    case DataType::INT64: return "int64";
    case DataType::BF16: return "bfloat16";
    case DataType::FP16: return "float16";
    }
    return "unknown";
}

const char* ReduceOpName(ReduceOp op) {
    switch (op) {
    case ReduceOp::SUM: return "sum";
    case ReduceOp::MAX: return "max";
    case ReduceOp::MIN: return "min";
    case ReduceOp::AVG: return "avg";
    }
    return "unknown";
}

const char* CollFuncName(CollFunc f) {
    switch (f) {
    case CollFunc::AllReduce: return "allreduce";
    case CollFunc::Broadcast: return "broadcast";
    case CollFunc::Reduce: return "reduce";
    case CollFunc::AllGather: return "allgather";
    case CollFunc::ReduceScatter: return "reducescatter";
    case CollFunc::Send: return "send";
    case CollFunc::Recv: return "recv";
    }
    return "unknown";
}

const char* AlgoName(Algo a) {
    switch (a) {
    case Algo::kAuto: return "auto";
    case Algo::kOneShot: return "oneshot";
    case Algo::kTwoShot: return "twoshot";
    case Algo::kNvls: return "nvls";
    case Algo::kRing: return "ring";
    case Algo::kHybrid: return "hybrid";
    case Algo::kLL: return "ll";
    }
    return "unknown";
}

Communicator::Communicator() : planner_(new Planner()) {}

Communicator::~Communicator() { Finalize(); }

bool Communicator::GetUniqueId(UniqueId& unique_id) { return MakeUniqueId(unique_id, true); }

bool Communicator::MakeUniqueId(UniqueId& unique_id, bool from_env) {
    if (have_unique_id_) {
        LOG_ERROR("GetUniqueId called twice on the same communicator");
        return false;
    }
    // BCCL_MASTER=<addr>:<port> (set by a multi-node launcher): the id is known in advance, so
    // rank 0 listens on that port and announces that address; no id file is exchanged.
    uint16_t want = 0;
    std::string ip;
    const char* m = from_env ? std::getenv("BCCL_MASTER") : nullptr;
    if (m != nullptr) {
        const std::string ms(m);
        const size_t colon = ms.rfind(':');
        const long p = colon == std::string::npos ? -1 : std::atol(ms.c_str() + colon + 1);
        if (p <= 0 || p > 65535) {
            LOG_ERROR("BCCL_MASTER must be <address>:<port>, got '%s'", m);
            return false;
        }
        want = static_cast<uint16_t>(p);
        ip = ms.substr(0, colon);
    }
    uint16_t port = 0;
    bootstrap_listen_fd_ = net::Listen(want, &port);
    if (bootstrap_listen_fd_ < 0) return false;
    if (ip.empty()) ip = net::LocalIpAddress();
    unique_id = UniqueId{};
    strncpy(unique_id.ip_addr, ip.c_str(), sizeof(unique_id.ip_addr) - 1);
    unique_id.port = port;
    have_unique_id_ = true;
    return true;
}

bool Communicator::Split(int color, int key, Communicator* out) {
    if (!inited_ || out == nullptr) {
        LOG_ERROR("Split needs an initialised communicator and an output");
        return false;
    }
    struct Entry {
        int32_t color, key, rank;
    };
    Entry me{color, key, config_.rank};
    std::vector<uint8_t> blob(sizeof(me));
    std::memcpy(blob.data(), &me, sizeof(me));
    std::vector<std::vector<uint8_t>> all;
    if (!bootstrap_->AllGather(blob, &all)) return false;
    std::vector<Entry> members;
    for (const auto& b : all) {
        if (b.size() != sizeof(Entry)) return false;
        Entry e;
        std::memcpy(&e, b.data(), sizeof(e));
        if (color >= 0 && e.color == color) members.push_back(e);
    }
    std::stable_sort(members.begin(), members.end(),
                     [](const Entry& a, const Entry& b) { return a.key != b.key ? a.key < b.key : a.rank < b.rank; });
    int new_rank = -1;
    for (size_t i = 0; i < members.size(); ++i)
        if (members[i].rank == config_.rank) new_rank = static_cast<int>(i);
    // Each color's first member creates the new unique id; everyone learns every color's id.
    UniqueId id;
    bool ok = true;
    std::vector<uint8_t> mine;
    if (color >= 0 && new_rank == 0) {
        ok = out->MakeUniqueId(id, false);
        const int32_t c = color;
        mine.resize(sizeof(c) + sizeof(id));
        std::memcpy(mine.data(), &c, sizeof(c));
        std::memcpy(mine.data() + sizeof(c), &id, sizeof(id));
    }
    std::vector<std::vector<uint8_t>> ids;
    if (!bootstrap_->AllGather(mine, &ids) || !ok) return false;
    if (color < 0) return true;
    bool found = false;
    for (const auto& b : ids) {
        int32_t c = -1;
        if (b.size() != sizeof(c) + sizeof(id)) continue;
        std::memcpy(&c, b.data(), sizeof(c));
        if (c == color) {
            std::memcpy(&id, b.data() + sizeof(c), sizeof(id));
            found = true;
        }
    }
    if (!found) return false;
    CommConfig cfg = config_;
    cfg.rank = new_rank;
    cfg.world_size = static_cast<int>(members.size());
    cfg.unique_id = id;
    return out->Init(cfg);
}

bool Communicator::Init(const CommConfig& cfg) {
    if (inited_) {
        LOG_ERROR("Init called twice");
        return false;
    }
    if (cfg.world_size <= 0 || cfg.rank < 0 || cfg.rank >= cfg.world_size) {
        LOG_ERROR("invalid rank %d / world size %d", cfg.rank, cfg.world_size);
        return false;
    }
    config_ = cfg;
    if (config_.get_hostname == nullptr) config_.get_hostname = DefaultHostname;
    user_stream_ = cfg.stream;
    has_user_stream_ = cfg.stream != nullptr;
    if (cfg.world_size > 1 && cfg.rank == 0 && bootstrap_listen_fd_ < 0) {
        LOG_ERROR("rank 0 must call GetUniqueId before Init");
        return false;
    }
    // Every listener exists before the bootstrap announces it (no port races).
    fdpass_.reset(new FdPasser());
    // A one-rank communicator has no unique id to share; its socket name must still be unique
    // among the communicators of this host (several may live in one process).
    static std::atomic<unsigned> solo_serial{0};
    const std::string ns = cfg.world_size > 1
                               ? std::string(cfg.unique_id.ip_addr) + ":" + std::to_string(cfg.unique_id.port)
                               : "solo." + std::to_string(static_cast<long>(getpid())) + "." +
                                     std::to_string(solo_serial.fetch_add(1));
    if (!fdpass_->Listen(ns, cfg.rank)) return false;
    uint16_t data_port = 0;
    if (cfg.device < 0) {
        data_listen_fd_ = net::Listen(0, &data_port);
        if (data_listen_fd_ < 0) return false;
    }
    NodeInfo me;
    me.rank = cfg.rank;
    me.ip_addr = net::LocalIpAddress();
    me.data_port = data_port;
    me.hostname = config_.get_hostname();
    me.device = cfg.device;
    me.pid = static_cast<int>(getpid());
    bootstrap_.reset(new Bootstrap());
    if (!bootstrap_->Run(config_, me, bootstrap_listen_fd_, &all_nodes_)) return false;
    if (cfg.world_size > 1 && EnvInt("BCCL_WATCHDOG", 1) != 0) {
        watchdog_.reset(new Watchdog());
        if (!watchdog_->Start(config_, bootstrap_listen_fd_, bootstrap_.get(), [this](int) { Abort(); })) {
            watchdog_.reset();
            return false;
        }
    }

    // Local and machine views: machines are numbered by first appearance of their hostname;
    // a machine's leader is its lowest rank.
    std::map<std::string, int> machine_id;
    std::vector<int> machine_of(cfg.world_size);
    std::vector<std::vector<int>> machine_ranks;
    for (int r = 0; r < cfg.world_size; ++r) {
        auto it = machine_id.find(all_nodes_[r].hostname);
        int m;
        if (it == machine_id.end()) {
            m = static_cast<int>(machine_ranks.size());
            machine_id[all_nodes_[r].hostname] = m;
            machine_ranks.emplace_back();
        } else {
            m = it->second;
        }
        machine_of[r] = m;
        machine_ranks[m].push_back(r);
    }
    machine_index_ = machine_of[cfg.rank];
    machine_count_ = static_cast<int>(machine_ranks.size());
    local_ranks_ = machine_ranks[machine_index_];
    local_size_ = static_cast<int>(local_ranks_.size());
    local_rank_ = static_cast<int>(std::find(local_ranks_.begin(), local_ranks_.end(), cfg.rank) - local_ranks_.begin());
    machine_leaders_.clear();
    for (const auto& mr : machine_ranks) machine_leaders_.push_back(mr.front());

    if (cfg.device >= 0) {
        if (machine_count_ != 1) {
            LOG_ERROR("device communicators span one NVSwitch node; %d machines were found", machine_count_);
            return false;
        }
        device_.reset(new DeviceEngine());
        if (!device_->Init(config_, bootstrap_.get(), fdpass_.get(), planner_.get())) {
            device_.reset();
            return false;
        }
    } else {
        MachineView v;
        v.local_rank = local_rank_;
        v.local_size = local_size_;
        v.local_ranks = local_ranks_;
        v.machine_index = machine_index_;
        v.machine_count = machine_count_;
        v.machine_leaders = machine_leaders_;
        v.machine_of = machine_of;
        v.machine_ranks = machine_ranks;
        v.local_index_of.assign(cfg.world_size, 0);
        for (const auto& mr : machine_ranks)
            for (size_t i = 0; i < mr.size(); ++i) v.local_index_of[mr[i]] = static_cast<int>(i);
        CommConfig hc = config_;
        if (hc.n_channels <= 0) {
            // Up to 4 channels (the reference's default), fewer where this machine's ranks would
            // otherwise run more busy channel threads than it has cores (each rank's calling
            // thread runs one channel itself); every rank takes the minimum, since the channel
            // plan must be the same everywhere.
            const long cores = std::max(1L, sysconf(_SC_NPROCESSORS_ONLN));
            const int want = static_cast<int>(std::max(1L, std::min(4L, cores / std::max(1, local_size_))));
            std::vector<uint8_t> mine(1, static_cast<uint8_t>(want));
            std::vector<std::vector<uint8_t>> all;
            if (!bootstrap_->AllGather(mine, &all)) return false;
            int agreed = want;
            for (const auto& a : all)
                if (!a.empty()) agreed = std::min<int>(agreed, a[0]);
            hc.n_channels = std::max(1, agreed);
        }
        host_.reset(new HostEngine());
        if (!host_->Init(hc, bootstrap_.get(), fdpass_.get(), all_nodes_, v, data_listen_fd_)) {
            host_.reset();
            return false;
        }
    }
    inited_ = true;
    return true;
}

void Communicator::Finalize() {
    std::lock_guard<std::mutex> lk(mu_);
    if (watchdog_) watchdog_->Stop();  // goodbye first: this rank's teardown is not a failure
    watchdog_.reset();
    if (device_) device_->Finalize();
    device_.reset();
    if (host_) host_->Finalize();
    host_.reset();
    if (bootstrap_) bootstrap_->Close();
    bootstrap_.reset();
    if (fdpass_) fdpass_->Close();
    fdpass_.reset();
    net::CloseFd(&bootstrap_listen_fd_);
    net::CloseFd(&data_listen_fd_);
    pending_.clear();
    group_depth_ = 0;
    inited_ = false;
}

int Communicator::GetNChannels() const {
    if (host_) return host_->n_channels();
    return config_.n_channels > 0 ? config_.n_channels : 4;
}

void Communicator::GroupStart() { ++group_depth_; }

bool Communicator::GroupEnd() {
    if (group_depth_ <= 0) {
        LOG_ERROR("GroupEnd without GroupStart");
        return false;
    }
    if (--group_depth_ > 0) return true;  // inner GroupEnd: nothing runs
    return Flush();
}

bool Communicator::Submit(const CollTask& task) {
    if (!inited_) {
        LOG_ERROR("communicator used before Init");
        return false;
    }
    const bool valid = IsP2p(task.func) ? planner_->ValidateP2p(task, config_.rank, config_.world_size)
                                        : planner_->ValidateCollectiveTask(task, config_.rank, config_.world_size);
    if (!valid) return false;  // rejected before it is queued, even inside a group
    pending_.push_back(task);
    if (group_depth_ > 0) return true;
    return Flush();
}

bool Communicator::Flush() {
    std::vector<CollTask> tasks;
    tasks.swap(pending_);
    if (tasks.empty()) return true;
    if (failed_) {
        LOG_ERROR("communicator is in an error state after an earlier failure");
        return false;
    }
    // One task was validated by Submit and needs no ordering: the per-call path of every
    // ungrouped collective skips the sort.
    if (tasks.size() > 1 && !planner_->SortTasks(tasks, config_.rank, config_.world_size)) return false;
    char range[48] = "bccl";
    if (NvtxEnabled()) {
        if (tasks.size() == 1) {
            std::snprintf(range, sizeof(range), "bccl:%s", CollFuncName(tasks[0].func));
        } else {
            std::snprintf(range, sizeof(range), "bccl:group(%zu)", tasks.size());
        }
    }
    NvtxRange nvtx(range);
    bool ok;
    if (device_) {
        cudaStream_t s = static_cast<cudaStream_t>(has_user_stream_ ? user_stream_ : device_->internal_stream());
        ok = device_->Execute(tasks, s);
        if (ok && !has_user_stream_) ok = device_->Synchronize(s);
    } else {
        ok = host_->Execute(tasks);
    }
    if (!ok) failed_ = true;
    return ok;
}

bool Communicator::AllReduce(const void* send_buf, void* recv_buf, size_t count, DataType dtype, ReduceOp op) {
    return AllReduceScaled(send_buf, recv_buf, count, dtype, op, 1.0f);
}

bool Communicator::AllReduceScaled(const void* send_buf, void* recv_buf, size_t count, DataType dtype, ReduceOp op,
                                   float scale) {
    CollTask t;
    t.func = CollFunc::AllReduce;
    t.send_buf = send_buf;
    t.recv_buf = recv_buf;
    t.count = count;
    t.dtype = dtype;
    t.op = op;
    t.scale = scale;
    return Submit(t);
}

bool Communicator::Broadcast(void* buffer, size_t count, DataType dtype, int root) {
    return BroadcastTo(buffer, buffer, count, dtype, root);
}

bool Communicator::BroadcastTo(const void* send_buf, void* recv_buf, size_t count, DataType dtype, int root) {
    CollTask t;
    t.func = CollFunc::Broadcast;
    t.send_buf = send_buf;
    t.recv_buf = recv_buf;
    t.count = count;
    t.dtype = dtype;
    t.root = root;
    return Submit(t);
}

bool Communicator::AllGather(const void* send_buf, void* recv_buf, size_t count, DataType dtype) {
    CollTask t;
    t.func = CollFunc::AllGather;
    t.send_buf = send_buf;
    t.recv_buf = recv_buf;
    t.count = count;
    t.dtype = dtype;
    return Submit(t);
}

bool Communicator::Reduce(const void* send_buf, void* recv_buf, size_t count, DataType dtype, ReduceOp op, int root) {
    CollTask t;
    t.func = CollFunc::Reduce;
    t.send_buf = send_buf;
    t.recv_buf = recv_buf;
    t.count = count;
    t.dtype = dtype;
    t.op = op;
    t.root = root;
    return Submit(t);
}

bool Communicator::ReduceScatter(const void* send_buf, void* recv_buf, size_t count, DataType dtype, ReduceOp op) {
    CollTask t;
    t.func = CollFunc::ReduceScatter;
    t.send_buf = send_buf;
    t.recv_buf = recv_buf;
    t.count = count;
    t.dtype = dtype;
    t.op = op;
    return Submit(t);
}

bool Communicator::Send(const void* buffer, size_t count, DataType dtype, int peer) {
    CollTask t;
    t.func = CollFunc::Send;
    t.send_buf = buffer;
    t.count = count;
    t.dtype = dtype;
    t.peer = peer;
    return Submit(t);
}

bool Communicator::Recv(void* buffer, size_t count, DataType dtype, int peer) {
    CollTask t;
    t.func = CollFunc::Recv;
    t.recv_buf = buffer;
    t.count = count;
    t.dtype = dtype;
    t.peer = peer;
    return Submit(t);
}

void Communicator::SetStream(void* stream) {
    user_stream_ = stream;
    has_user_stream_ = true;
}
void Communicator::ClearStream() {
    user_stream_ = nullptr;
    has_user_stream_ = false;
}
void* Communicator::GetStream() const {
    if (has_user_stream_) return user_stream_;
    return device_ ? static_cast<void*>(device_->internal_stream()) : nullptr;
}

int Communicator::AsyncError() const {
    if (device_) {
        const int code = device_->PeekDeviceError();
        if (code != 0) return code;
    }
    return failed_ ? 1 : 0;
}

bool Communicator::Synchronize() {
    if (!device_) return true;
    cudaStream_t s = static_cast<cudaStream_t>(GetStream());
    bool ok = device_->Synchronize(s);
    if (!ok) failed_ = true;
    return ok;
}

void* Communicator::SymmetricAlloc(size_t bytes) { return device_ ? device_->SymAlloc(bytes) : nullptr; }
bool Communicator::SymmetricFree(void* ptr) { return device_ ? device_->SymFree(ptr) : false; }
bool Communicator::RegisterBuffer(void* ptr, size_t bytes) { return device_ ? device_->RegisterBuffer(ptr, bytes) : true; }
bool Communicator::DeregisterBuffer(void* ptr) { return device_ ? device_->DeregisterBuffer(ptr) : true; }
bool Communicator::Barrier() { return bootstrap_ && bootstrap_->Barrier(); }

long Communicator::DumpTrace(const char* path) {
    if (device_) return device_->DumpTrace(path);
    if (host_) return host_->DumpTrace(path);
    return -1;
}

void Communicator::Abort() {
    failed_ = true;
    if (device_) device_->Abort();
    if (host_) host_->Abort();
}
bool Communicator::NvlsEnabled() const { return device_ && device_->nvls_enabled(); }
const char* Communicator::LastAlgorithm() const { return device_ ? device_->last_algo() : "host"; }
unsigned long long Communicator::KernelLaunches() const { return device_ ? device_->launches() : 0; }
const char* Communicator::P2pTransportName(int peer) const {
    if (host_) return host_->p2p_transport_name(peer);
    return device_ ? "nccl" : "none";
}
const char* Communicator::HostExecutorName() const { return host_ ? host_->executor_name() : "cuda-stream"; }
bool Communicator::HostZeroCopyP2p() const { return host_ && host_->zero_copy_p2p(); }
unsigned long long Communicator::HostZeroCopyTransfers() const { return host_ ? host_->zero_copy_transfers() : 0; }

}  // namespace bccl
