// Host-memory communicator engine (CommConfig::device == -1).
//
// This is the reference's own domain (collectives on host buffers between processes,
// OriginCCL README.md:3), rebuilt around one shared-memory segment per machine instead of
// per-edge rings:
//   * every machine's local ranks map one memfd segment (created by the local leader and
//     passed with SCM_RIGHTS). Per channel it holds a staging slot per global rank, a
//     result area and a generation barrier; directed SPSC rings carry Send/Recv;
//   * collectives are two-shot in shared memory: copy-in, barrier, each local rank reduces
//     1/L of the chunk over all slots, barrier, copy-out. Machines (distinguished by
//     CommConfig::get_hostname, so one host can emulate several) are joined by their
//     leaders over TCP, reducing in machine order so every rank gets identical bits;
//   * channels (CommConfig::n_channels) are worker threads that each own a contiguous
//     slice of every payload, with their own barrier and sockets -- the reference's
//     MultiThreadExecutor channels (src/executor/multi_thread_executor.cpp:141-198);
//   * Send/Recv are progressed by a polling or epoll executor over the TrySend/TryRecv
//     contract (src/executor/polling_executor.cpp, epoll_executor.cpp), FIFO per peer.
#pragma once

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <functional>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include "bccl/types.h"
#include "host/transport.h"

namespace bccl {

class Bootstrap;
class FdPasser;

struct MachineView {
    int local_rank = 0;
    int local_size = 1;
    std::vector<int> local_ranks;      // global ranks on this machine, ascending
    int machine_index = 0;
    int machine_count = 1;
    std::vector<int> machine_leaders;  // lowest rank of each machine, machine order
    std::vector<int> machine_of;       // per global rank
    std::vector<int> local_index_of;   // per global rank: index within its machine
    std::vector<std::vector<int>> machine_ranks;
};

struct alignas(64) ShmBarrier {
    std::atomic<uint32_t> count;
    char pad0[60];
    std::atomic<uint32_t> gen;
    char pad1[60];
};

class HostEngine {
public:
    HostEngine() = default;
    ~HostEngine() { Finalize(); }

    // data_listen_fd: this rank's TCP listener announced in NodeInfo::data_port (borrowed).
    bool Init(const CommConfig& cfg, Bootstrap* bs, FdPasser* fp, const std::vector<NodeInfo>& nodes,
              const MachineView& view, int data_listen_fd);
    void Finalize();
    bool Execute(const std::vector<CollTask>& sorted);

    int n_channels() const { return n_channels_; }
    const char* p2p_transport_name(int peer) const;
    const char* executor_name() const { return epoll_ ? "epoll" : "polling"; }
    bool zero_copy_p2p() const { return cma_; }
    unsigned long long zero_copy_transfers() const { return cma_transfers_.load(); }
    // Host trace (BCCL_TRACE=<events per channel>): writes the phases recorded so far (copy-in,
    // barrier waits, reduction, leader exchange, copy-out) as Chrome-trace duration events, one
    // track per channel, and clears them. Call while no collective runs. Returns events written.
    long DumpTrace(const char* path);

    enum TraceEvent : uint16_t { kTrSliceBegin = 1, kTrCopyIn, kTrBarrier, kTrReduce, kTrExchange, kTrCopyOut, kTrSliceEnd };

private:
    struct TraceRec {
        uint64_t t_ns;
        uint16_t event;
        uint16_t func;
        uint32_t slice;
    };
    size_t trace_cap_ = 0;  // events kept per channel; 0 = tracing off
    void Mark(int ch, TraceEvent ev) {
        if (trace_cap_ == 0) return;
        Channel& c = chans_[ch];
        if (c.trace.size() < trace_cap_)
            c.trace.push_back({static_cast<uint64_t>(std::chrono::duration_cast<std::chrono::nanoseconds>(
                                   std::chrono::steady_clock::now().time_since_epoch()).count()),
                               static_cast<uint16_t>(ev), c.trace_func, c.trace_slice});
    }

    // Chunks alternate between two buffer sets. A chunk's buffers are last read within that
    // chunk, and every chunk crosses at least one barrier after its first write, so when a rank
    // starts chunk k (having passed chunk k-1's first barrier) every rank has finished chunk
    // k-2, the previous user of the same set: no barrier is needed at the end of a chunk.
    struct Channel {
        ShmBarrier* barrier = nullptr;
        char* slots = nullptr;   // current set: [world][slot_bytes]
        char* result = nullptr;  // current set: [slot_bytes]
        char* set_slots[2] = {nullptr, nullptr};
        char* set_result[2] = {nullptr, nullptr};
        unsigned chunks = 0;     // chunks started on this channel (same count on every rank)
        std::vector<std::unique_ptr<TcpTransport>> leader_links;  // per machine (leaders only)
        std::vector<char> scratch;                                // leader-private receive space
        std::vector<TraceRec> trace;                              // BCCL_TRACE (this channel's thread only)
        uint16_t trace_func = 0;
        uint32_t trace_slice = 0;
    };

    struct WorkUnit {
        const CollTask* task;
        size_t e0, e1;  // element range of this slice
    };
    std::vector<std::vector<WorkUnit>> PlanChannels(const std::vector<const CollTask*>& work) const;
    size_t split_bytes_ = 1u << 20;
    bool RunSlice(int ch, const CollTask& t, size_t e0, size_t e1);
    bool AllReduceSlice(int ch, const CollTask& t, size_t e0, size_t e1, bool reduce_only);
    bool BroadcastSlice(int ch, const CollTask& t, size_t e0, size_t e1);
    bool AllGatherSlice(int ch, const CollTask& t, size_t e0, size_t e1);
    bool ReduceScatterSlice(int ch, const CollTask& t, size_t e0, size_t e1);
    bool Barrier(int ch);
    // Leaders: send `send[m]` (bytes[m]) to machine m's leader and receive `recv[m]` from it,
    // for every m in `peers`, all concurrently.
    bool LeaderRingAllReduce(int ch, char* buf, size_t count, DataType dt, ReduceOp op, float scale);
    bool LeaderExchange(int ch, const std::vector<int>& peers, const std::vector<const void*>& send,
                        const std::vector<size_t>& send_bytes, const std::vector<void*>& recv,
                        const std::vector<size_t>& recv_bytes);
    bool RunP2p(const std::vector<CollTask>& tasks);
    // Runs fn(ch) for every channel in `busy` and waits: channel inline_ch (one of them) on the
    // calling thread, the others on their channel threads; channels not in `busy` stay asleep.
    bool RunOnChannels(const std::function<bool(int)>& fn, int inline_ch, const std::vector<int>& busy);
    void WorkerLoop(int ch);
    char* Slot(int ch, int rank) { return chans_[ch].slots + static_cast<size_t>(rank) * slot_bytes_; }
    // Switches channel ch to the other buffer set; called at the start of every chunk.
    void NextBuffers(int ch) {
        Channel& c = chans_[ch];
        const unsigned k = c.chunks++ & 1u;
        c.slots = c.set_slots[k];
        c.result = c.set_result[k];
    }

    int rank_ = 0;
    int world_ = 1;
    int listen_fd_ = -1;
    MachineView view_;
    int n_channels_ = 1;
    size_t slot_bytes_ = 1u << 20;
    size_t ring_bytes_ = 1u << 20;
    int timeout_ms_ = 30000;
    bool epoll_ = false;
    bool inited_ = false;

    void* seg_ = nullptr;
    size_t seg_bytes_ = 0;
    std::vector<Channel> chans_;
    std::vector<std::unique_ptr<Transport>> p2p_send_;  // per peer
    std::vector<std::unique_ptr<Transport>> p2p_recv_;  // per peer (same object for TCP)
    std::vector<std::shared_ptr<TcpTransport>> p2p_tcp_;
    // Single-copy Send/Recv within a machine (messages of at least cma_bytes_): the receiver
    // reads the sender's buffer with process_vm_readv; the sender completes when acked.
    bool SetupCma(Bootstrap* bs);
    bool cma_ = false;
    size_t cma_bytes_ = 256u << 10;
    uint64_t cma_probe_ = 0;
    std::atomic<uint64_t>* cma_acks_ = nullptr;  // [sender local][receiver local], in the segment
    std::vector<uint64_t> cma_sent_;             // per peer: zero-copy messages sent
    std::atomic<uint64_t> cma_transfers_{0};     // completed zero-copy receives (statistics)

    // Channel worker pool.
    std::vector<std::thread> workers_;
    std::mutex mu_;
    std::condition_variable cv_done_;
    // Per channel: jobs handed to its worker so far, and the worker's wake-up. Only channels
    // with work in a job are woken (not the one the caller runs itself, not idle ones).
    std::unique_ptr<std::atomic<uint64_t>[]> chan_seq_;
    std::unique_ptr<std::condition_variable[]> cv_chan_;
    std::function<bool(int)> job_;
    std::atomic<int> job_pending_{0};
    std::atomic<bool> job_ok_{true};
    std::atomic<bool> stop_{false};
    // Spin before blocking on the condition variables (dispatch and completion), when every
    // channel thread and the caller of every local rank can have a core (BCCL_HOST_SPIN forces).
    bool spin_ = false;
    std::atomic<bool> aborted_{false};

public:
    // Makes every wait of the in-flight and later operations give up (thread-safe).
    void Abort() { aborted_.store(true); }
};

}  // namespace bccl
