// The communicator: the library's public C++ API.
//
// Method names, arguments and semantics follow the reference (OriginCCL
// include/communicator.h:19-75, docs/layers/communicator.md):
//   * GetUniqueId (rank 0 only; binds the bootstrap listener held until Finalize), Init,
//     Finalize; the local/machine views;
//   * AllReduce / Broadcast / Reduce / AllGather / ReduceScatter, Send / Recv;
//   * GroupStart / GroupEnd nest; only the outermost GroupEnd executes, once, for the
//     whole batch; invalid operations return false before they are queued;
//   * count 0 succeeds with null buffers; Reduce's non-root recv may be null; AllGather's
//     output is ordered by rank; ReduceScatter takes N*count inputs; in place is allowed;
//   * AVG is SUM divided by the rank count.
// A communicator is used by one thread at a time (like the reference's and NCCL's): calls from
// several threads, e.g. from autograd hooks during backward, must not overlap.
// Device communicators (CommConfig::device >= 0) take device pointers; with no stream in
// the config every call blocks until its result is ready (the reference's contract); with
// a stream, calls only enqueue (NCCL's contract) and errors surface on the next call or
// in Synchronize().
#pragma once

#include <atomic>
#include <cstddef>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "bccl/types.h"

namespace bccl {

class Bootstrap;
class FdPasser;
class Planner;
class DeviceEngine;
class HostEngine;
class Watchdog;

class Communicator {
public:
    Communicator();
    ~Communicator();
    Communicator(const Communicator&) = delete;
    Communicator& operator=(const Communicator&) = delete;

    bool GetUniqueId(UniqueId& unique_id);
    bool Init(const CommConfig& cfg);
    void Finalize();
    // Collective over this communicator (like MPI_Comm_split / ncclCommSplit): the ranks that
    // pass the same color >= 0 form a new communicator in *out, ranked by (key, rank); it has the
    // same kind (host or device), channels and timeouts. A negative color joins none (*out is
    // left untouched). This communicator stays usable.
    bool Split(int color, int key, Communicator* out);

    int GetRank() const { return config_.rank; }
    int GetWorldSize() const { return config_.world_size; }
    int GetNChannels() const;
    int GetLocalRank() const { return local_rank_; }
    int GetLocalSize() const { return local_size_; }
    const std::vector<int>& GetLocalRanks() const { return local_ranks_; }
    bool IsSingleMachine() const { return machine_count_ == 1; }
    int GetMachineIndex() const { return machine_index_; }
    int GetMachineCount() const { return machine_count_; }
    const std::vector<int>& GetMachineLeaders() const { return machine_leaders_; }

    void GroupStart();
    bool GroupEnd();

    bool AllReduce(const void* send_buf, void* recv_buf, size_t count, DataType dtype, ReduceOp op);
    bool Broadcast(void* buffer, size_t count, DataType dtype, int root);
    bool AllGather(const void* send_buf, void* recv_buf, size_t count, DataType dtype);
    bool Reduce(const void* send_buf, void* recv_buf, size_t count, DataType dtype, ReduceOp op, int root);
    bool ReduceScatter(const void* send_buf, void* recv_buf, size_t count, DataType dtype, ReduceOp op);
    bool Send(const void* buffer, size_t count, DataType dtype, int peer);
    bool Recv(void* buffer, size_t count, DataType dtype, int peer);

    // ---- extensions
    // AllReduce with a fused multiplier on the result (data-parallel gradient scaling).
    bool AllReduceScaled(const void* send_buf, void* recv_buf, size_t count, DataType dtype, ReduceOp op, float scale);
    // Out-of-place Broadcast (root reads send_buf, every rank writes recv_buf).
    bool BroadcastTo(const void* send_buf, void* recv_buf, size_t count, DataType dtype, int root);
    // Submits a prepared task (used by the C API and bindings).
    bool Submit(const CollTask& task);
    // Device communicators: later calls enqueue on `stream` and return without waiting
    // (any cudaStream_t, including 0 = the legacy default stream). ClearStream() returns to
    // the internal stream with blocking calls.
    void SetStream(void* stream);
    void ClearStream();
    void* GetStream() const;
    bool Synchronize();
    // Without synchronising: 0, or the code a device kernel recorded (1 timeout, 2 aborted,
    // 3 bad arguments); host communicators report 1 once a host operation has failed.
    int AsyncError() const;
    // Device communicators: collective allocation of peer-addressable memory.
    void* SymmetricAlloc(size_t bytes);
    bool SymmetricFree(void* ptr);
    // Device communicators: collective registration of existing device memory (e.g. a
    // cudaMalloc'd gradient buffer); every rank registers its own buffer of the same size, in the
    // same order. AllReduce / AllGather / ReduceScatter of at least 1 MiB whose buffers lie in
    // registered memory, at the same offset on every rank, then read and write the peers'
    // buffers directly instead of staging. Host communicators accept and ignore it.
    // Each rank decides from its own registrations whether a call runs zero-copy, so a call's
    // buffers must be registered on every rank or on none: deregister (collectively) before the
    // memory is freed or handed to other tensors, since a reused range would still count as
    // registered on this rank only.
    bool RegisterBuffer(void* ptr, size_t bytes);
    bool DeregisterBuffer(void* ptr);
    bool Barrier();
    // Stops the operations in flight from any thread: host waits return at once, device waits
    // within ~1 ms (kernels record kDevAborted and return). The communicator stays in the error
    // state; only Finalize is meaningful afterwards.
    void Abort();
    bool IsDevice() const { return config_.device >= 0; }
    bool NvlsEnabled() const;
    const char* LastAlgorithm() const;
    unsigned long long KernelLaunches() const;
    const char* P2pTransportName(int peer) const;
    const char* HostExecutorName() const;
    // Host communicators: whether large Send/Recv within a machine go single-copy (cross-memory
    // attach), and how many such messages this rank has received.
    bool HostZeroCopyP2p() const;
    unsigned long long HostZeroCopyTransfers() const;
    const Planner& planner() const { return *planner_; }
    DeviceEngine* device_engine() { return device_.get(); }
    // With BCCL_TRACE=<records> at Init: writes the recorded device events (device
    // communicators) or host channel phases (host communicators) as Chrome-trace JSON and
    // clears them. Returns the number of events, or -1 when tracing is off.
    long DumpTrace(const char* path);

private:
    bool MakeUniqueId(UniqueId& unique_id, bool from_env);
    bool Flush();

    CommConfig config_;
    bool inited_ = false;
    std::atomic<bool> failed_{false};
    int bootstrap_listen_fd_ = -1;
    int data_listen_fd_ = -1;
    bool have_unique_id_ = false;
    std::unique_ptr<Bootstrap> bootstrap_;
    std::unique_ptr<FdPasser> fdpass_;
    std::unique_ptr<Planner> planner_;
    std::unique_ptr<DeviceEngine> device_;
    std::unique_ptr<HostEngine> host_;
    std::unique_ptr<Watchdog> watchdog_;
    std::vector<NodeInfo> all_nodes_;
    int group_depth_ = 0;
    std::vector<CollTask> pending_;
    void* user_stream_ = nullptr;
    bool has_user_stream_ = false;
    int local_rank_ = 0;
    int local_size_ = 1;
    std::vector<int> local_ranks_;
    int machine_index_ = 0;
    int machine_count_ = 1;
    std::vector<int> machine_leaders_;
    std::mutex mu_;
};

}  // namespace bccl
