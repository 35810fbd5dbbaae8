// Executor of the device communicator: turns a sorted batch of tasks into kernel launches.
//
// The reference's executors decide how CPU threads wait on sockets (OriginCCL
// src/executor/*.cpp); here waiting happens inside the kernels (bounded flag spins) and
// the host only enqueues. A batch becomes:
//   * consecutive one-shot collectives -> ONE push-engine launch (the whole group; the
//     reference's dynamic executor and its per-slice control broadcast become the kernel's
//     CTA-owns-piece rule);
//   * each large collective -> one NVLS or two-shot launch, in sorted order;
//   * all Send/Recv -> one NCCL group on a side stream forked from the caller's stream before
//     the collectives launch and joined back after them, so a group's point-to-point traffic
//     overlaps its collective kernels (the collectives then leave SMs free for NCCL's kernels).
// Every rank derives the same launches from the same sorted batch, so no control message
// is needed at run time.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <map>
#include <string>
#include <vector>

#include "bccl/types.h"
#include "core/planner.h"
#include "device/dev_types.h"
#include "device/nccl_p2p.h"
#include "device/symmem.h"

namespace bccl {

class Bootstrap;
class FdPasser;

class DeviceEngine {
public:
    DeviceEngine() = default;
    ~DeviceEngine() { Finalize(); }

    bool Init(const CommConfig& cfg, Bootstrap* bs, FdPasser* fp, const Planner* planner);
    void Finalize();

    // Enqueues the batch on `stream` (collectives first, in order, then P2P).
    bool Execute(const std::vector<CollTask>& sorted, cudaStream_t stream);
    // Reads the host-mapped error record; false if any kernel reported a failure.
    bool CheckDeviceError();
    // The host-mapped error record's code (kDevOk, kDevTimeout, kDevAborted, kDevBadArgs) as the
    // kernels left it so far, without synchronising (ncclCommGetAsyncError's role).
    int PeekDeviceError() const { return err_host_ ? static_cast<const volatile ErrorRecord*>(err_host_)->code : kDevOk; }
    bool Synchronize(cudaStream_t stream);
    void Abort();
    // Runs the bounded-wait self-test; returns the error code it recorded (kDevTimeout
    // expected) and clears the record so the communicator stays usable.
    int WaitProbe(int timeout_ms);
    // Transport probe (no peer participation needed; run it while peers are idle):
    // mode 0 local copy, 1 write to `peer`, 2 read from `peer`, 3 multimem.st. Returns GB/s
    // of the copied bytes, or a negative value on error.
    double BandwidthProbe(int mode, int peer, size_t bytes, int ctas, int iters);
    // Copies the DevState counters (see bcclDebugDeviceState) after a device synchronize.
    bool ReadState(unsigned long long* out);
    // Device trace (BCCL_TRACE=<records>): writes the records gathered so far as a Chrome
    // trace (chrome://tracing, Perfetto) and resets the buffer. Returns records written.
    long DumpTrace(const char* path);

    // Collective allocation of memory every rank can address directly (NVLS-bound when
    // available); AllReduce on such a buffer in place skips the staging copies.
    void* SymAlloc(size_t bytes);
    // Whether [p, p + bytes) lies in a multicast-bound symmetric user buffer; *mc = its
    // multicast address.
    bool UserMulticast(const void* p, size_t bytes, char** mc) const;
    bool SymFree(void* ptr);
    // Registration of existing device memory (cudaMalloc'd, e.g. PyTorch tensors); collective:
    // every rank passes its own buffer of the same size, registrations in the same order. The
    // peers map it with CUDA IPC (one mapping per allocation, shared by the registrations that
    // fall in it). A collective whose buffers lie in registered or symmetric memory, at the same
    // offset of the same registration on every rank, then runs over peer memory without staging.
    bool RegisterBuffer(void* ptr, size_t bytes);
    bool DeregisterBuffer(void* ptr);
    // Every rank's address of [p, p + bytes) when it lies in registered or symmetric memory.
    bool PeerPointers(const void* p, size_t bytes, char* (&peers)[kMaxRanks]) const;

    // Fused tensor-parallel GEMMs (bf16). x_local [ms,K] -> y [nranks*ms, n] = act(AllGather(x) * w^T)
    // with w [n,K]; h [nranks*ms, K] -> out [ms, n] = this rank's rows of sum_ranks(h * w^T).
    bool TpAllGatherGemm(const void* x_local, const void* w, void* y, int ms, int k, int n, int act,
                         cudaStream_t stream);
    bool TpGemmReduceScatter(const void* h, const void* w, void* out, int ms, int k, int n, cudaStream_t stream);

    cudaStream_t internal_stream() const { return stream_; }
    bool nvls_enabled() const { return nvls_.mc != nullptr; }
    const DevComm& dev_comm() const { return dc_; }
    unsigned long long launches() const { return launches_.load(); }
    const char* last_algo() const { return last_algo_; }
    int device() const { return device_; }
    const char* nccl_version() const { return p2p_.version(); }

private:
    bool FlushBatch(std::vector<WorkItem>* batch, unsigned long long* stream_bytes, cudaStream_t stream);
    // Send/Recv of one group with the native kernel (p2p_native.cu).
    bool RunNativeP2p(const std::vector<CollTask>& tasks, cudaStream_t stream);
    bool LaunchLarge(const CollTask& t, const AlgoChoice& c, cudaStream_t stream);
    bool ExecuteCollectives(const std::vector<CollTask>& sorted, cudaStream_t stream);
    bool RunP2p(const std::vector<CollTask>& p2p, cudaStream_t stream);
    // SMs left to NCCL's point-to-point kernels while a mixed group's collectives run.
    static constexpr int kP2pReservedSms = 32;
    // Collectives of a group up to this many bytes per rank run in the group's push launch.
    static constexpr size_t kGroupPushMaxBytes = 1u << 20;

    int rank_ = 0;
    int nranks_ = 1;
    int device_ = -1;
    int max_ctas_ = 0;
    int num_sms_ = 148;
    Algo forced_ = Algo::kAuto;
    // Environment knobs of the per-call path, read at Init.
    long knob_max_ctas_ = 0;
    bool knob_zero_copy_ = true;
    size_t knob_p2p_zc_min_ = 1u << 20;
    int knob_pipe_slots_ = 3;
    int knob_pipe_lag_ = 1;           // BCCL_PIPE_LAG: barrier lag of the pipelined kernels (1 or 2)
    long knob_pipe_rounds_ = 0;  // 0: by size
    long knob_pipe_min_chunk_ = 4 << 20;
    long knob_pipe_kind_ = -1;
    double knob_hybrid_frac_ = 0.6;  // BCCL_HYBRID_NVLS_PERMILLE / 1000: bytes of a hybrid AllReduce through NVLS
    long knob_hybrid_ctas_ = 0;      // BCCL_HYBRID_NVLS_CTAS: its NVLS CTAs (0: the same share of the CTAs)
    size_t knob_ll_max_ = 512u << 10;  // BCCL_LL_MAX_BYTES: largest ungrouped AllReduce on the low-latency kernel
    size_t knob_ll_block_max_ = 256u << 10;  // BCCL_LL_BLOCK_MAX_BYTES: same for AllGather / ReduceScatter blocks
    bool knob_local_copy_ = true;  // BCCL_LOCAL_COPY=0: one-rank collectives back on the push kernel
    bool knob_p2p_native_ = false; // BCCL_P2P_NATIVE=1: Send/Recv on the native kernel instead of NCCL
    const Planner* planner_ = nullptr;
    Bootstrap* bs_ = nullptr;
    SymmetricMemory sm_;
    SymBuffer uc_;
    SymBuffer nvls_;
    std::vector<SymBuffer> user_bufs_;
    struct RegBuffer {
        char* ptr[kMaxRanks] = {};  // every rank's registered buffer, mapped here
        size_t bytes = 0;
        std::string ipc[kMaxRanks];  // the peers' IPC handles (keys of ipc_maps_)
    };
    std::vector<RegBuffer> reg_bufs_;
    struct IpcMapping {
        void* base = nullptr;
        int refs = 0;
    };
    std::map<std::string, IpcMapping> ipc_maps_;  // a peer's allocation, opened once
    void ReleaseIpc(const std::string& key);
    DevState* state_ = nullptr;
    ErrorRecord* err_host_ = nullptr;
    int* abort_host_ = nullptr;
    DevComm dc_{};
    unsigned long long data_bytes_ = 0;
    cudaStream_t stream_ = nullptr;
    NcclP2p p2p_;
    // Side stream and fork/join events of the NCCL Send/Recv of a mixed group.
    cudaStream_t p2p_stream_ = nullptr;
    cudaEvent_t p2p_fork_ = nullptr, p2p_join_ = nullptr;
    bool EnsureP2pStream();
    std::atomic<unsigned long long> launches_{0};
    const char* last_algo_ = "none";
    // Tensor-parallel workspaces (symmetric, double-buffered by call parity) and call counters.
    SymBuffer tp_xg_[2];
    size_t tp_xg_bytes_ = 0;
    SymBuffer tp_rs_[2];
    size_t tp_rs_bytes_ = 0;
    unsigned long long tp_ag_calls_ = 0, tp_rs_calls_ = 0;
    int* tp_err_ = nullptr;
    bool EnsureTpBuffer(SymBuffer (&bufs)[2], size_t* have, size_t need, bool multicast);
    TraceRecord* trace_ = nullptr;
    unsigned int* trace_count_ = nullptr;
    unsigned int kernel_serial_ = 0;
    bool inited_ = false;
};

}  // namespace bccl
