// C interface over bccl::Communicator (see bccl/c_api.h).
#include "bccl/c_api.h"

#include <cstring>
#include <string>

#include "bccl/communicator.h"
#include "core/logger.h"
#include "core/planner.h"
#include "device/device_engine.h"
#include "kernels/gemm.h"
#include "kernels/ll_epoch.h"
#include "kernels/p2p_sched.h"

#include <mutex>

struct bcclComm {
    bccl::Communicator comm;
};

namespace {

// Logical-machine hostname injection for bcclConfig::logical_machine_size: Init calls the
// hostname function synchronously on the calling thread, so a thread-local carries the name.
thread_local std::string t_logical_host;
std::string LogicalHostname() { return t_logical_host; }

int Fail() { return 1; }

void ApplyStream(bcclComm_t c, uintptr_t stream, int has_stream) {
    if (!c->comm.IsDevice()) return;
    if (has_stream) {
        c->comm.SetStream(reinterpret_cast<void*>(stream));
    } else {
        c->comm.ClearStream();
    }
}

bccl::CollTask MakeTask(bccl::CollFunc f, const void* send, void* recv, size_t count, int dtype, int op, int root,
                        int peer, float scale, int algo) {
    bccl::CollTask t;
    t.func = f;
    t.send_buf = send;
    t.recv_buf = recv;
    t.count = count;
    t.dtype = static_cast<bccl::DataType>(dtype);
    t.op = static_cast<bccl::ReduceOp>(op);
    t.root = root;
    t.peer = peer;
    t.scale = scale;
    t.algo = static_cast<bccl::Algo>(algo);
    return t;
}

}  // namespace

extern "C" {

int bcclCommCreate(bcclComm_t* comm) {
    if (comm == nullptr) return Fail();
    *comm = new bcclComm();
    return 0;
}

int bcclGetUniqueId(bcclComm_t comm, char ip_addr[64], uint16_t* port) {
    bccl::UniqueId id;
    if (comm == nullptr || !comm->comm.GetUniqueId(id)) return Fail();
    memcpy(ip_addr, id.ip_addr, sizeof(id.ip_addr));
    *port = id.port;
    return 0;
}

int bcclCommInit(bcclComm_t comm, const bcclConfig* cfg) {
    if (comm == nullptr || cfg == nullptr) return Fail();
    bccl::CommConfig c;
    c.rank = cfg->rank;
    c.world_size = cfg->world_size;
    memcpy(c.unique_id.ip_addr, cfg->ip_addr, sizeof(c.unique_id.ip_addr));
    c.unique_id.ip_addr[sizeof(c.unique_id.ip_addr) - 1] = '\0';
    c.unique_id.port = cfg->port;
    c.n_channels = cfg->n_channels;
    c.device = cfg->device;
    c.buffer_bytes = cfg->buffer_bytes;
    c.timeout_ms = cfg->timeout_ms;
    c.enable_nvls = cfg->enable_nvls != 0;
    c.enable_nccl_p2p = cfg->enable_nccl_p2p != 0;
    if (cfg->logical_machine_size > 0) {
        t_logical_host = "logical-machine-" + std::to_string(cfg->rank / cfg->logical_machine_size);
        c.get_hostname = LogicalHostname;
    }
    return comm->comm.Init(c) ? 0 : Fail();
}

int bcclCommFinalize(bcclComm_t comm) {
    if (comm == nullptr) return Fail();
    comm->comm.Finalize();
    return 0;
}

int bcclCommDestroy(bcclComm_t comm) {
    delete comm;
    return 0;
}

int bcclCommSplit(bcclComm_t comm, int color, int key, bcclComm_t* out) {
    if (comm == nullptr || out == nullptr) return Fail();
    *out = nullptr;
    bcclComm_t child = new bcclComm();
    if (!comm->comm.Split(color, key, &child->comm)) {
        delete child;
        return Fail();
    }
    if (color < 0) {
        delete child;
        return 0;
    }
    *out = child;
    return 0;
}

const char* bcclGetLastError(void) { return bccl::LastErrorMessage(); }

const char* bcclVersion(void) { return "bccl 0.1.0 (sm_100a)"; }

int bcclCommInfo(bcclComm_t comm, int* rank, int* world, int* local_rank, int* local_size, int* machine_index,
                 int* machine_count, int* n_channels) {
    if (comm == nullptr) return Fail();
    const bccl::Communicator& c = comm->comm;
    if (rank) *rank = c.GetRank();
    if (world) *world = c.GetWorldSize();
    if (local_rank) *local_rank = c.GetLocalRank();
    if (local_size) *local_size = c.GetLocalSize();
    if (machine_index) *machine_index = c.GetMachineIndex();
    if (machine_count) *machine_count = c.GetMachineCount();
    if (n_channels) *n_channels = c.GetNChannels();
    return 0;
}

int bcclCommLocalRanks(bcclComm_t comm, int* out, int max) {
    if (comm == nullptr) return -1;
    const auto& v = comm->comm.GetLocalRanks();
    for (int i = 0; i < max && i < static_cast<int>(v.size()); ++i) out[i] = v[i];
    return static_cast<int>(v.size());
}

int bcclCommMachineLeaders(bcclComm_t comm, int* out, int max) {
    if (comm == nullptr) return -1;
    const auto& v = comm->comm.GetMachineLeaders();
    for (int i = 0; i < max && i < static_cast<int>(v.size()); ++i) out[i] = v[i];
    return static_cast<int>(v.size());
}

int bcclCommNvlsEnabled(bcclComm_t comm) { return comm && comm->comm.NvlsEnabled() ? 1 : 0; }
const char* bcclCommLastAlgorithm(bcclComm_t comm) { return comm ? comm->comm.LastAlgorithm() : ""; }
unsigned long long bcclCommKernelLaunches(bcclComm_t comm) { return comm ? comm->comm.KernelLaunches() : 0; }
const char* bcclCommP2pTransport(bcclComm_t comm, int peer) { return comm ? comm->comm.P2pTransportName(peer) : ""; }
const char* bcclCommHostExecutor(bcclComm_t comm) { return comm ? comm->comm.HostExecutorName() : ""; }
unsigned long long bcclCommHostZeroCopyTransfers(bcclComm_t comm, int* enabled) {
    if (comm == nullptr) return 0;
    if (enabled) *enabled = comm->comm.HostZeroCopyP2p() ? 1 : 0;
    return comm->comm.HostZeroCopyTransfers();
}

int bcclGroupStart(bcclComm_t comm) {
    if (comm == nullptr) return Fail();
    comm->comm.GroupStart();
    return 0;
}

int bcclGroupEnd(bcclComm_t comm, uintptr_t stream, int has_stream) {
    if (comm == nullptr) return Fail();
    ApplyStream(comm, stream, has_stream);
    return comm->comm.GroupEnd() ? 0 : Fail();
}

#define BCCL_SUBMIT(task)                        \
    if (comm == nullptr) return Fail();          \
    ApplyStream(comm, stream, has_stream);       \
    return comm->comm.Submit(task) ? 0 : Fail();

int bcclAllReduce(bcclComm_t comm, const void* send, void* recv, size_t count, int dtype, int op, float scale, int algo,
                  uintptr_t stream, int has_stream) {
    BCCL_SUBMIT(MakeTask(bccl::CollFunc::AllReduce, send, recv, count, dtype, op, 0, -1, scale, algo));
}

int bcclAllReduceMany(bcclComm_t comm, int n, const void* const* send, void* const* recv, const size_t* counts,
                      int dtype, int op, float scale, int grouped, uintptr_t stream, int has_stream) {
    if (comm == nullptr || n < 0 || (n > 0 && (send == nullptr || recv == nullptr || counts == nullptr))) return Fail();
    ApplyStream(comm, stream, has_stream);
    if (grouped) comm->comm.GroupStart();
    bool ok = true;
    for (int i = 0; i < n && ok; ++i) {
        ok = comm->comm.Submit(MakeTask(bccl::CollFunc::AllReduce, send[i], recv[i], counts[i], dtype, op, 0, -1, scale,
                                        0));
    }
    if (grouped) ok = comm->comm.GroupEnd() && ok;  // always leave the group
    return ok ? 0 : Fail();
}

int bcclBroadcast(bcclComm_t comm, const void* send, void* recv, size_t count, int dtype, int root, int algo,
                  uintptr_t stream, int has_stream) {
    BCCL_SUBMIT(MakeTask(bccl::CollFunc::Broadcast, send ? send : recv, recv, count, dtype, 0, root, -1, 1.0f, algo));
}

int bcclReduce(bcclComm_t comm, const void* send, void* recv, size_t count, int dtype, int op, int root, int algo,
               uintptr_t stream, int has_stream) {
    BCCL_SUBMIT(MakeTask(bccl::CollFunc::Reduce, send, recv, count, dtype, op, root, -1, 1.0f, algo));
}

int bcclAllGather(bcclComm_t comm, const void* send, void* recv, size_t count, int dtype, uintptr_t stream,
                  int has_stream) {
    return bcclAllGatherAlgo(comm, send, recv, count, dtype, 0, stream, has_stream);
}

int bcclAllGatherAlgo(bcclComm_t comm, const void* send, void* recv, size_t count, int dtype, int algo,
                      uintptr_t stream, int has_stream) {
    BCCL_SUBMIT(MakeTask(bccl::CollFunc::AllGather, send, recv, count, dtype, 0, 0, -1, 1.0f, algo));
}

int bcclReduceScatter(bcclComm_t comm, const void* send, void* recv, size_t count, int dtype, int op,
                      uintptr_t stream, int has_stream) {
    return bcclReduceScatterAlgo(comm, send, recv, count, dtype, op, 0, stream, has_stream);
}

int bcclReduceScatterAlgo(bcclComm_t comm, const void* send, void* recv, size_t count, int dtype, int op, int algo,
                          uintptr_t stream, int has_stream) {
    BCCL_SUBMIT(MakeTask(bccl::CollFunc::ReduceScatter, send, recv, count, dtype, op, 0, -1, 1.0f, algo));
}

int bcclSend(bcclComm_t comm, const void* buf, size_t count, int dtype, int peer, uintptr_t stream, int has_stream) {
    BCCL_SUBMIT(MakeTask(bccl::CollFunc::Send, buf, nullptr, count, dtype, 0, 0, peer, 1.0f, 0));
}

int bcclRecv(bcclComm_t comm, void* buf, size_t count, int dtype, int peer, uintptr_t stream, int has_stream) {
    BCCL_SUBMIT(MakeTask(bccl::CollFunc::Recv, nullptr, buf, count, dtype, 0, 0, peer, 1.0f, 0));
}

int bcclCommGetAsyncError(bcclComm_t comm, int* code) {
    if (comm == nullptr || code == nullptr) return Fail();
    *code = comm->comm.AsyncError();
    return 0;
}
int bcclSynchronize(bcclComm_t comm) { return comm && comm->comm.Synchronize() ? 0 : Fail(); }
int bcclBarrier(bcclComm_t comm) { return comm && comm->comm.Barrier() ? 0 : Fail(); }
int bcclCommAbort(bcclComm_t comm) {
    if (comm == nullptr) return Fail();
    comm->comm.Abort();
    return 0;
}
void* bcclSymmetricAlloc(bcclComm_t comm, size_t bytes) { return comm ? comm->comm.SymmetricAlloc(bytes) : nullptr; }
int bcclSymmetricFree(bcclComm_t comm, void* ptr) { return comm && comm->comm.SymmetricFree(ptr) ? 0 : Fail(); }
int bcclCommRegister(bcclComm_t comm, void* ptr, size_t bytes) {
    return comm && comm->comm.RegisterBuffer(ptr, bytes) ? 0 : Fail();
}
int bcclCommDeregister(bcclComm_t comm, void* ptr) { return comm && comm->comm.DeregisterBuffer(ptr) ? 0 : Fail(); }

int bcclDebugWaitProbe(bcclComm_t comm, int timeout_ms) {
    if (comm == nullptr || comm->comm.device_engine() == nullptr) return -1;
    return comm->comm.device_engine()->WaitProbe(timeout_ms);
}

double bcclDebugBandwidth(bcclComm_t comm, int mode, int peer, size_t bytes, int ctas, int iters) {
    if (comm == nullptr || comm->comm.device_engine() == nullptr) return -1.0;
    return comm->comm.device_engine()->BandwidthProbe(mode, peer, bytes, ctas, iters);
}

int bcclDebugDeviceState(bcclComm_t comm, unsigned long long* out) {
    if (comm == nullptr || out == nullptr || comm->comm.device_engine() == nullptr) return -1;
    return comm->comm.device_engine()->ReadState(out) ? 0 : -1;
}

long bcclTraceDump(bcclComm_t comm, const char* path) {
    if (comm == nullptr || path == nullptr) return -1;
    return comm->comm.DumpTrace(path);
}

namespace {
std::mutex g_gemm_mu;
int* g_gemm_err[64] = {};
int* GemmErrWord() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_gemm_mu);
    if (g_gemm_err[dev] == nullptr) {
        if (cudaMalloc(&g_gemm_err[dev], sizeof(int)) != cudaSuccess) return nullptr;
        cudaMemset(g_gemm_err[dev], 0, sizeof(int));
    }
    return g_gemm_err[dev];
}
}  // namespace

int bcclGemmBf16(const void* A, const void* B, void* C, int M, int N, int K, int ldc, int act, void* stream) {
    int* err = GemmErrWord();
    if (err == nullptr) {
        LOG_ERROR("gemm: no device error word");
        return 1;
    }
    cudaError_t e = bccl::LaunchGemmBf16(A, B, C, M, N, K, ldc, act, err, 0, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        LOG_ERROR("gemm launch failed: %s (M=%d N=%d K=%d)", cudaGetErrorString(e), M, N, K);
        return 1;
    }
    return 0;
}

int bcclTpAllGatherGemm(bcclComm_t comm, const void* x, const void* w, void* y, int ms, int k, int n, int act,
                        uintptr_t stream, int has_stream) {
    if (comm == nullptr || comm->comm.device_engine() == nullptr) {
        LOG_ERROR("bcclTpAllGatherGemm needs a device communicator");
        return 1;
    }
    ApplyStream(comm, stream, has_stream);
    bccl::DeviceEngine* d = comm->comm.device_engine();
    cudaStream_t s = static_cast<cudaStream_t>(comm->comm.GetStream());
    if (!d->TpAllGatherGemm(x, w, y, ms, k, n, act, s)) return 1;
    if (!has_stream && !d->Synchronize(s)) return 1;
    return 0;
}

int bcclTpGemmReduceScatter(bcclComm_t comm, const void* h, const void* w, void* out, int ms, int k, int n,
                            uintptr_t stream, int has_stream) {
    if (comm == nullptr || comm->comm.device_engine() == nullptr) {
        LOG_ERROR("bcclTpGemmReduceScatter needs a device communicator");
        return 1;
    }
    ApplyStream(comm, stream, has_stream);
    bccl::DeviceEngine* d = comm->comm.device_engine();
    cudaStream_t s = static_cast<cudaStream_t>(comm->comm.GetStream());
    if (!d->TpGemmReduceScatter(h, w, out, ms, k, n, s)) return 1;
    if (!has_stream && !d->Synchronize(s)) return 1;
    return 0;
}

int bcclGemmUsesPair(void) { return bccl::GemmUsesPair() ? 1 : 0; }
int bcclGemmTileWidth(int m, int n) { return bccl::GemmTileWidth(m, n); }

int bcclGemmCheckError(void) {
    int* err = GemmErrWord();
    if (err == nullptr) return -1;
    int v = 0;
    cudaDeviceSynchronize();
    cudaMemcpy(&v, err, sizeof(int), cudaMemcpyDeviceToHost);
    cudaMemset(err, 0, sizeof(int));
    return v;
}

int bcclP2pChannels(unsigned long long pair_bytes) { return bccl::P2pChannels(pair_bytes); }
unsigned int bcclLLEpoch(unsigned long long seq) { return bccl::LLEpoch(seq); }

int bcclP2pPlan(const unsigned long long* bytes, int nops, int nch, int ch, int max_out, int* op_out,
                unsigned long long* off_out, unsigned long long* len_out) {
    if (nops < 0 || nch < 1 || nch > bccl::kP2pMaxChannels || ch < 0 || ch >= nch || max_out < 0) return -1;
    std::vector<bccl::P2pNativeOp> ops(static_cast<size_t>(nops));
    for (int i = 0; i < nops; ++i) ops[i] = bccl::P2pNativeOp{nullptr, bytes[i]};
    bccl::P2pCursor cur(0, nch, ch);
    int n = 0, i = 0;
    unsigned long long off = 0, len = 0;
    while (n < max_out && cur.next(ops.data(), nops, &i, &off, &len)) {
        op_out[n] = i;
        off_out[n] = off;
        len_out[n] = len;
        ++n;
    }
    return n;
}

int bcclPlannerSort(int rank, int world, int n, const int* func, const size_t* count, const int* dtype, const int* op,
                    const int* root, const int* peer, int* order) {
    std::vector<bccl::CollTask> tasks(n);
    static const char kMark = 0;
    for (int i = 0; i < n; ++i) {
        tasks[i] = MakeTask(static_cast<bccl::CollFunc>(func[i]), &kMark, const_cast<char*>(&kMark), count[i], dtype[i],
                            op[i], root[i], peer[i], 1.0f, 0);
        // Tag each task with its input index through the scale field (planner ignores it).
        tasks[i].scale = static_cast<float>(i);
    }
    bccl::Planner planner;
    if (!planner.SortTasks(tasks, rank, world)) return Fail();
    for (int i = 0; i < n; ++i) order[i] = static_cast<int>(tasks[i].scale);
    return 0;
}

int bcclPlannerP2pRound(int func, int rank, int peer, int world) {
    return bccl::Planner::P2pRoundOf(static_cast<bccl::CollFunc>(func), rank, peer, world);
}

int bcclPlannerValidate(int rank, int world, int func, size_t count, int dtype, int op, int root, int peer,
                        int has_send, int has_recv) {
    static char buf[16];
    bccl::CollTask t = MakeTask(static_cast<bccl::CollFunc>(func), has_send ? buf : nullptr, has_recv ? buf : nullptr,
                                count, dtype, op, root, peer, 1.0f, 0);
    bccl::Planner planner;
    bool ok = bccl::IsP2p(t.func) ? planner.ValidateP2p(t, rank, world) : planner.ValidateCollectiveTask(t, rank, world);
    return ok ? 0 : Fail();
}

int bcclPlannerChoose(int func, int dtype, int op, size_t bytes, int world, int nvls_ok, int max_ctas, int* algo,
                      int* ctas) {
    bccl::Planner planner;
    bccl::AlgoChoice c = planner.ChooseAlgo(static_cast<bccl::CollFunc>(func), static_cast<bccl::DataType>(dtype),
                                            static_cast<bccl::ReduceOp>(op), bytes, world, nvls_ok != 0, max_ctas,
                                            bccl::Algo::kAuto);
    *algo = static_cast<int>(c.algo);
    *ctas = c.ctas;
    return 0;
}

}  // extern "C"
