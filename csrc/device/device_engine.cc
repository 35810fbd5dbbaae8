#include "device/device_engine.h"

#include <algorithm>
#include <cstring>

#include "core/bootstrap.h"
#include "core/env.h"
#include "core/logger.h"
#include "core/nvtx.h"
#include "device/cuda_driver.h"
#include <cuda_bf16.h>

#include "kernels/gemm.h"
#include "kernels/launch.h"

namespace bccl {
namespace {

#define CUDA_OK(call, what)                                                              \
    do {                                                                                 \
        cudaError_t _e = (call);                                                         \
        if (_e != cudaSuccess) {                                                         \
            LOG_ERROR("%s failed: %s", what, cudaGetErrorString(_e));                    \
            return false;                                                                \
        }                                                                                \
    } while (0)


size_t RoundDown(size_t x, size_t a) { return x / a * a; }
size_t RoundUp(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Per-peer payload bytes of a collective in the push engine's stream.
size_t PeerPayload(const CollTask& t) { return t.count * DataTypeSize(t.dtype); }

// CTAs for a push-engine launch: few for latency-bound payloads (each CTA pays one
// cross-rank barrier per round), up to one per SM for bandwidth-bound ones.
// One CTA moves ~40 GB/s to peers or to local memory (measured), so a payload needs about one
// CTA per 16 KiB for its copy time to stay near the ~2 us a cross-rank barrier costs; barriers
// are per CTA and run in parallel, so extra CTAs cost flags, not time.
int PushCtas(size_t stream_bytes, int num_sms) {
    return static_cast<int>(std::min<size_t>(std::max<size_t>(1, stream_bytes / (16u << 10)), static_cast<size_t>(num_sms)));
}

}  // namespace

bool DeviceEngine::Init(const CommConfig& cfg, Bootstrap* bs, FdPasser* fp, const Planner* planner) {
    rank_ = cfg.rank;
    nranks_ = cfg.world_size;
    device_ = cfg.device;
    planner_ = planner;
    bs_ = bs;
    max_ctas_ = cfg.n_channels;
    forced_ = Planner::ParseAlgo(EnvStr("BCCL_ALGO", ""));
    CUDA_OK(cudaSetDevice(device_), "cudaSetDevice");
    CUDA_OK(cudaDeviceGetAttribute(&num_sms_, cudaDevAttrMultiProcessorCount, device_), "cudaDeviceGetAttribute");
    const int timeout_ms = cfg.timeout_ms > 0 ? cfg.timeout_ms : static_cast<int>(EnvInt("BCCL_TIMEOUT_MS", 10000));
    if (!sm_.Init(device_, rank_, nranks_, bs, fp, std::max(timeout_ms, 30000), cfg.enable_nvls)) return false;

    data_bytes_ = cfg.buffer_bytes ? cfg.buffer_bytes : static_cast<size_t>(EnvInt("BCCL_BUFFSIZE", 512l << 20));
    data_bytes_ = std::max<size_t>(RoundUp(data_bytes_, 1u << 20), 4u << 20);
    // Control region, data region, then the inboxes of the native Send/Recv.
    if (!sm_.Alloc(kCtrlBytes + data_bytes_ + (nranks_ > 1 ? kP2pRegionBytes + kLLRegionBytes : 0), false, &uc_)) {
        return false;
    }
    // Every flag starts at zero; no peer writes here before the barrier at the end of Init.
    CUDA_OK(cudaMemset(uc_.ptr[rank_], 0, kCtrlBytes), "cudaMemset(control region)");
    const unsigned long long ll_off = nranks_ > 1 ? kCtrlBytes + data_bytes_ + kP2pRegionBytes : 0;
    if (ll_off != 0) CUDA_OK(cudaMemset(uc_.ptr[rank_] + ll_off, 0, kLLRegionBytes), "cudaMemset(LL lines)");
    if (sm_.multicast_supported()) {
        size_t nb = static_cast<size_t>(EnvInt("BCCL_NVLS_BUFFSIZE", 256l << 20));
        if (!sm_.Alloc(nb, true, &nvls_)) return false;
        if (nvls_.mc == nullptr) sm_.Free(&nvls_);
    }
    CUDA_OK(cudaMalloc(&state_, sizeof(DevState)), "cudaMalloc(state)");
    CUDA_OK(cudaMemset(state_, 0, sizeof(DevState)), "cudaMemset(state)");
    CUDA_OK(cudaHostAlloc(&err_host_, sizeof(ErrorRecord), cudaHostAllocMapped), "cudaHostAlloc(err)");
    CUDA_OK(cudaHostAlloc(&abort_host_, sizeof(int), cudaHostAllocMapped), "cudaHostAlloc(abort)");
    memset(err_host_, 0, sizeof(ErrorRecord));
    *abort_host_ = 0;
    ErrorRecord* err_dev = nullptr;
    int* abort_dev = nullptr;
    CUDA_OK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&err_dev), err_host_, 0), "cudaHostGetDevicePointer");
    CUDA_OK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&abort_dev), abort_host_, 0), "cudaHostGetDevicePointer");
    // A blocking stream: the synchronous API runs here, and a blocking stream starts its work
    // only after what the caller queued on the legacy default stream, e.g. a pageable
    // cudaMemcpy whose DMA may still be in flight when that call returns.
    CUDA_OK(cudaStreamCreateWithFlags(&stream_, cudaStreamDefault), "cudaStreamCreate");

    memset(&dc_, 0, sizeof(dc_));
    dc_.rank = rank_;
    dc_.nranks = nranks_;
    for (int p = 0; p < nranks_; ++p) dc_.uc[p] = uc_.ptr[p];
    dc_.nvls_uc = nvls_.mc ? nvls_.ptr[rank_] : nullptr;
    dc_.nvls_mc = nvls_.mc;
    dc_.nvls_bytes = nvls_.mc ? nvls_.bytes : 0;
    dc_.state = state_;
    dc_.err = err_dev;
    dc_.abort = abort_dev;
    dc_.timeout_ns = static_cast<unsigned long long>(timeout_ms) * 1000000ull;
    dc_.spin_wait = EnvInt("BCCL_SPIN_WAIT", 0) != 0 ? 1 : 0;
    // Knobs of the per-call path, read once here (a getenv per call costs microseconds of a
    // small collective's latency). Every rank must agree on the pipeline ones.
    knob_max_ctas_ = EnvInt("BCCL_MAX_CTAS", 0);
    knob_zero_copy_ = EnvInt("BCCL_ZERO_COPY", 1) != 0;
    knob_p2p_zc_min_ = static_cast<size_t>(std::max<long>(16, EnvInt("BCCL_P2P_ZC_MIN_BYTES", 1 << 20)));
    knob_pipe_slots_ = static_cast<int>(std::max<long>(3, std::min<long>(16, EnvInt("BCCL_PIPE_SLOTS", 3))));
    knob_pipe_lag_ = static_cast<int>(std::max<long>(1, std::min<long>(2, EnvInt("BCCL_PIPE_LAG", 1))));
    knob_pipe_rounds_ = EnvInt("BCCL_PIPE_ROUNDS", 0);
    knob_pipe_min_chunk_ = EnvInt("BCCL_PIPE_MIN_CHUNK", 4 << 20);
    knob_pipe_kind_ = EnvInt("BCCL_PIPE_KIND", -1);
    knob_hybrid_frac_ = std::min(0.95, std::max(0.05, EnvInt("BCCL_HYBRID_NVLS_PERMILLE", 600) / 1000.0));
    knob_hybrid_ctas_ = EnvInt("BCCL_HYBRID_NVLS_CTAS", 0);
    // Measured on 2 and 4 x B200 up to 128 KiB: 6.0-9.7 us against 10.5-18.1 us for the push
    // engine and 9.5-16.2 us for NCCL; the one-shot push lost to NCCL from 256 KiB to 1 MiB.
    knob_ll_max_ = static_cast<size_t>(std::max<long>(0, EnvInt("BCCL_LL_MAX_BYTES", 512 << 10)));
    knob_ll_block_max_ = static_cast<size_t>(std::max<long>(0, EnvInt("BCCL_LL_BLOCK_MAX_BYTES", 256 << 10)));
    knob_local_copy_ = EnvInt("BCCL_LOCAL_COPY", 1) != 0;
    knob_p2p_native_ = EnvInt("BCCL_P2P_NATIVE", 0) != 0;
    dc_.data_bytes = data_bytes_;
    dc_.ll_off = ll_off;
    const long trace_cap = EnvInt("BCCL_TRACE", 0);
    if (trace_cap > 0) {
        CUDA_OK(cudaMalloc(&trace_, sizeof(TraceRecord) * static_cast<size_t>(trace_cap)), "cudaMalloc(trace)");
        CUDA_OK(cudaMalloc(&trace_count_, sizeof(unsigned int)), "cudaMalloc(trace count)");
        CUDA_OK(cudaMemset(trace_count_, 0, sizeof(unsigned int)), "cudaMemset(trace count)");
        dc_.trace = trace_;
        dc_.trace_count = trace_count_;
        dc_.trace_cap = static_cast<unsigned int>(trace_cap);
    }
    CUDA_OK(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    if (nranks_ > 1 && cfg.enable_nccl_p2p && !knob_p2p_native_ && !EnvFlag("BCCL_DISABLE_NCCL_P2P")) {
        if (!p2p_.Init(rank_, nranks_, bs)) LOG_WARN("rank %d: Send/Recv unavailable (NCCL init failed)", rank_);
    }
    if (!bs->Barrier()) return false;
    inited_ = true;
    LOG_INFO("rank %d: device engine ready (device %d, data %llu bytes, nvls %s)", rank_, device_, data_bytes_,
             nvls_.mc ? "on" : "off");
    return true;
}

void DeviceEngine::Finalize() {
    if (!inited_) return;
    inited_ = false;
    cudaSetDevice(device_);
    cudaDeviceSynchronize();
    p2p_.Destroy();
    if (p2p_stream_ != nullptr) cudaStreamDestroy(p2p_stream_);
    if (p2p_fork_ != nullptr) cudaEventDestroy(p2p_fork_);
    if (p2p_join_ != nullptr) cudaEventDestroy(p2p_join_);
    p2p_stream_ = nullptr;
    p2p_fork_ = p2p_join_ = nullptr;
    // Nobody may unmap while a peer could still touch our memory.
    if (bs_ != nullptr && bs_->ready()) bs_->Barrier();
    for (SymBuffer& b : user_bufs_) sm_.Free(&b);
    user_bufs_.clear();
    reg_bufs_.clear();
    for (auto& m : ipc_maps_) cudaIpcCloseMemHandle(m.second.base);
    ipc_maps_.clear();
    for (SymBuffer& b : tp_xg_) sm_.Free(&b);
    for (SymBuffer& b : tp_rs_) sm_.Free(&b);
    tp_xg_bytes_ = tp_rs_bytes_ = 0;
    if (tp_err_) cudaFree(tp_err_);
    tp_err_ = nullptr;
    sm_.Free(&nvls_);
    sm_.Free(&uc_);
    if (stream_) cudaStreamDestroy(stream_);
    stream_ = nullptr;
    if (state_) cudaFree(state_);
    state_ = nullptr;
    if (err_host_) cudaFreeHost(err_host_);
    err_host_ = nullptr;
    if (trace_) cudaFree(trace_);
    if (trace_count_) cudaFree(trace_count_);
    trace_ = nullptr;
    trace_count_ = nullptr;
    if (abort_host_) cudaFreeHost(abort_host_);
    abort_host_ = nullptr;
}

bool DeviceEngine::CheckDeviceError() {
    if (err_host_ == nullptr) return false;
    if (tp_err_ != nullptr) {
        int v = 0;
        if (cudaMemcpy(&v, tp_err_, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess && v != 0) {
            cudaMemset(tp_err_, 0, sizeof(int));
            LOG_ERROR("rank %d: a fused tensor-parallel GEMM gave up waiting for a peer", rank_);
            return false;
        }
    }
    const volatile ErrorRecord* e = err_host_;
    if (e->code == kDevOk) return true;
    LOG_ERROR("rank %d: device collective failed (code %d: %s) in CTA %d waiting on rank %d, phase %d, seq %llu, "
              "after %.3f ms",
              rank_, e->code, e->code == kDevTimeout ? "timeout" : e->code == kDevAborted ? "aborted" : "bad args",
              e->cta, e->peer, e->phase, static_cast<unsigned long long>(e->seq), e->waited_ns / 1e6);
    return false;
}

bool DeviceEngine::Synchronize(cudaStream_t stream) {
    cudaError_t e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) {
        LOG_ERROR("rank %d: stream synchronisation failed: %s", rank_, cudaGetErrorString(e));
        return false;
    }
    return CheckDeviceError();
}

bool DeviceEngine::EnsureTpBuffer(SymBuffer (&bufs)[2], size_t* have, size_t need, bool multicast) {
    if (*have >= need) return true;
    cudaDeviceSynchronize();
    if (!bs_->Barrier()) return false;  // no peer may still use the old buffers
    for (SymBuffer& b : bufs) sm_.Free(&b);
    *have = 0;
    for (SymBuffer& b : bufs) {
        if (!sm_.Alloc(need, multicast && sm_.multicast_supported(), &b)) return false;
    }
    *have = need;
    return true;
}

namespace {
bool FillTpCommon(TpArgs* t, const DevComm& dc, int ms, unsigned long long seq) {
    memset(t, 0, sizeof(*t));
    t->rank = dc.rank;
    t->nranks = dc.nranks;
    t->ms = ms;
    t->seq = seq;
    return true;
}
unsigned long long* TpFlags(char* uc_base, size_t off) {
    return reinterpret_cast<unsigned long long*>(uc_base + kTpFlagsOff + off);
}
constexpr size_t kAgCountersOff = 0;         // [kMaxRanks][kTpMaxChunks]
constexpr size_t kRsStartedOff = 8u << 10;   // [kMaxRanks]
constexpr size_t kRsCountersOff = 16u << 10; // [own tiles] (<= 16K tiles)
}  // namespace

bool DeviceEngine::TpAllGatherGemm(const void* x_local, const void* w, void* y, int ms, int k, int n, int act,
                                   cudaStream_t stream) {
    if (!inited_) return false;
    NvtxRange nvtx("bccl:AllGatherGemm");
    cudaSetDevice(device_);
    if (tp_err_ == nullptr) {
        CUDA_OK(cudaMalloc(&tp_err_, sizeof(int)), "cudaMalloc(tp err)");
        CUDA_OK(cudaMemset(tp_err_, 0, sizeof(int)), "cudaMemset(tp err)");
    }
    const int m = ms * nranks_;
    cudaError_t e;
    if (nranks_ == 1) {
        e = LaunchGemmBf16(x_local, w, y, m, n, k, n, act, tp_err_, 0, stream);
    } else {
        // BCCL_TP_MULTICAST=1 pushes each gathered chunk once through the switch (multimem.st)
        // instead of once per peer. Off by default: on 4 x B200 the multicast push ran 4.6% slower
        // (1.636 vs 1.564 ms for a Llama-3-8B-shaped TP=4 MLP block). Read per call (a fused op
        // costs far more than a getenv); the buffer is multicast-bound only if the knob was set
        // when it was allocated, and a buffer without a multicast handle always takes the stores.
        const bool multicast = EnvInt("BCCL_TP_MULTICAST", 0) != 0;
        if (!EnsureTpBuffer(tp_xg_, &tp_xg_bytes_, static_cast<size_t>(m) * k * 2, multicast)) return false;
        const unsigned long long seq = ++tp_ag_calls_;
        const int par = static_cast<int>(seq & 1ull);
        TpArgs t;
        FillTpCommon(&t, dc_, ms, seq);
        t.x_local = x_local;
        for (int p = 0; p < nranks_; ++p) {
            t.xg[p] = tp_xg_[par].ptr[p];
            t.ag_counters_peer[p] = TpFlags(uc_.ptr[p], kAgCountersOff);
        }
        t.ag_counters = TpFlags(uc_.ptr[rank_], kAgCountersOff);
        t.xg_mc = multicast ? tp_xg_[par].mc : nullptr;
        e = LaunchTpGemm(kModeAllGather, x_local, tp_xg_[par].ptr[rank_], w, y, m, n, k, act, tp_err_, t, stream);
    }
    if (e != cudaSuccess) {
        LOG_ERROR("rank %d: AllGather-GEMM launch failed: %s", rank_, cudaGetErrorString(e));
        return false;
    }
    launches_++;
    last_algo_ = "tp_ag_gemm";
    return true;
}

bool DeviceEngine::TpGemmReduceScatter(const void* h, const void* w, void* out, int ms, int k, int n,
                                       cudaStream_t stream) {
    if (!inited_) return false;
    NvtxRange nvtx("bccl:GemmReduceScatter");
    cudaSetDevice(device_);
    if (tp_err_ == nullptr) {
        CUDA_OK(cudaMalloc(&tp_err_, sizeof(int)), "cudaMalloc(tp err)");
        CUDA_OK(cudaMemset(tp_err_, 0, sizeof(int)), "cudaMemset(tp err)");
    }
    const int m = ms * nranks_;
    cudaError_t e;
    if (nranks_ == 1) {
        e = LaunchGemmBf16(h, w, out, m, n, k, n, 0, tp_err_, 0, stream);
    } else {
        if ((static_cast<size_t>(ms) / 128) * ((static_cast<size_t>(n) + 255) / 256) > (16u << 10) / 8) {
            LOG_ERROR("GEMM-ReduceScatter: too many output tiles per rank");
            return false;
        }
        if (!EnsureTpBuffer(tp_rs_, &tp_rs_bytes_, static_cast<size_t>(m) * n * 2, false)) return false;
        const unsigned long long seq = ++tp_rs_calls_;
        const int par = static_cast<int>(seq & 1ull);
        TpArgs t;
        FillTpCommon(&t, dc_, ms, seq);
        for (int p = 0; p < nranks_; ++p) {
            t.rs_stage[p] = reinterpret_cast<__nv_bfloat16*>(tp_rs_[par].ptr[p]);
            t.rs_counters[p] = TpFlags(uc_.ptr[p], kRsCountersOff);
            t.rs_started_peer[p] = TpFlags(uc_.ptr[p], kRsStartedOff);
        }
        t.rs_started = TpFlags(uc_.ptr[rank_], kRsStartedOff);
        t.out = static_cast<__nv_bfloat16*>(out);
        e = LaunchTpGemm(kModeReduceScatter, h, nullptr, w, tp_rs_[par].ptr[rank_], m, n, k, 0, tp_err_, t, stream);
    }
    if (e != cudaSuccess) {
        LOG_ERROR("rank %d: GEMM-ReduceScatter launch failed: %s", rank_, cudaGetErrorString(e));
        return false;
    }
    launches_++;
    last_algo_ = "tp_gemm_rs";
    return true;
}

int DeviceEngine::WaitProbe(int timeout_ms) {
    if (!inited_) return -1;
    cudaSetDevice(device_);
    if (LaunchWaitProbe(dc_, static_cast<unsigned long long>(timeout_ms) * 1000000ull, stream_) != cudaSuccess) return -1;
    if (cudaStreamSynchronize(stream_) != cudaSuccess) return -1;
    launches_++;
    int code = err_host_->code;
    memset(err_host_, 0, sizeof(ErrorRecord));
    return code;
}

bool DeviceEngine::ReadState(unsigned long long* out) {
    if (!inited_) return false;
    cudaSetDevice(device_);
    DevState s;
    if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpy(&s, state_, sizeof(s), cudaMemcpyDeviceToHost) != cudaSuccess) {
        return false;
    }
    out[0] = s.round_seq;
    out[1] = s.barrier_seq;
    out[2] = s.nvls_round_seq;
    out[3] = s.ring_seq;
    out[4] = s.tp_seq;
    out[5] = s.done_ctas;
    return true;
}

double DeviceEngine::BandwidthProbe(int mode, int peer, size_t bytes, int ctas, int iters) {
    if (!inited_ || mode < 0 || mode > 3 || peer < 0 || peer >= nranks_ || ctas <= 0 || ctas > 1024 || iters <= 0)
        return -1.0;
    cudaSetDevice(device_);
    // Both halves of the own data region serve as source/destination; the peer's data region
    // is the remote end. Probes must not overlap a collective on the peer.
    bytes = std::min(RoundDown(bytes, 16), static_cast<size_t>(data_bytes_ / 2));
    char* mine = uc_.ptr[rank_] + kCtrlBytes;
    char* theirs = uc_.ptr[peer] + kCtrlBytes;
    char *dst = mine + data_bytes_ / 2, *src = mine;
    bool mc = false;
    if (mode == 1) dst = theirs;
    if (mode == 2) src = theirs;
    if (mode == 3) {
        if (nvls_.mc == nullptr) return -1.0;
        bytes = std::min(bytes, static_cast<size_t>(nvls_.bytes));
        dst = nvls_.mc;
        mc = true;
    }
    auto launch = [&]() { LaunchBandwidthProbe(dst, src, bytes, mc, ctas, stream_); };
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    launch();  // warm-up
    cudaEventRecord(e0, stream_);
    for (int i = 0; i < iters; ++i) launch();
    cudaEventRecord(e1, stream_);
    cudaError_t err = cudaStreamSynchronize(stream_);
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    launches_ += static_cast<unsigned long long>(iters) + 1;
    if (err != cudaSuccess || ms <= 0) return -1.0;
    return static_cast<double>(bytes) * iters / (ms * 1e-3) / 1e9;
}

long DeviceEngine::DumpTrace(const char* path) {
    if (trace_ == nullptr) return -1;
    cudaSetDevice(device_);
    cudaDeviceSynchronize();
    unsigned int n = 0;
    cudaMemcpy(&n, trace_count_, sizeof(n), cudaMemcpyDeviceToHost);
    n = std::min(n, dc_.trace_cap);
    std::vector<TraceRecord> recs(n);
    if (n) cudaMemcpy(recs.data(), trace_, sizeof(TraceRecord) * n, cudaMemcpyDeviceToHost);
    cudaMemset(trace_count_, 0, sizeof(unsigned int));
    FILE* f = fopen(path, "w");
    if (f == nullptr) return -1;
    static const char* kNames[] = {"?", "begin", "staged", "ready_seen", "reduced", "reduced_seen", "finished",
                                   "barrier", "end", "slot_free"};
    fprintf(f, "{\"traceEvents\":[\n");
    for (unsigned int i = 0; i < n; ++i) {
        const TraceRecord& r = recs[i];
        fprintf(f, "%s{\"name\":\"%s r%u\",\"ph\":\"i\",\"s\":\"t\",\"ts\":%.3f,\"pid\":%d,\"tid\":%u,"
                   "\"args\":{\"kernel\":%u,\"group\":%u,\"round\":%u}}\n",
                i ? "," : "", kNames[r.event < 10 ? r.event : 0], r.round, r.t_ns / 1000.0, rank_, r.cta * 4 + r.group,
                r.kernel, r.group, r.round);
    }
    fprintf(f, "]}\n");
    fclose(f);
    return static_cast<long>(n);
}

void DeviceEngine::Abort() {
    if (abort_host_) *reinterpret_cast<volatile int*>(abort_host_) = 1;
}

bool DeviceEngine::UserMulticast(const void* p, size_t bytes, char** mc) const {
    const char* q = static_cast<const char*>(p);
    for (const SymBuffer& b : user_bufs_) {
        const char* base = b.ptr[rank_];
        if (b.mc != nullptr && q >= base && q + bytes <= base + b.bytes) {
            *mc = b.mc + (q - base);
            return true;
        }
    }
    return false;
}

void* DeviceEngine::SymAlloc(size_t bytes) {
    cudaSetDevice(device_);
    SymBuffer b;
    if (!sm_.Alloc(bytes, true, &b)) return nullptr;
    user_bufs_.push_back(b);
    return b.ptr[rank_];
}

bool DeviceEngine::SymFree(void* ptr) {
    for (size_t i = 0; i < user_bufs_.size(); ++i) {
        if (user_bufs_[i].ptr[rank_] == ptr) {
            cudaDeviceSynchronize();
            if (!bs_->Barrier()) return false;
            sm_.Free(&user_bufs_[i]);
            user_bufs_.erase(user_bufs_.begin() + static_cast<long>(i));
            return true;
        }
    }
    return false;
}

namespace {

// What each rank contributes to a registration: its allocation's IPC handle, where the buffer
// sits in it, and the sizes (checked for agreement).
struct RegBlob {
    uint32_t ok;
    uint32_t pad;
    cudaIpcMemHandle_t handle;
    uint64_t offset;      // buffer - allocation base
    uint64_t bytes;       // registered bytes
    uint64_t alloc_size;  // allocation size
};

}  // namespace

bool DeviceEngine::RegisterBuffer(void* ptr, size_t bytes) {
    if (!inited_) return false;
    cudaSetDevice(device_);
    RegBlob mine;
    std::memset(&mine, 0, sizeof(mine));
    mine.bytes = bytes;
    const DriverApi* d = Driver();
    CUdeviceptr base = 0;
    size_t size = 0;
    bool ok = ptr != nullptr && bytes > 0 && d != nullptr && d->cuMemGetAddressRange != nullptr &&
              d->cuMemGetAddressRange(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) == CUDA_SUCCESS;
    if (ok) {
        mine.offset = reinterpret_cast<uintptr_t>(ptr) - base;
        mine.alloc_size = size;
        ok = mine.offset + bytes <= size;
    }
    if (ok && nranks_ > 1) {
        cudaError_t e = cudaIpcGetMemHandle(&mine.handle, reinterpret_cast<void*>(base));
        if (e != cudaSuccess) {
            LOG_ERROR("rank %d: register: no CUDA IPC handle for %p (%s); memory from cuMemCreate (symmetric "
                      "allocations, expandable segments) cannot be registered",
                      rank_, ptr, cudaGetErrorString(e));
            cudaGetLastError();
            ok = false;
        }
    }
    mine.ok = ok ? 1 : 0;
    std::vector<uint8_t> blob(sizeof(mine));
    std::memcpy(blob.data(), &mine, sizeof(mine));
    std::vector<std::vector<uint8_t>> all;
    if (!bs_->AllGather(blob, &all) || static_cast<int>(all.size()) != nranks_) return false;
    std::vector<RegBlob> info(nranks_);
    bool agree = true;
    for (int q = 0; q < nranks_; ++q) {
        if (all[q].size() != sizeof(RegBlob)) return false;
        std::memcpy(&info[q], all[q].data(), sizeof(RegBlob));
        agree = agree && info[q].ok == 1 && info[q].bytes == bytes;
    }
    if (!agree) {
        LOG_ERROR("rank %d: register: a rank could not export its buffer or the sizes differ", rank_);
        return false;
    }
    RegBuffer rb;
    rb.bytes = bytes;
    rb.ptr[rank_] = static_cast<char*>(ptr);
    bool opened = true;
    for (int q = 0; q < nranks_ && opened; ++q) {
        if (q == rank_) continue;
        std::string key(reinterpret_cast<const char*>(&info[q].handle), sizeof(cudaIpcMemHandle_t));
        auto it = ipc_maps_.find(key);
        if (it == ipc_maps_.end()) {
            void* pb = nullptr;
            cudaError_t e = cudaIpcOpenMemHandle(&pb, info[q].handle, cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess) {
                LOG_ERROR("rank %d: register: cannot map rank %d's buffer (%s)", rank_, q, cudaGetErrorString(e));
                cudaGetLastError();
                opened = false;
                break;
            }
            it = ipc_maps_.emplace(key, IpcMapping{pb, 0}).first;
        }
        it->second.refs++;
        rb.ipc[q] = key;
        rb.ptr[q] = static_cast<char*>(it->second.base) + info[q].offset;
    }
    // Every rank keeps the registration only if every rank mapped every peer.
    std::vector<uint8_t> flag(1, opened ? 1 : 0);
    std::vector<std::vector<uint8_t>> flags;
    bool all_ok = bs_->AllGather(flag, &flags);
    for (const auto& f : flags) all_ok = all_ok && !f.empty() && f[0] == 1;
    if (!all_ok) {
        for (int q = 0; q < nranks_; ++q) {
            if (!rb.ipc[q].empty()) ReleaseIpc(rb.ipc[q]);
        }
        return false;
    }
    reg_bufs_.push_back(rb);
    return true;
}

void DeviceEngine::ReleaseIpc(const std::string& key) {
    auto it = ipc_maps_.find(key);
    if (it == ipc_maps_.end()) return;
    if (--it->second.refs <= 0) {
        cudaIpcCloseMemHandle(it->second.base);
        ipc_maps_.erase(it);
    }
}

bool DeviceEngine::DeregisterBuffer(void* ptr) {
    for (size_t i = 0; i < reg_bufs_.size(); ++i) {
        if (reg_bufs_[i].ptr[rank_] != ptr) continue;
        cudaSetDevice(device_);
        cudaDeviceSynchronize();
        if (!bs_->Barrier()) return false;  // no peer still reads or writes through the mapping
        for (int q = 0; q < nranks_; ++q) {
            if (!reg_bufs_[i].ipc[q].empty()) ReleaseIpc(reg_bufs_[i].ipc[q]);
        }
        reg_bufs_.erase(reg_bufs_.begin() + static_cast<long>(i));
        return true;
    }
    LOG_ERROR("rank %d: deregister: %p is not a registered buffer", rank_, ptr);
    return false;
}

bool DeviceEngine::PeerPointers(const void* p, size_t bytes, char* (&peers)[kMaxRanks]) const {
    const char* q = static_cast<const char*>(p);
    for (const RegBuffer& b : reg_bufs_) {
        const char* base = b.ptr[rank_];
        if (q >= base && q + bytes <= base + b.bytes) {
            for (int r = 0; r < nranks_; ++r) peers[r] = b.ptr[r] + (q - base);
            return true;
        }
    }
    for (const SymBuffer& b : user_bufs_) {
        const char* base = b.ptr[rank_];
        if (q >= base && q + bytes <= base + b.bytes) {
            for (int r = 0; r < nranks_; ++r) peers[r] = b.ptr[r] + (q - base);
            return true;
        }
    }
    return false;
}

bool DeviceEngine::FlushBatch(std::vector<WorkItem>* batch, unsigned long long* stream_bytes, cudaStream_t stream) {
    if (batch->empty()) return true;
    // The push engine owns the first half of the UC data region (two halves x N sources).
    const unsigned long long slot = RoundDown(data_bytes_ / 2 / (2ull * nranks_), 256);
    size_t i = 0;
    while (i < batch->size()) {
        size_t n = std::min<size_t>(kPushMaxItems, batch->size() - i);
        // Re-base this launch's stream offsets at zero.
        std::vector<WorkItem> part(batch->begin() + static_cast<long>(i), batch->begin() + static_cast<long>(i + n));
        const unsigned long long base = part.front().stream_off;
        for (WorkItem& w : part) w.stream_off -= base;
        const WorkItem& last = part.back();
        unsigned long long bytes = last.stream_off + RoundUp(last.count * DataTypeSize(static_cast<DataType>(last.dtype)), 16);
        int ctas = PushCtas(std::min<unsigned long long>(bytes, slot), num_sms_);
        if (max_ctas_ > 0) ctas = std::min(ctas, max_ctas_);
        const long env_max = knob_max_ctas_;
        if (env_max > 0) ctas = std::min<int>(ctas, static_cast<int>(env_max));
        dc_.kernel_serial = ++kernel_serial_;
        cudaError_t e = LaunchPushEngine(dc_, part.data(), static_cast<int>(n), bytes, slot, ctas, stream);
        if (e != cudaSuccess) {
            LOG_ERROR("rank %d: push-engine launch failed: %s", rank_, cudaGetErrorString(e));
            return false;
        }
        launches_++;
        i += n;
    }
    last_algo_ = "oneshot";
    batch->clear();
    *stream_bytes = 0;
    return true;
}

bool DeviceEngine::LaunchLarge(const CollTask& t, const AlgoChoice& c, cudaStream_t stream) {
    cudaError_t e = cudaSuccess;
    const int dt = static_cast<int>(t.dtype), op = static_cast<int>(t.op);
    const size_t bytes = t.count * DataTypeSize(t.dtype);
    const unsigned long long q = 16ull * nranks_;
    // The slot ring must be 2L+1 deep for a barrier lag of L (ar_pipe.cu); every NVLS launch kind
    // uses the same slot count, so their rings line up.
    const int lag = knob_pipe_lag_;
    const int slots = std::max(knob_pipe_slots_, 2 * lag + 1);
    // Rounds of at least `min_chunk` bytes (each CTA then moves >= ~100 KB between fences),
    // about `rounds` of them so the software pipeline has something to overlap.
    // Two rounds up to 64 MiB, four above (measured on 2 and 8 x B200: fewer, larger rounds win
    // until the pipeline's fill and drain dominate).
    const unsigned long long rounds = static_cast<unsigned long long>(
        std::max<long>(1, knob_pipe_rounds_ > 0 ? knob_pipe_rounds_ : (bytes <= (64u << 20) ? 2 : 4)));
    const unsigned long long min_chunk = static_cast<unsigned long long>(knob_pipe_min_chunk_);
    auto pick_chunk_for = [&](unsigned long long part, unsigned long long cap) {
        unsigned long long want = RoundUp((part + rounds - 1) / rounds, q);
        want = std::max<unsigned long long>(want, RoundUp(min_chunk, q));
        return std::max<unsigned long long>(q, std::min<unsigned long long>(want, RoundDown(cap, q)));
    };
    auto pick_chunk = [&](unsigned long long cap) { return pick_chunk_for(bytes, cap); };
    int ctas = c.ctas;
    dc_.kernel_serial = ++kernel_serial_;
    if (c.algo == Algo::kHybrid) {
        // The switch's reduction rate, not NVLink, bounds NVLS; the two-shot part uses the link
        // bandwidth NVLS leaves idle. Split by BCCL_HYBRID_NVLS_PERMILLE (bytes through NVLS).
        const unsigned long long nb = RoundDown(static_cast<unsigned long long>(bytes * knob_hybrid_frac_), q);
        if (nb > 0 && nb < bytes && ctas >= 2 && nvls_.mc != nullptr && nranks_ > 1) {
            int nv_ctas = knob_hybrid_ctas_ > 0 ? static_cast<int>(knob_hybrid_ctas_)
                                                : static_cast<int>(ctas * knob_hybrid_frac_ + 0.5);
            nv_ctas = std::max(1, std::min(ctas - 1, nv_ctas));
            const unsigned long long nslot = RoundDown(nvls_.bytes / slots, 256);
            const unsigned long long tslot =
                RoundDown(data_bytes_ / 2 / (static_cast<unsigned long long>(slots) * 2ull * nranks_), 256);
            e = LaunchAllReduceHybrid(dc_, t.send_buf, t.recv_buf, t.count, dt, op, t.scale, nb,
                                      pick_chunk_for(nb, nslot), nslot, nv_ctas,
                                      pick_chunk_for(bytes - nb, tslot * nranks_), tslot, ctas - nv_ctas, slots,
                                      stream, lag);
            last_algo_ = "hybrid";
            if (e != cudaSuccess) {
                LOG_ERROR("rank %d: hybrid launch failed: %s", rank_, cudaGetErrorString(e));
                return false;
            }
            launches_++;
            return true;
        }
    }
    if (c.algo == Algo::kRing) {
        // Messages of up to 128 KiB, small enough that every SM gets a channel.
        const unsigned long long per = (bytes + static_cast<unsigned long long>(nranks_) * num_sms_ - 1) /
                                       (static_cast<unsigned long long>(nranks_) * num_sms_);
        // Every CTA's two inbox slots must fit the second half of the data region.
        const unsigned long long fit = RoundDown(data_bytes_ / 2 / (2ull * static_cast<unsigned long long>(std::max(1, ctas))), 256);
        const unsigned long long block = std::max<unsigned long long>(
            256, std::min<unsigned long long>(fit, std::min<unsigned long long>(128u << 10, std::max<unsigned long long>(256, RoundUp(per, 256)))));
        e = LaunchRingAllReduce(dc_, t.send_buf, t.recv_buf, t.count, dt, op, t.scale, block, ctas, stream);
        last_algo_ = "ring";
    } else if (c.algo == Algo::kNvls || (c.algo == Algo::kHybrid && nvls_.mc != nullptr)) {
        const unsigned long long slot = RoundDown(nvls_.bytes / slots, 256);
        const unsigned long long chunk = pick_chunk(slot);
        if (t.func == CollFunc::AllReduce) {
            e = LaunchAllReducePipe(dc_, kPipeNvls, t.send_buf, t.recv_buf, t.count, dt, op, t.scale, chunk, slot, slots,
                                    ctas, stream, lag);
        } else if (t.func == CollFunc::AllGather || t.func == CollFunc::ReduceScatter) {
            // A slot holds one chunk of every rank's block.
            const unsigned long long cap = RoundDown(slot / static_cast<unsigned long long>(nranks_), 16);
            unsigned long long want = RoundUp((bytes + rounds - 1) / rounds, 16);
            want = std::max<unsigned long long>(want, RoundUp(min_chunk / static_cast<unsigned long long>(nranks_), 16));
            const unsigned long long pc = std::max<unsigned long long>(16, std::min<unsigned long long>(want, cap));
            e = LaunchNvls(dc_, static_cast<int>(t.func), t.send_buf, t.recv_buf, t.count, dt, op, t.root, t.scale,
                           pc, slot, slots, ctas, stream);
        } else {
            e = LaunchNvls(dc_, static_cast<int>(t.func), t.send_buf, t.recv_buf, t.count, dt, op, t.root, t.scale,
                           chunk, slot, slots, ctas, stream);
        }
        last_algo_ = "nvls";
    } else {
        // Two ranks: a one-shot push moves the same NVLink bytes as two-shot with one
        // reduction step per round instead of two; from 32 MiB the two-shot schedule measured
        // faster (its rounds move half as much per phase).
        int kind = (nranks_ == 2 && bytes < (32u << 20)) ? kPipeOneShot : kPipeTwoShot;
        const long forced_kind = knob_pipe_kind_;
        if (forced_kind == kPipeOneShot || forced_kind == kPipeTwoShot) kind = static_cast<int>(forced_kind);
        unsigned long long slot, chunk;
        if (kind == kPipeOneShot) {
            slot = RoundDown(data_bytes_ / 2 / (static_cast<unsigned long long>(slots) * nranks_), 256);
            chunk = pick_chunk(slot);
        } else {
            slot = RoundDown(data_bytes_ / 2 / (static_cast<unsigned long long>(slots) * 2ull * nranks_), 256);
            chunk = pick_chunk(slot * nranks_);
        }
        e = LaunchAllReducePipe(dc_, kind, t.send_buf, t.recv_buf, t.count, dt, op, t.scale, chunk, slot, slots, ctas,
                                stream, lag);
        last_algo_ = kind == kPipeOneShot ? "oneshot_pipe" : "twoshot";
    }
    if (e != cudaSuccess) {
        LOG_ERROR("rank %d: %s launch failed: %s", rank_, last_algo_, cudaGetErrorString(e));
        return false;
    }
    launches_++;
    return true;
}

bool DeviceEngine::EnsureP2pStream() {
    if (p2p_stream_ != nullptr) return true;
    CUDA_OK(cudaStreamCreateWithFlags(&p2p_stream_, cudaStreamNonBlocking), "cudaStreamCreate(p2p)");
    CUDA_OK(cudaEventCreateWithFlags(&p2p_fork_, cudaEventDisableTiming), "cudaEventCreate(p2p fork)");
    CUDA_OK(cudaEventCreateWithFlags(&p2p_join_, cudaEventDisableTiming), "cudaEventCreate(p2p join)");
    return true;
}

bool DeviceEngine::Execute(const std::vector<CollTask>& sorted, cudaStream_t stream) {
    if (!inited_) {
        LOG_ERROR("device engine not initialised");
        return false;
    }
    if (err_host_->code != kDevOk) return CheckDeviceError();
    std::vector<CollTask> p2p;
    bool has_coll = false;
    for (const CollTask& t : sorted) {
        if (IsP2p(t.func)) {
            if (t.count > 0) p2p.push_back(t);
        } else if (t.count > 0) {
            has_coll = true;
        }
    }
    // A group with both kinds: NCCL's Send/Recv go first, on the side stream forked here, and
    // the collectives use at most num_sms - kP2pReservedSms CTAs, so NCCL's kernels find SMs
    // while ours (whose CTAs wait on their peers' CTAs) are resident. The join follows below.
    const int sms_all = num_sms_;
    bool forked = false;
    if (!p2p.empty() && has_coll && !knob_p2p_native_ && p2p_.ready()) {
        if (!EnsureP2pStream()) return false;
        CUDA_OK(cudaEventRecord(p2p_fork_, stream), "cudaEventRecord(p2p fork)");
        CUDA_OK(cudaStreamWaitEvent(p2p_stream_, p2p_fork_, 0), "cudaStreamWaitEvent(p2p fork)");
        const bool p2p_ok = p2p_.Run(p2p, p2p_stream_);
        CUDA_OK(cudaEventRecord(p2p_join_, p2p_stream_), "cudaEventRecord(p2p join)");
        if (!p2p_ok) {
            // What was enqueued on the side stream still orders before the caller's later work.
            CUDA_OK(cudaStreamWaitEvent(stream, p2p_join_, 0), "cudaStreamWaitEvent(p2p join)");
            return false;
        }
        p2p.clear();
        forked = true;
        num_sms_ = std::max(16, sms_all - kP2pReservedSms);
    }
    const bool ok = ExecuteCollectives(sorted, stream) && (p2p.empty() || RunP2p(p2p, stream));
    num_sms_ = sms_all;
    if (forked) {
        // Joined even after a failure, so the caller's stream never outruns the side stream.
        CUDA_OK(cudaStreamWaitEvent(stream, p2p_join_, 0), "cudaStreamWaitEvent(p2p join)");
        if (ok && has_coll) last_algo_ = "mixed+nccl_p2p";
    }
    return ok;
}

bool DeviceEngine::RunP2p(const std::vector<CollTask>& p2p, cudaStream_t stream) {
    if (knob_p2p_native_) return RunNativeP2p(p2p, stream);
    if (!p2p_.Run(p2p, stream)) return false;
    last_algo_ = "nccl_p2p";
    return true;
}

bool DeviceEngine::ExecuteCollectives(const std::vector<CollTask>& sorted, cudaStream_t stream) {
    std::vector<WorkItem> batch;
    unsigned long long stream_bytes = 0;
    int ncoll = 0;
    for (const CollTask& t : sorted) ncoll += (!IsP2p(t.func) && t.count > 0) ? 1 : 0;
    for (const CollTask& t : sorted) {
        if (IsP2p(t.func)) continue;
        if (t.count == 0) continue;
        const size_t bytes = t.count * DataTypeSize(t.dtype);
        const bool nvls_ok = nvls_.mc != nullptr &&
                             (t.func == CollFunc::Broadcast || t.func == CollFunc::AllGather ||
                              NvlsSupports(static_cast<int>(t.dtype), static_cast<int>(t.op)));
        AlgoChoice c = planner_->ChooseAlgo(t.func, t.dtype, t.op, bytes, nranks_, nvls_ok, max_ctas_,
                                            t.algo != Algo::kAuto ? t.algo : forced_);
        // An ungrouped small AllReduce runs the low-latency kernel: no barrier, one NVLink trip
        // (what the push engine would pay a fenced flag barrier for).
        // AllGather / ReduceScatter too, up to knob_ll_block_max_ per rank block.
        const bool ll_func = t.func == CollFunc::AllReduce || t.func == CollFunc::AllGather ||
                             t.func == CollFunc::ReduceScatter;
        const size_t ll_max = t.func == CollFunc::AllReduce ? knob_ll_max_ : knob_ll_block_max_;
        // c.algo is kLL when the call, BCCL_ALGO or a tuning-file row asked for it.
        const bool want_ll = c.algo == Algo::kLL || (t.algo == Algo::kAuto && forced_ == Algo::kAuto &&
                                                       c.algo == Algo::kOneShot && bytes <= ll_max);
        const bool ll_ok = ll_func && nranks_ > 1 && ncoll == 1 && dc_.ll_off != 0 && bytes <= kLLMaxLines * 8;
        if (c.algo == Algo::kLL && !ll_ok) c.algo = Algo::kOneShot;  // grouped, one rank: the push engine
        if (ll_ok && want_ll) {
            if (!FlushBatch(&batch, &stream_bytes, stream)) return false;
            dc_.kernel_serial = ++kernel_serial_;
            cudaError_t e = LaunchCollectiveLL(dc_, static_cast<int>(t.func), t.send_buf, t.recv_buf, t.count,
                                               static_cast<int>(t.dtype), static_cast<int>(t.op), t.scale, stream);
            if (e != cudaSuccess) {
                LOG_ERROR("rank %d: low-latency launch failed: %s", rank_, cudaGetErrorString(e));
                return false;
            }
            launches_++;
            last_algo_ = "ll";
            continue;
        }
        // Inside a group, a collective of up to kGroupPushMaxBytes per rank joins the batched push
        // launch even where the planner would give it a launch of its own: the launch and its
        // barriers cost more than the push moves extra at that size, and the group stays one
        // kernel (the reference's dynamic executor keeps a batch on its channels for the same reason).
        if (ncoll > 1 && t.algo == Algo::kAuto && forced_ == Algo::kAuto && bytes <= kGroupPushMaxBytes) {
            c.algo = Algo::kOneShot;
        }
        const bool ring = c.algo == Algo::kRing && t.func == CollFunc::AllReduce && nranks_ > 1;
        if (ring) c.ctas = max_ctas_ > 0 ? std::min(num_sms_, max_ctas_) : num_sms_;
        // Symmetric (multicast-bound) user buffers: NVLS without staging. AllReduce when the
        // planner picks NVLS and both buffers are symmetric; AllGather when the output is,
        // ReduceScatter when the input is (any size: one pass, two barriers).
        char* send_mc = nullptr;
        char* recv_mc = nullptr;
        const size_t all_bytes = bytes * static_cast<size_t>(nranks_);
        bool zc = false;
        const void* zc_send = nullptr;
        void* zc_recv = nullptr;
        // Zero-copy kernels move 16-byte vectors: sizes and addresses must be 16-byte aligned
        // (otherwise the staged kernels below run).
        const bool aligned16 = (bytes % 16) == 0 && ((reinterpret_cast<uintptr_t>(t.send_buf) |
                                                      reinterpret_cast<uintptr_t>(t.recv_buf)) & 15) == 0;
        if (nranks_ > 1 && aligned16 && nvls_.mc != nullptr && knob_zero_copy_) {
            if (t.func == CollFunc::AllReduce && c.algo == Algo::kNvls && UserMulticast(t.send_buf, bytes, &send_mc) &&
                UserMulticast(t.recv_buf, bytes, &recv_mc)) {
                zc = true;
                zc_send = send_mc;
                zc_recv = recv_mc;
            } else if (t.func == CollFunc::AllGather && UserMulticast(t.recv_buf, all_bytes, &recv_mc)) {
                zc = true;
                zc_send = t.send_buf;
                zc_recv = recv_mc;
            } else if (t.func == CollFunc::ReduceScatter && NvlsSupports(static_cast<int>(t.dtype), static_cast<int>(t.op)) &&
                       UserMulticast(t.send_buf, all_bytes, &send_mc)) {
                zc = true;
                zc_send = send_mc;
                zc_recv = t.recv_buf;
            }
        }
        // Registered or symmetric buffers at the same place on every rank: AllReduce /
        // AllGather / ReduceScatter over peer memory without staging, for payloads of at least
        // BCCL_P2P_ZC_MIN_BYTES (the batched push kernel stays better for small ones).
        char* in_peers[kMaxRanks] = {};
        char* out_peers[kMaxRanks] = {};
        bool p2p_zc = false;
        if (!zc && nranks_ > 1 && aligned16 && knob_zero_copy_ && (!reg_bufs_.empty() || !user_bufs_.empty()) &&
            (t.func == CollFunc::AllReduce ? bytes : all_bytes) >= knob_p2p_zc_min_) {
            if (t.func == CollFunc::AllReduce) {
                p2p_zc = PeerPointers(t.send_buf, bytes, in_peers) && PeerPointers(t.recv_buf, bytes, out_peers);
            } else if (t.func == CollFunc::AllGather) {
                p2p_zc = PeerPointers(t.recv_buf, all_bytes, out_peers);
                for (int q = 0; q < nranks_; ++q) in_peers[q] = const_cast<char*>(static_cast<const char*>(t.send_buf));
            } else if (t.func == CollFunc::ReduceScatter) {
                p2p_zc = PeerPointers(t.send_buf, all_bytes, in_peers);
                for (int q = 0; q < nranks_; ++q) out_peers[q] = static_cast<char*>(t.recv_buf);
            }
        }
        if (p2p_zc) {
            if (!FlushBatch(&batch, &stream_bytes, stream)) return false;
            const size_t moved = t.func == CollFunc::AllReduce ? bytes : all_bytes;
            int ctas = static_cast<int>(std::min<size_t>(std::max<size_t>(moved / (32u << 10), 8),
                                                         static_cast<size_t>(num_sms_)));
            if (max_ctas_ > 0) ctas = std::min(ctas, max_ctas_);
            const long env_max = knob_max_ctas_;
            if (env_max > 0) ctas = std::min<int>(ctas, static_cast<int>(env_max));
            dc_.kernel_serial = ++kernel_serial_;
            cudaError_t e = LaunchP2pZeroCopy(dc_, static_cast<int>(t.func), in_peers, out_peers, t.count,
                                              static_cast<int>(t.dtype), static_cast<int>(t.op), t.scale, ctas, stream);
            if (e != cudaSuccess) {
                LOG_ERROR("rank %d: zero-copy peer launch failed: %s", rank_, cudaGetErrorString(e));
                return false;
            }
            launches_++;
            last_algo_ = "p2p_zero_copy";
            continue;
        }
        if (zc) {
            if (!FlushBatch(&batch, &stream_bytes, stream)) return false;
            const size_t moved = t.func == CollFunc::AllReduce ? bytes : all_bytes;
            int zc_ctas = static_cast<int>(std::min<size_t>(std::max<size_t>(moved / (64u << 10), 8),
                                                            static_cast<size_t>(num_sms_)));
            if (max_ctas_ > 0) zc_ctas = std::min(zc_ctas, max_ctas_);
            dc_.kernel_serial = ++kernel_serial_;
            cudaError_t e = LaunchNvlsZeroCopy(dc_, static_cast<int>(t.func), zc_send, zc_recv, t.count,
                                               static_cast<int>(t.dtype), static_cast<int>(t.op), t.scale, zc_ctas,
                                               stream);
            if (e != cudaSuccess) {
                LOG_ERROR("rank %d: zero-copy NVLS launch failed: %s", rank_, cudaGetErrorString(e));
                return false;
            }
            launches_++;
            last_algo_ = "nvls_zero_copy";
            continue;
        }
        if (c.algo == Algo::kTwoShot || c.algo == Algo::kNvls || c.algo == Algo::kHybrid) {
            // Large-payload kernels: per-CTA barriers with the same CTA index on every rank, so
            // every CTA must be resident: at most one per SM.
            const size_t moved = (t.func == CollFunc::AllGather || t.func == CollFunc::ReduceScatter) ? all_bytes : bytes;
            int want = static_cast<int>(std::min<size_t>(std::max<size_t>(moved / (32u << 10), 8),
                                                         static_cast<size_t>(num_sms_)));
            c.ctas = std::min(want, kMaxCtas);
            if (max_ctas_ > 0) c.ctas = std::min(c.ctas, max_ctas_);
            const long env_max = knob_max_ctas_;
            if (env_max > 0) c.ctas = std::min<int>(c.ctas, static_cast<int>(env_max));
        }
        // One rank, 1 MiB or more: every collective is a copy (times the AllReduce scale); a
        // streaming copy kernel instead of the N-source push kernel.
        if (nranks_ == 1 && knob_local_copy_ && bytes >= (1u << 20) && aligned16) {
            if (!FlushBatch(&batch, &stream_bytes, stream)) return false;
            const void* src = t.send_buf != nullptr ? t.send_buf : t.recv_buf;
            const bool reducing = t.func == CollFunc::AllReduce || t.func == CollFunc::Reduce ||
                                  t.func == CollFunc::ReduceScatter;
            const float scale = reducing ? t.scale : 1.0f;
            last_algo_ = "local_copy";
            if (src == t.recv_buf && scale == 1.0f) continue;  // in place: nothing moves
            cudaError_t e = LaunchLocalCopy(src, t.recv_buf, bytes, static_cast<int>(t.dtype), scale, num_sms_, stream);
            if (e != cudaSuccess) {
                LOG_ERROR("rank %d: local copy launch failed: %s", rank_, cudaGetErrorString(e));
                return false;
            }
            launches_++;
            continue;
        }
        if (nranks_ == 1 || c.algo == Algo::kOneShot || (c.algo == Algo::kRing && !ring)) {
            WorkItem w;
            w.src = t.send_buf;
            w.dst = t.recv_buf;
            w.count = t.count;
            w.stream_off = stream_bytes;
            w.func = static_cast<unsigned char>(t.func);
            w.dtype = static_cast<unsigned char>(t.dtype);
            w.op = static_cast<unsigned char>(t.op);
            w.root = static_cast<unsigned char>(t.root);
            w.scale = t.scale;
            if (t.func == CollFunc::Broadcast && w.src == nullptr) w.src = w.dst;
            batch.push_back(w);
            stream_bytes += RoundUp(PeerPayload(t), 16);
            continue;
        }
        if (!FlushBatch(&batch, &stream_bytes, stream)) return false;
        if (!LaunchLarge(t, c, stream)) return false;
    }
    return FlushBatch(&batch, &stream_bytes, stream);
}

bool DeviceEngine::RunNativeP2p(const std::vector<CollTask>& tasks, cudaStream_t stream) {
    // Operations grouped by (direction, peer), each pair's in the order the group issued them.
    std::vector<P2pNativeOp> ops;
    std::vector<P2pNativeRole> roles;
    for (int dir = 0; dir < 2; ++dir) {
        for (int q = 0; q < nranks_; ++q) {
            if (q == rank_) continue;
            const int begin = static_cast<int>(ops.size());
            unsigned long long total = 0;
            for (const CollTask& t : tasks) {
                if (t.peer != q || t.count == 0 || (t.func == CollFunc::Send) != (dir == 0)) continue;
                const unsigned long long b = static_cast<unsigned long long>(t.count) * DataTypeSize(t.dtype);
                P2pNativeOp op;
                op.buf = dir == 0 ? const_cast<char*>(static_cast<const char*>(t.send_buf)) : static_cast<char*>(t.recv_buf);
                op.bytes = b;
                ops.push_back(op);
                total += b;
            }
            if (total == 0) continue;
            const int nch = P2pChannels(total);
            for (int ch = 0; ch < nch; ++ch) {
                P2pNativeRole r;
                r.peer = static_cast<short>(q);
                r.dir = static_cast<short>(dir);
                r.channel = static_cast<short>(ch);
                r.nch = static_cast<short>(nch);
                r.op_begin = begin;
                r.op_end = static_cast<int>(ops.size());
                roles.push_back(r);
            }
        }
    }
    if (roles.empty()) return true;
    if (static_cast<int>(ops.size()) > kP2pMaxOps) {
        LOG_ERROR("rank %d: native Send/Recv takes at most %d operations per group (got %zu)", rank_, kP2pMaxOps,
                  ops.size());
        return false;
    }
    dc_.kernel_serial = ++kernel_serial_;
    cudaError_t e = LaunchP2pNative(dc_, ops.data(), static_cast<int>(ops.size()), roles.data(),
                                    static_cast<int>(roles.size()), stream);
    if (e != cudaSuccess) {
        LOG_ERROR("rank %d: native Send/Recv launch failed: %s", rank_, cudaGetErrorString(e));
        return false;
    }
    launches_++;
    last_algo_ = "native_p2p";
    return true;
}

}  // namespace bccl
