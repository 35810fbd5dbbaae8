#include "host/host_engine.h"

#include <poll.h>
#include <sched.h>
#include <sys/epoll.h>
#include <sys/mman.h>
#include <sys/uio.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <chrono>
#include <cstring>
#include <map>

#include "core/bootstrap.h"
#include "core/env.h"
#include "core/fdpass.h"
#include "core/logger.h"
#include "core/net.h"
#include "host/host_reduce.h"

namespace bccl {
namespace {

constexpr uint64_t kSegMagic = 0xBCC15E6D00000001ull;
constexpr uint32_t kSegFdTag = 0x5E600000u;
constexpr uint32_t kLinkMagic = 0xBCC1714Bu;

struct SegHeader {
    uint64_t magic;
    uint32_t local_size;
    uint32_t n_channels;
    uint64_t slot_bytes;
    uint64_t ring_bytes;
    uint64_t world;
};

// Single-copy Send/Recv within a machine (cross-memory attach): each local rank publishes its pid
// and the address of a probe word here; acks[i][j] counts the zero-copy messages rank j (local
// index) has finished reading from rank i.
struct CmaInfo {
    int32_t pid;
    int32_t pad;
    uint64_t probe_addr;
    uint64_t pad2[2];
};
constexpr uint64_t kCmaMagic = 0xBCC1C0DE5E4D0001ull;
// What the sender puts in the ring instead of the payload: where the receiver reads it.
struct CmaDesc {
    uint64_t magic;
    int64_t pid;
    uint64_t addr;
    uint64_t bytes;
};
size_t CmaInfoOff() { return 64; }
size_t CmaAcksOff(int L) { return (CmaInfoOff() + sizeof(CmaInfo) * static_cast<size_t>(L) + 63) / 64 * 64; }

struct LinkHello {
    uint32_t magic;
    int32_t rank;
    int32_t channel;  // -1 for the P2P link
};

size_t AlignUp(size_t x, size_t a) { return (x + a - 1) / a * a; }

using Clock = std::chrono::steady_clock;

inline void CpuRelax() {
#if defined(__x86_64__) || defined(__i386__)
    __builtin_ia32_pause();
#elif defined(__aarch64__)
    asm volatile("yield");
#endif
}

// Chunks from this size on go around the leaders' ring instead of the one-step exchange.
constexpr size_t kLeaderRingBytes = 128u << 10;

// How long an idle channel thread (and a caller waiting for the channels) spins before
// blocking, when spinning is on: about the gap between back-to-back collectives.
constexpr int kSpinUs = 200;

// Elements [e0, e1) of channel ch when `count` elements are cut into n contiguous slices.
void ChannelSlice(size_t count, int n, int ch, size_t* e0, size_t* e1) {
    size_t per = (count + static_cast<size_t>(n) - 1) / static_cast<size_t>(n);
    *e0 = std::min(count, per * static_cast<size_t>(ch));
    *e1 = std::min(count, *e0 + per);
}

}  // namespace

// Every rank as its own machine: all exchanges then go over TCP (BCCL_DISABLE_SHM).
static MachineView SplitView(int rank, int world) {
    MachineView v;
    v.local_rank = 0;
    v.local_size = 1;
    v.local_ranks = {rank};
    v.machine_index = rank;
    v.machine_count = world;
    for (int p = 0; p < world; ++p) {
        v.machine_leaders.push_back(p);
        v.machine_of.push_back(p);
        v.local_index_of.push_back(0);
        v.machine_ranks.push_back({p});
    }
    return v;
}

bool HostEngine::Init(const CommConfig& cfg, Bootstrap* bs, FdPasser* fp, const std::vector<NodeInfo>& nodes,
                      const MachineView& view, int data_listen_fd) {
    rank_ = cfg.rank;
    listen_fd_ = data_listen_fd;
    world_ = cfg.world_size;
    // BCCL_DISABLE_SHM=1 (the reference's OCCL_DISABLE_SHM, src/communicator.cpp:47-60): ranks on
    // one host talk over TCP as if each were a machine of its own. Only the engine's routing
    // changes; the communicator's machine view stays the host's.
    view_ = EnvFlag("BCCL_DISABLE_SHM") ? SplitView(cfg.rank, cfg.world_size) : view;
    timeout_ms_ = cfg.timeout_ms > 0 ? cfg.timeout_ms : static_cast<int>(EnvInt("BCCL_TIMEOUT_MS", 30000));
    const long ncores = sysconf(_SC_NPROCESSORS_ONLN);
    n_channels_ = cfg.n_channels > 0 ? cfg.n_channels : 4;
    n_channels_ = std::max(1, std::min(n_channels_, 16));
    // Collectives of at least split_bytes_ are cut into one slice per channel. With four channels
    // (four or more cores per local rank; the channel count is agreed over all ranks, so this
    // default agrees too) the cut starts at 256 KiB: on a 16-core host with 4 ranks, a 512 KiB
    // int32 AllReduce took 100-103 us cut and 132-161 us whole, while 128 KiB ran in 32 us whole
    // and 58 us cut. With fewer channels a cut below 1 MiB costs more than it saves (2 channels on
    // 8 cores: 512 KiB 1.5x slower cut).
    const long split_default = n_channels_ >= 4 ? (256L << 10) : (1L << 20);
    split_bytes_ = static_cast<size_t>(std::max<long>(0, EnvInt("BCCL_HOST_SPLIT_BYTES", split_default)));
    {
        const long cores = sysconf(_SC_NPROCESSORS_ONLN);
        const long want = static_cast<long>(view.local_size) * (n_channels_ + 1);
        spin_ = EnvInt("BCCL_HOST_SPIN", cores >= want ? 1 : 0) != 0;
    }
    // The reference switches to its epoll executor when ranks outnumber cores
    // (src/communicator.cpp:37-45); here that choice drives how Send/Recv wait.
    std::string ex = EnvStr("BCCL_HOST_EXECUTOR", "");
    epoll_ = ex == "epoll" || (ex.empty() && ncores > 0 && view_.local_size > ncores);
    slot_bytes_ = static_cast<size_t>(EnvInt("BCCL_HOST_SLOT_BYTES", 0));
    if (slot_bytes_ == 0) slot_bytes_ = std::max<size_t>(64u << 10, (8u << 20) / static_cast<size_t>(std::max(world_, 1)));
    slot_bytes_ = AlignUp(slot_bytes_, 256);
    ring_bytes_ = static_cast<size_t>(EnvInt("BCCL_HOST_RING_BYTES", 1 << 20));
    trace_cap_ = static_cast<size_t>(std::max<long>(0, EnvInt("BCCL_TRACE", 0)));

    // ---- shared segment of this machine
    const int L = view_.local_size;
    // Header page(s): SegHeader, the ranks' CmaInfo, the zero-copy acks[L][L].
    const size_t hdr = AlignUp(CmaAcksOff(L) + sizeof(uint64_t) * static_cast<size_t>(L) * static_cast<size_t>(L), 4096);
    cma_bytes_ = static_cast<size_t>(std::max<long>(1, EnvInt("BCCL_HOST_ZC_BYTES", 256 << 10)));
    const size_t bar_bytes = AlignUp(sizeof(ShmBarrier) * static_cast<size_t>(n_channels_), 4096);
    // Two buffer sets per channel (slots of every rank + a result area), used by alternate chunks.
    const size_t set_bytes = static_cast<size_t>(world_ + 1) * slot_bytes_;
    const size_t chan_bytes = 2 * set_bytes;
    const size_t ring_stride = sizeof(ShmRingCtrl) + AlignUp(ring_bytes_, 64);
    seg_bytes_ = hdr + bar_bytes + chan_bytes * static_cast<size_t>(n_channels_) +
                 ring_stride * static_cast<size_t>(L) * static_cast<size_t>(L);
    int seg_fd = -1;
    bool ok = true;
    if (view_.local_rank == 0) {
        seg_fd = static_cast<int>(memfd_create("bccl-host", MFD_CLOEXEC));
        ok = seg_fd >= 0 && ftruncate(seg_fd, static_cast<off_t>(seg_bytes_)) == 0;
        if (ok && !FaultActive("segment_drop", rank_)) {
            for (int i = 1; ok && i < L; ++i) ok = fp->SendFd(view_.local_ranks[i], kSegFdTag, seg_fd, timeout_ms_);
        }
        if (!ok) LOG_ERROR("rank %d: creating the shared segment failed", rank_);
    } else {
        ok = fp->RecvFd(view_.local_ranks[0], kSegFdTag, &seg_fd, timeout_ms_);
    }
    if (ok) {
        seg_ = mmap(nullptr, seg_bytes_, PROT_READ | PROT_WRITE, MAP_SHARED, seg_fd, 0);
        if (seg_ == MAP_FAILED) {
            seg_ = nullptr;
            ok = false;
            LOG_ERROR("rank %d: mmap of the shared segment failed", rank_);
        }
    }
    if (seg_fd >= 0) close(seg_fd);
    if (ok && view_.local_rank == 0) {
        auto* h = static_cast<SegHeader*>(seg_);
        h->local_size = static_cast<uint32_t>(L);
        h->n_channels = static_cast<uint32_t>(n_channels_);
        h->slot_bytes = slot_bytes_;
        h->ring_bytes = ring_bytes_;
        h->world = static_cast<uint64_t>(world_);
        // memfd pages start zeroed: barriers and ring cursors are already 0.
        std::atomic_thread_fence(std::memory_order_release);
        h->magic = kSegMagic;
    }
    if (!bs->Barrier() || !ok) return false;
    auto* h = static_cast<SegHeader*>(seg_);
    if (h->magic != kSegMagic || h->slot_bytes != slot_bytes_ || h->n_channels != static_cast<uint32_t>(n_channels_)) {
        LOG_ERROR("rank %d: shared segment header mismatch (n_channels and slot sizes must match on all ranks)", rank_);
        return false;
    }
    char* base = static_cast<char*>(seg_);
    if (!SetupCma(bs)) return false;
    chans_.resize(n_channels_);
    for (int c = 0; c < n_channels_; ++c) {
        chans_[c].barrier = reinterpret_cast<ShmBarrier*>(base + hdr) + c;
        for (int k = 0; k < 2; ++k) {
            chans_[c].set_slots[k] = base + hdr + bar_bytes + chan_bytes * static_cast<size_t>(c) + set_bytes * k;
            chans_[c].set_result[k] = chans_[c].set_slots[k] + static_cast<size_t>(world_) * slot_bytes_;
        }
        chans_[c].slots = chans_[c].set_slots[0];
        chans_[c].result = chans_[c].set_result[0];
    }
    char* rings = base + hdr + bar_bytes + chan_bytes * static_cast<size_t>(n_channels_);
    p2p_send_.resize(world_);
    p2p_recv_.resize(world_);
    p2p_tcp_.resize(world_);
    for (int i = 0; i < L; ++i) {
        for (int j = 0; j < L; ++j) {
            if (i == j) continue;
            char* r = rings + ring_stride * (static_cast<size_t>(i) * L + static_cast<size_t>(j));
            auto* ctrl = reinterpret_cast<ShmRingCtrl*>(r);
            char* data = r + sizeof(ShmRingCtrl);
            int gi = view_.local_ranks[i], gj = view_.local_ranks[j];
            if (gi == rank_) p2p_send_[gj].reset(new ShmRingTransport(ctrl, data, ring_bytes_, true));
            if (gj == rank_) p2p_recv_[gi].reset(new ShmRingTransport(ctrl, data, ring_bytes_, false));
        }
    }

    // ---- TCP links: leader mesh per channel, and P2P links between ranks on different machines.
    const bool leader = view_.local_rank == 0;
    const int M = view_.machine_count;
    struct Want {
        int peer;
        int channel;
    };
    std::vector<Want> outgoing;
    int incoming = 0;
    if (leader && M > 1) {
        for (int c = 0; c < n_channels_; ++c) chans_[c].leader_links.resize(M);
        for (int m = 0; m < M; ++m) {
            if (m == view_.machine_index) continue;
            for (int c = 0; c < n_channels_; ++c) {
                if (view_.machine_index < m) outgoing.push_back({view_.machine_leaders[m], c});
                else ++incoming;
            }
        }
    }
    for (int p = 0; p < world_; ++p) {
        if (p == rank_ || view_.machine_of[p] == view_.machine_index) continue;
        if (rank_ < p) outgoing.push_back({p, -1});
        else ++incoming;
    }
    auto bind_link = [&](int peer, int channel, int fd) {
        if (channel < 0) {
            std::shared_ptr<TcpTransport> t(new TcpTransport(fd));
            p2p_tcp_[peer] = t;
        } else {
            chans_[channel].leader_links[view_.machine_of[peer]].reset(new TcpTransport(fd));
        }
    };
    for (const Want& w : outgoing) {
        int fd = net::Connect(nodes[w.peer].ip_addr, nodes[w.peer].data_port, timeout_ms_);
        if (fd < 0) return false;
        LinkHello hello{kLinkMagic, rank_, w.channel};
        if (!net::SendAll(fd, &hello, sizeof(hello), timeout_ms_)) {
            close(fd);
            return false;
        }
        bind_link(w.peer, w.channel, fd);
    }
    for (int i = 0; i < incoming; ++i) {
        int fd = net::Accept(listen_fd_, timeout_ms_);
        LinkHello hello{};
        if (fd < 0 || !net::RecvAll(fd, &hello, sizeof(hello), timeout_ms_) || hello.magic != kLinkMagic ||
            hello.rank < 0 || hello.rank >= world_ || hello.channel >= n_channels_) {
            LOG_ERROR("rank %d: bad or missing link handshake", rank_);
            if (fd >= 0) close(fd);
            return false;
        }
        bind_link(hello.rank, hello.channel, fd);
    }
    for (int p = 0; p < world_; ++p) {
        if (p2p_tcp_[p]) {
            // TCP is full duplex: one socket serves both directions of the pair.
            struct Shared : Transport {
                std::shared_ptr<TcpTransport> t;
                explicit Shared(std::shared_ptr<TcpTransport> x) : t(std::move(x)) {}
                bool TrySend(const void* d, size_t s, size_t* p, bool* done) override { return t->TrySend(d, s, p, done); }
                bool TryRecv(void* d, size_t s, size_t* p, bool* done) override { return t->TryRecv(d, s, p, done); }
                int GetFd() const override { return t->GetFd(); }
                const char* Name() const override { return "tcp"; }
            };
            p2p_send_[p].reset(new Shared(p2p_tcp_[p]));
            p2p_recv_[p].reset(new Shared(p2p_tcp_[p]));
        }
    }
    chan_seq_.reset(new std::atomic<uint64_t>[n_channels_]());
    cv_chan_.reset(new std::condition_variable[n_channels_]);
    for (int c = 0; c < n_channels_; ++c) workers_.emplace_back(&HostEngine::WorkerLoop, this, c);
    if (!bs->Barrier()) return false;
    inited_ = true;
    return true;
}

// Zero-copy Send/Recv between ranks of this machine: enabled when every local rank can read
// every other's memory with process_vm_readv (same user, no ptrace restriction), checked by
// reading each peer's published probe word; the decision is agreed over all ranks.
bool HostEngine::SetupCma(Bootstrap* bs) {
    const int L = view_.local_size;
    char* base = static_cast<char*>(seg_);
    auto* info = reinterpret_cast<CmaInfo*>(base + CmaInfoOff());
    cma_acks_ = reinterpret_cast<std::atomic<uint64_t>*>(base + CmaAcksOff(L));
    cma_probe_ = kCmaMagic ^ static_cast<uint64_t>(rank_);
    info[view_.local_rank].pid = static_cast<int32_t>(getpid());
    info[view_.local_rank].probe_addr = reinterpret_cast<uint64_t>(&cma_probe_);
    cma_sent_.assign(static_cast<size_t>(world_), 0);
    const bool enabled = EnvInt("BCCL_HOST_CMA", 1) != 0;
    if (!bs->Barrier()) return false;  // every rank's info is published
    bool ok = enabled;
    for (int i = 0; ok && i < L; ++i) {
        if (i == view_.local_rank) continue;
        uint64_t v = 0;
        struct iovec mine = {&v, sizeof(v)};
        struct iovec theirs = {reinterpret_cast<void*>(info[i].probe_addr), sizeof(v)};
        ok = process_vm_readv(info[i].pid, &mine, 1, &theirs, 1, 0) == static_cast<ssize_t>(sizeof(v)) &&
             v == (kCmaMagic ^ static_cast<uint64_t>(view_.local_ranks[i]));
    }
    // Every rank reports whether it can read all of its local peers (trivially when it has none).
    std::vector<uint8_t> flag(1, ok ? 1 : 0);
    std::vector<std::vector<uint8_t>> all;
    if (!bs->AllGather(flag, &all)) return false;
    cma_ = enabled && L > 1;
    for (const auto& a : all) cma_ = cma_ && !a.empty() && a[0] == 1;
    if (enabled && L > 1 && !cma_) {
        LOG_INFO("rank %d: single-copy Send/Recv unavailable (process_vm_readv refused)", rank_);
    }
    return true;
}

void HostEngine::Finalize() {
    {
        std::lock_guard<std::mutex> lk(mu_);
        stop_.store(true);
    }
    for (int c = 0; c < static_cast<int>(workers_.size()); ++c) cv_chan_[c].notify_all();
    for (auto& t : workers_)
        if (t.joinable()) t.join();
    workers_.clear();
    stop_.store(false);
    chans_.clear();
    p2p_send_.clear();
    p2p_recv_.clear();
    p2p_tcp_.clear();
    if (seg_) munmap(seg_, seg_bytes_);
    seg_ = nullptr;
    inited_ = false;
}

const char* HostEngine::p2p_transport_name(int peer) const {
    if (peer < 0 || peer >= static_cast<int>(p2p_send_.size()) || !p2p_send_[peer]) return "none";
    return p2p_send_[peer]->Name();
}

void HostEngine::WorkerLoop(int ch) {
    if (EnvFlag("BCCL_HOST_PIN")) {
        const long ncores = sysconf(_SC_NPROCESSORS_ONLN);
        cpu_set_t set;
        CPU_ZERO(&set);
        CPU_SET(static_cast<int>((view_.local_rank * n_channels_ + ch) % std::max<long>(ncores, 1)), &set);
        if (sched_setaffinity(0, sizeof(set), &set) != 0) LOG_WARN("rank %d: pinning channel %d failed", rank_, ch);
    }
    std::atomic<uint64_t>& my_seq = chan_seq_[ch];
    uint64_t seen = 0;
    for (;;) {
        if (my_seq.load(std::memory_order_acquire) == seen && !stop_.load(std::memory_order_acquire)) {
            if (spin_) {
                const auto until = Clock::now() + std::chrono::microseconds(kSpinUs);
                for (uint32_t i = 0; my_seq.load(std::memory_order_acquire) == seen && !stop_.load(); ++i) {
                    CpuRelax();
                    if ((i & 255u) == 255u && Clock::now() > until) break;
                }
            }
            std::unique_lock<std::mutex> lk(mu_);
            cv_chan_[ch].wait(lk, [&] { return stop_.load() || my_seq.load() != seen; });
        }
        if (stop_.load()) return;
        seen = my_seq.load(std::memory_order_acquire);
        // job_ was written before this channel's sequence number was bumped and is not rewritten
        // until every woken channel finished this job, so reading it here needs no lock.
        const std::function<bool(int)> job = job_;
        if (!job(ch)) job_ok_.store(false);
        if (job_pending_.fetch_sub(1, std::memory_order_acq_rel) == 1) {
            std::lock_guard<std::mutex> lk(mu_);
            cv_done_.notify_all();
        }
    }
}

bool HostEngine::RunOnChannels(const std::function<bool(int)>& fn, int inline_ch, const std::vector<int>& busy) {
    std::vector<int> woken;
    {
        std::lock_guard<std::mutex> lk(mu_);
        // Channel inline_ch runs on the calling thread; the workers of the other busy channels
        // run theirs; the remaining workers are not woken at all.
        job_ = fn;
        job_ok_.store(true);
        for (int ch : busy)
            if (ch != inline_ch) woken.push_back(ch);
        job_pending_.store(static_cast<int>(woken.size()));
        for (int ch : woken) chan_seq_[ch].fetch_add(1, std::memory_order_release);
    }
    for (int ch : woken) cv_chan_[ch].notify_one();
    if (inline_ch >= 0 && !fn(inline_ch)) job_ok_.store(false);
    if (spin_) {
        const auto until = Clock::now() + std::chrono::microseconds(kSpinUs);
        for (uint32_t i = 0; job_pending_.load(std::memory_order_acquire) != 0; ++i) {
            CpuRelax();
            if ((i & 255u) == 255u && Clock::now() > until) break;
        }
    }
    if (job_pending_.load(std::memory_order_acquire) != 0) {
        std::unique_lock<std::mutex> lk(mu_);
        cv_done_.wait(lk, [&] { return job_pending_.load() == 0; });
    }
    return job_ok_.load();
}

bool HostEngine::Barrier(int ch) {
    ShmBarrier* b = chans_[ch].barrier;
    const uint32_t n = static_cast<uint32_t>(view_.local_size);
    if (n == 1) return true;
    const uint32_t g = b->gen.load(std::memory_order_acquire);
    if (b->count.fetch_add(1, std::memory_order_acq_rel) == n - 1) {
        b->count.store(0, std::memory_order_relaxed);
        b->gen.store(g + 1, std::memory_order_release);
        Mark(ch, kTrBarrier);
        return true;
    }
    auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms_);
    uint32_t spins = 0;
    while (b->gen.load(std::memory_order_acquire) == g) {
        if (++spins < 2000) {
            CpuRelax();
            continue;
        }
        sched_yield();
        if ((spins & 1023) == 0 && aborted_.load(std::memory_order_relaxed)) {
            LOG_ERROR("rank %d: channel %d barrier aborted", rank_, ch);
            return false;
        }
        if ((spins & 1023) == 0 && Clock::now() > deadline) {
            LOG_ERROR("rank %d: channel %d barrier timed out after %d ms", rank_, ch, timeout_ms_);
            return false;
        }
    }
    Mark(ch, kTrBarrier);
    return true;
}

bool HostEngine::LeaderExchange(int ch, const std::vector<int>& peers, const std::vector<const void*>& send,
                                const std::vector<size_t>& send_bytes, const std::vector<void*>& recv,
                                const std::vector<size_t>& recv_bytes) {
    const size_t n = peers.size();
    std::vector<size_t> sp(n, 0), rp(n, 0);
    std::vector<char> sd(n, 0), rd(n, 0);
    for (size_t i = 0; i < n; ++i) {
        sd[i] = send[i] == nullptr || send_bytes[i] == 0;
        rd[i] = recv[i] == nullptr || recv_bytes[i] == 0;
    }
    auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms_);
    for (;;) {
        bool all = true, progress = false;
        for (size_t i = 0; i < n; ++i) {
            TcpTransport* t = chans_[ch].leader_links[peers[i]].get();
            if (!sd[i]) {
                size_t before = sp[i];
                bool done = false;
                if (!t->TrySend(send[i], send_bytes[i], &sp[i], &done)) return false;
                sd[i] = done;
                progress |= sp[i] != before;
            }
            if (!rd[i]) {
                size_t before = rp[i];
                bool done = false;
                if (!t->TryRecv(recv[i], recv_bytes[i], &rp[i], &done)) return false;
                rd[i] = done;
                progress |= rp[i] != before;
            }
            all &= sd[i] && rd[i];
        }
        if (all) return true;
        if (!progress) {
            std::vector<struct pollfd> pf;
            for (size_t i = 0; i < n; ++i) {
                short ev = static_cast<short>((sd[i] ? 0 : POLLOUT) | (rd[i] ? 0 : POLLIN));
                if (ev) pf.push_back({chans_[ch].leader_links[peers[i]]->GetFd(), ev, 0});
            }
            poll(pf.data(), pf.size(), 50);
            if (aborted_.load(std::memory_order_relaxed)) {
                LOG_ERROR("rank %d: leader exchange on channel %d aborted", rank_, ch);
                return false;
            }
            if (Clock::now() > deadline) {
                LOG_ERROR("rank %d: leader exchange on channel %d timed out", rank_, ch);
                return false;
            }
        }
    }
}

// Ring AllReduce among the machine leaders over their TCP links (the reference's ring,
// src/topology/topology_ring.cpp:255-290, between machines): `buf` holds this machine's partial
// of `count` elements, cut into M blocks. Reduce-scatter: in step s, send block (m - s) to the
// next leader and add block (m - s - 1) from the previous one; block (m + 1) is then complete
// here and gets the AVG / scale epilogue. All-gather: pass the complete blocks around.
bool HostEngine::LeaderRingAllReduce(int ch, char* buf, size_t count, DataType dt, ReduceOp op, float scale) {
    const int M = view_.machine_count, m = view_.machine_index;
    const int next = (m + 1) % M, prev = (m + M - 1) % M;
    const size_t es = DataTypeSize(dt);
    const size_t per = (count + static_cast<size_t>(M) - 1) / static_cast<size_t>(M);
    auto blk = [&](int k, size_t* off, size_t* len) {
        k = ((k % M) + M) % M;
        *off = std::min(count, per * static_cast<size_t>(k));
        *len = std::min(count, *off + per) - *off;
    };
    Channel& C = chans_[ch];
    C.scratch.resize(per * es);
    const ReduceOp partial = op == ReduceOp::AVG ? ReduceOp::SUM : op;
    for (int s = 0; s < M - 1; ++s) {
        size_t so, sl, ro, rl;
        blk(m - s, &so, &sl);
        blk(m - s - 1, &ro, &rl);
        if (!LeaderExchange(ch, {next, prev}, {buf + so * es, nullptr}, {sl * es, 0}, {nullptr, C.scratch.data()},
                            {0, rl * es})) {
            return false;
        }
        const void* srcs[2] = {buf + ro * es, C.scratch.data()};
        hostmath::Reduce(dt, partial, buf + ro * es, srcs, 2, rl, world_, 1.0f, false);
    }
    size_t fo, fl;
    blk(m + 1, &fo, &fl);
    hostmath::Finish(dt, op, buf + fo * es, buf + fo * es, fl, world_, scale);
    for (int s = 0; s < M - 1; ++s) {
        size_t so, sl, ro, rl;
        blk(m + 1 - s, &so, &sl);
        blk(m - s, &ro, &rl);
        if (!LeaderExchange(ch, {next, prev}, {buf + so * es, nullptr}, {sl * es, 0}, {nullptr, buf + ro * es},
                            {0, rl * es})) {
            return false;
        }
    }
    return true;
}

// Reduction family (AllReduce, and Reduce when reduce_only): intra-machine two-shot, then
// leaders across machines.
bool HostEngine::AllReduceSlice(int ch, const CollTask& t, size_t e0, size_t e1, bool reduce_only) {
    const size_t es = DataTypeSize(t.dtype);
    const size_t chunk = slot_bytes_ / es;
    const int L = view_.local_size, li = view_.local_rank, M = view_.machine_count;
    const bool leader = li == 0;
    const int root_machine = reduce_only ? view_.machine_of[t.root] : -1;
    Channel& C = chans_[ch];
    const char* src = static_cast<const char*>(t.send_buf);
    char* dst = static_cast<char*>(t.recv_buf);
    for (size_t off = e0; off < e1; off += chunk) {
        NextBuffers(ch);
        const size_t clen = std::min(chunk, e1 - off);
        const size_t share = (clen + L - 1) / L;
        const size_t s0 = std::min(clen, share * li), s1 = std::min(clen, s0 + share);
        // Every share but this rank's own goes to the slot; this rank reduces its own share
        // reading its input in place.
        char* mine = Slot(ch, rank_);
        if (s0 > 0) memcpy(mine, src + off * es, s0 * es);
        if (clen > s1) memcpy(mine + s1 * es, src + (off + s1) * es, (clen - s1) * es);
        Mark(ch, kTrCopyIn);
        if (!Barrier(ch)) return false;
        if (s1 > s0) {
            const void* srcs[64];
            for (int i = 0; i < L; ++i) {
                const int q = view_.local_ranks[i];
                srcs[i] = q == rank_ ? static_cast<const void*>(src + (off + s0) * es)
                                     : static_cast<const void*>(Slot(ch, q) + s0 * es);
            }
            hostmath::Reduce(t.dtype, t.op, C.result + s0 * es, srcs, L, s1 - s0, world_, t.scale, M == 1);
        }
        Mark(ch, kTrReduce);
        if (!Barrier(ch)) return false;
        if (M > 2 && leader && !reduce_only && clen * es >= kLeaderRingBytes) {
            // Three or more machines and a large chunk: ring among the leaders (each sends
            // 2(M-1)/M of the chunk). Smaller chunks take the one-step exchange below, the
            // latency-bound role the reference gives its tree below 128 KiB
            // (src/planner.cpp:260-262).
            if (!LeaderRingAllReduce(ch, C.result, clen, t.dtype, t.op, t.scale)) return false;
        } else if (M > 1 && leader) {
            // Every leader receives the other machines' partials (Reduce: only the root's
            // leader needs them) and reduces all machines in machine order.
            std::vector<int> peers;
            std::vector<const void*> sends;
            std::vector<size_t> sbytes, rbytes;
            std::vector<void*> recvs;
            C.scratch.resize(static_cast<size_t>(M) * clen * es);
            for (int m = 0; m < M; ++m) {
                if (m == view_.machine_index) continue;
                const bool i_recv = !reduce_only || view_.machine_index == root_machine;
                const bool i_send = !reduce_only || m == root_machine;
                if (!i_recv && !i_send) continue;
                peers.push_back(m);
                sends.push_back(i_send ? C.result : nullptr);
                sbytes.push_back(i_send ? clen * es : 0);
                recvs.push_back(i_recv ? C.scratch.data() + static_cast<size_t>(m) * clen * es : nullptr);
                rbytes.push_back(i_recv ? clen * es : 0);
            }
            if (!LeaderExchange(ch, peers, sends, sbytes, recvs, rbytes)) return false;
            if (!reduce_only || view_.machine_index == root_machine) {
                memcpy(C.scratch.data() + static_cast<size_t>(view_.machine_index) * clen * es, C.result, clen * es);
                std::vector<const void*> srcs(M);
                for (int m = 0; m < M; ++m) srcs[m] = C.scratch.data() + static_cast<size_t>(m) * clen * es;
                hostmath::Reduce(t.dtype, t.op, C.result, srcs.data(), M, clen, world_, t.scale, true);
            }
        }
        if (M > 1 && leader) Mark(ch, kTrExchange);
        if (M > 1 && !Barrier(ch)) return false;
        if (!reduce_only || rank_ == t.root) memcpy(dst + off * es, C.result, clen * es);
        Mark(ch, kTrCopyOut);
    }
    return true;
}

bool HostEngine::BroadcastSlice(int ch, const CollTask& t, size_t e0, size_t e1) {
    const size_t es = DataTypeSize(t.dtype);
    const size_t chunk = slot_bytes_ / es;
    const int M = view_.machine_count;
    const int root_machine = view_.machine_of[t.root];
    Channel& C = chans_[ch];
    char* buf = static_cast<char*>(t.recv_buf);
    const char* in = static_cast<const char*>(t.send_buf ? t.send_buf : t.recv_buf);
    for (size_t off = e0; off < e1; off += chunk) {
        NextBuffers(ch);
        const size_t clen = std::min(chunk, e1 - off);
        if (rank_ == t.root) memcpy(C.result, in + off * es, clen * es);
        Mark(ch, kTrCopyIn);
        if (!Barrier(ch)) return false;
        if (M > 1 && view_.local_rank == 0) {
            std::vector<int> peers;
            std::vector<const void*> sends;
            std::vector<size_t> sb, rb;
            std::vector<void*> recvs;
            for (int m = 0; m < M; ++m) {
                if (m == view_.machine_index) continue;
                if (view_.machine_index == root_machine) {
                    peers.push_back(m);
                    sends.push_back(C.result);
                    sb.push_back(clen * es);
                    recvs.push_back(nullptr);
                    rb.push_back(0);
                } else if (m == root_machine) {
                    peers.push_back(m);
                    sends.push_back(nullptr);
                    sb.push_back(0);
                    recvs.push_back(C.result);
                    rb.push_back(clen * es);
                }
            }
            if (!LeaderExchange(ch, peers, sends, sb, recvs, rb)) return false;
            Mark(ch, kTrExchange);
        }
        if (M > 1 && !Barrier(ch)) return false;
        if (rank_ != t.root || buf != in) memcpy(buf + off * es, C.result, clen * es);
        Mark(ch, kTrCopyOut);
    }
    return true;
}

bool HostEngine::AllGatherSlice(int ch, const CollTask& t, size_t e0, size_t e1) {
    const size_t es = DataTypeSize(t.dtype);
    const size_t chunk = slot_bytes_ / es;
    const int M = view_.machine_count;
    const char* src = static_cast<const char*>(t.send_buf);
    char* dst = static_cast<char*>(t.recv_buf);
    for (size_t off = e0; off < e1; off += chunk) {
        NextBuffers(ch);
        const size_t clen = std::min(chunk, e1 - off);
        memcpy(Slot(ch, rank_), src + off * es, clen * es);
        Mark(ch, kTrCopyIn);
        if (!Barrier(ch)) return false;
        if (M > 1 && view_.local_rank == 0) {
            // Exchange whole machines' slots; a machine's ranks are not contiguous in
            // general, so each slot travels separately in machine-rank order.
            std::vector<int> peers;
            std::vector<const void*> sends;
            std::vector<size_t> sb, rb;
            std::vector<void*> recvs;
            for (int m = 0; m < M; ++m) {
                if (m == view_.machine_index) continue;
                size_t nmine = view_.machine_ranks[view_.machine_index].size();
                size_t ntheirs = view_.machine_ranks[m].size();
                for (size_t k = 0; k < std::max(nmine, ntheirs); ++k) {
                    peers.push_back(m);
                    sends.push_back(k < nmine ? Slot(ch, view_.machine_ranks[view_.machine_index][k]) : nullptr);
                    sb.push_back(k < nmine ? clen * es : 0);
                    recvs.push_back(k < ntheirs ? Slot(ch, view_.machine_ranks[m][k]) : nullptr);
                    rb.push_back(k < ntheirs ? clen * es : 0);
                }
            }
            // Slots to one peer must go in order on its single socket: run one k at a time.
            size_t i = 0;
            while (i < peers.size()) {
                std::vector<int> p1;
                std::vector<const void*> s1;
                std::vector<size_t> sb1, rb1;
                std::vector<void*> r1;
                std::vector<char> used(M, 0);
                size_t j = i;
                for (; j < peers.size() && !used[peers[j]]; ++j) {
                    used[peers[j]] = 1;
                    p1.push_back(peers[j]);
                    s1.push_back(sends[j]);
                    sb1.push_back(sb[j]);
                    r1.push_back(recvs[j]);
                    rb1.push_back(rb[j]);
                }
                if (!LeaderExchange(ch, p1, s1, sb1, r1, rb1)) return false;
                i = j;
            }
            Mark(ch, kTrExchange);
        }
        if (M > 1 && !Barrier(ch)) return false;
        for (int q = 0; q < world_; ++q) {
            char* out = dst + (static_cast<size_t>(q) * t.count + off) * es;
            const char* in = (q == rank_) ? src + off * es : Slot(ch, q);
            if (out != in) memcpy(out, in, clen * es);
        }
        Mark(ch, kTrCopyOut);
    }
    return true;
}

bool HostEngine::ReduceScatterSlice(int ch, const CollTask& t, size_t e0, size_t e1) {
    const size_t es = DataTypeSize(t.dtype);
    const size_t chunk = std::max<size_t>(1, slot_bytes_ / (es * static_cast<size_t>(world_)));
    const int L = view_.local_size, li = view_.local_rank, M = view_.machine_count;
    Channel& C = chans_[ch];
    const char* src = static_cast<const char*>(t.send_buf);
    char* dst = static_cast<char*>(t.recv_buf);
    for (size_t off = e0; off < e1; off += chunk) {
        NextBuffers(ch);
        const size_t clen = std::min(chunk, e1 - off);
        const size_t sub = clen * es;
        // My slot holds [world][clen]: sub-chunk s is my contribution to rank s's output.
        for (int s = 0; s < world_; ++s)
            memcpy(Slot(ch, rank_) + static_cast<size_t>(s) * sub, src + (static_cast<size_t>(s) * t.count + off) * es, sub);
        Mark(ch, kTrCopyIn);
        if (!Barrier(ch)) return false;
        for (int s = li; s < world_; s += L) {
            const void* srcs[64];
            for (int i = 0; i < L; ++i) srcs[i] = Slot(ch, view_.local_ranks[i]) + static_cast<size_t>(s) * sub;
            hostmath::Reduce(t.dtype, t.op, C.result + static_cast<size_t>(s) * sub, srcs, L, clen, world_, t.scale, M == 1);
        }
        Mark(ch, kTrReduce);
        if (!Barrier(ch)) return false;
        if (M > 1 && view_.local_rank == 0) {
            // Send machine m the partials of its ranks; receive our ranks' partials from every machine.
            const std::vector<int>& mine = view_.machine_ranks[view_.machine_index];
            C.scratch.resize(static_cast<size_t>(M) * mine.size() * sub);
            std::vector<char> sendbuf;
            std::vector<std::vector<char>> outs(M);
            std::vector<int> peers;
            std::vector<const void*> sends;
            std::vector<size_t> sb, rb;
            std::vector<void*> recvs;
            for (int m = 0; m < M; ++m) {
                if (m == view_.machine_index) continue;
                for (int q : view_.machine_ranks[m])
                    outs[m].insert(outs[m].end(), C.result + static_cast<size_t>(q) * sub, C.result + static_cast<size_t>(q + 1) * sub);
                peers.push_back(m);
                sends.push_back(outs[m].data());
                sb.push_back(outs[m].size());
                recvs.push_back(C.scratch.data() + static_cast<size_t>(m) * mine.size() * sub);
                rb.push_back(mine.size() * sub);
            }
            if (!LeaderExchange(ch, peers, sends, sb, recvs, rb)) return false;
            for (size_t k = 0; k < mine.size(); ++k) {
                std::vector<const void*> srcs(M);
                for (int m = 0; m < M; ++m) {
                    srcs[m] = (m == view_.machine_index) ? static_cast<const void*>(C.result + static_cast<size_t>(mine[k]) * sub)
                                                         : static_cast<const void*>(C.scratch.data() + (static_cast<size_t>(m) * mine.size() + k) * sub);
                }
                hostmath::Reduce(t.dtype, t.op, C.result + static_cast<size_t>(mine[k]) * sub, srcs.data(), M, clen, world_, t.scale, true);
            }
            Mark(ch, kTrExchange);
        }
        if (M > 1 && !Barrier(ch)) return false;
        memcpy(dst + off * es, C.result + static_cast<size_t>(rank_) * sub, sub);
        Mark(ch, kTrCopyOut);
    }
    return true;
}

bool HostEngine::RunSlice(int ch, const CollTask& t, size_t e0, size_t e1) {
    if (trace_cap_) {
        chans_[ch].trace_func = static_cast<uint16_t>(t.func);
        chans_[ch].trace_slice++;
        Mark(ch, kTrSliceBegin);
    }
    bool ok = false;
    switch (t.func) {
    case CollFunc::AllReduce: ok = AllReduceSlice(ch, t, e0, e1, false); break;
    case CollFunc::Reduce: ok = AllReduceSlice(ch, t, e0, e1, true); break;
    case CollFunc::Broadcast: ok = BroadcastSlice(ch, t, e0, e1); break;
    case CollFunc::AllGather: ok = AllGatherSlice(ch, t, e0, e1); break;
    case CollFunc::ReduceScatter: ok = ReduceScatterSlice(ch, t, e0, e1); break;
    default: break;
    }
    Mark(ch, kTrSliceEnd);
    return ok;
}

long HostEngine::DumpTrace(const char* path) {
    if (trace_cap_ == 0) return -1;
    FILE* f = fopen(path, "w");
    if (f == nullptr) return -1;
    // The phase that ends at an event, by event.
    static const char* kPhase[] = {"?", "idle", "copy_in", "barrier_wait", "reduce", "leader_exchange", "copy_out",
                                   "tail"};
    fprintf(f, "{\"traceEvents\":[\n");
    long n = 0;
    for (int ch = 0; ch < n_channels_; ++ch) {
        std::vector<TraceRec>& tr = chans_[ch].trace;
        for (size_t i = 1; i < tr.size(); ++i) {
            const TraceRec& a = tr[i - 1];
            const TraceRec& b = tr[i];
            if (b.event == kTrSliceBegin || b.slice != a.slice) continue;  // between slices: idle
            fprintf(f, "%s{\"name\":\"%s\",\"ph\":\"X\",\"ts\":%.3f,\"dur\":%.3f,\"pid\":%d,\"tid\":%d,"
                       "\"args\":{\"op\":\"%s\",\"slice\":%u}}\n",
                    n ? "," : "", kPhase[b.event < 8 ? b.event : 0], a.t_ns / 1000.0, (b.t_ns - a.t_ns) / 1000.0, rank_,
                    ch, CollFuncName(static_cast<CollFunc>(b.func)), b.slice);
            ++n;
        }
        tr.clear();
    }
    fprintf(f, "]}\n");
    fclose(f);
    return n;
}

bool HostEngine::RunP2p(const std::vector<CollTask>& tasks) {
    // FIFO per (peer, direction): only the head op of each queue is active.
    // Messages of at least cma_bytes_ to a rank of this machine go single-copy: the sender
    // writes a CmaDesc into the ring instead of the payload and completes once the receiver has
    // acked; the receiver reads the descriptor, copies the payload straight out of the sender's
    // buffer (process_vm_readv) and acks. Both sides take the same decision from the size.
    struct Op {
        const CollTask* t;
        size_t progress;
        int state;        // zero-copy: 0 descriptor in flight, 1 waiting for the ack / copying
        uint64_t target;  // zero-copy send: the ack count that completes it
        CmaDesc desc;
    };
    std::map<std::pair<int, int>, std::vector<Op>> queues;
    for (const CollTask& t : tasks) {
        if (t.count == 0) continue;
        Op op{&t, 0, 0, 0, {}};
        if (t.func == CollFunc::Send) {
            op.desc = {kCmaMagic, static_cast<int64_t>(getpid()), reinterpret_cast<uint64_t>(t.send_buf),
                       t.count * DataTypeSize(t.dtype)};
        }
        queues[{t.peer, t.func == CollFunc::Send ? 0 : 1}].push_back(op);
    }
    auto zero_copy = [&](const CollTask& t, size_t bytes) {
        return cma_ && bytes >= cma_bytes_ && view_.machine_of[t.peer] == view_.machine_index;
    };
    auto acks = [&](int sender, int receiver) -> std::atomic<uint64_t>& {
        return cma_acks_[static_cast<size_t>(view_.local_index_of[sender]) * static_cast<size_t>(view_.local_size) +
                         static_cast<size_t>(view_.local_index_of[receiver])];
    };
    std::map<std::pair<int, int>, size_t> head;
    for (auto& kv : queues) head[kv.first] = 0;
    int ep = -1;
    if (epoll_) ep = epoll_create1(EPOLL_CLOEXEC);
    auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms_);
    bool ok = true;
    for (;;) {
        bool all = true, progress = false, need_poll_shm = false;
        for (auto& kv : queues) {
            size_t& h = head[kv.first];
            while (h < kv.second.size()) {
                Op& op = kv.second[h];
                const CollTask& t = *op.t;
                const size_t bytes = t.count * DataTypeSize(t.dtype);
                Transport* tr = kv.first.second == 0 ? p2p_send_[t.peer].get() : p2p_recv_[t.peer].get();
                if (tr == nullptr) {
                    LOG_ERROR("rank %d: no transport to rank %d", rank_, t.peer);
                    ok = false;
                    break;
                }
                size_t before = op.progress;
                bool done = false;
                const bool send = kv.first.second == 0;
                bool r = true;
                if (!zero_copy(t, bytes)) {
                    r = send ? tr->TrySend(t.send_buf, bytes, &op.progress, &done)
                             : tr->TryRecv(t.recv_buf, bytes, &op.progress, &done);
                } else if (op.state == 0) {  // the descriptor goes through the ring, in FIFO order
                    bool sent = false;
                    r = send ? tr->TrySend(&op.desc, sizeof(CmaDesc), &op.progress, &sent)
                             : tr->TryRecv(&op.desc, sizeof(CmaDesc), &op.progress, &sent);
                    if (r && sent) {
                        op.state = 1;
                        if (send) op.target = ++cma_sent_[static_cast<size_t>(t.peer)];
                    }
                }
                if (r && zero_copy(t, bytes) && op.state == 1) {
                    if (send) {
                        done = acks(rank_, t.peer).load(std::memory_order_acquire) >= op.target;
                    } else if (op.desc.magic != kCmaMagic || op.desc.bytes != bytes) {
                        LOG_ERROR("rank %d: zero-copy message from rank %d does not match the receive (%llu vs %zu bytes)",
                                  rank_, t.peer, static_cast<unsigned long long>(op.desc.bytes), bytes);
                        r = false;
                    } else {
                        size_t got = 0;
                        while (r && got < bytes) {
                            struct iovec mine = {static_cast<char*>(t.recv_buf) + got, bytes - got};
                            struct iovec theirs = {reinterpret_cast<char*>(op.desc.addr) + got, bytes - got};
                            const ssize_t k = process_vm_readv(static_cast<pid_t>(op.desc.pid), &mine, 1, &theirs, 1, 0);
                            if (k <= 0) {
                                LOG_ERROR("rank %d: zero-copy read from rank %d failed: %s", rank_, t.peer, strerror(errno));
                                r = false;
                            } else {
                                got += static_cast<size_t>(k);
                            }
                        }
                        if (r) {
                            acks(t.peer, rank_).fetch_add(1, std::memory_order_release);
                            cma_transfers_.fetch_add(1, std::memory_order_relaxed);
                            done = true;
                        }
                    }
                    progress |= done;
                }
                if (!r) {
                    ok = false;
                    break;
                }
                progress |= op.progress != before;
                if (!done) {
                    if (tr->GetFd() < 0 || zero_copy(t, bytes)) need_poll_shm = true;
                    break;
                }
                ++h;
            }
            if (!ok) break;
            all &= h == kv.second.size();
        }
        if (!ok || all) break;
        if (!progress) {
            if (aborted_.load(std::memory_order_relaxed)) {
                LOG_ERROR("rank %d: Send/Recv aborted", rank_);
                ok = false;
                break;
            }
            if (Clock::now() > deadline) {
                LOG_ERROR("rank %d: Send/Recv timed out after %d ms", rank_, timeout_ms_);
                ok = false;
                break;
            }
            if (ep >= 0 && !need_poll_shm) {
                // Event-driven wait on the sockets of every pending head op.
                for (auto& kv : queues) {
                    size_t h = head[kv.first];
                    if (h >= kv.second.size()) continue;
                    int fd = p2p_send_[kv.first.first] ? p2p_send_[kv.first.first]->GetFd() : -1;
                    if (fd < 0) continue;
                    struct epoll_event ev;
                    ev.events = kv.first.second == 0 ? EPOLLOUT : EPOLLIN;
                    ev.data.fd = fd;
                    if (epoll_ctl(ep, EPOLL_CTL_ADD, fd, &ev) != 0) epoll_ctl(ep, EPOLL_CTL_MOD, fd, &ev);
                }
                struct epoll_event evs[16];
                epoll_wait(ep, evs, 16, 50);
            } else {
                sched_yield();
            }
        }
    }
    if (ep >= 0) close(ep);
    return ok;
}

bool HostEngine::Execute(const std::vector<CollTask>& sorted) {
    if (!inited_) {
        LOG_ERROR("host engine not initialised");
        return false;
    }
    std::vector<CollTask> p2p;
    std::vector<const CollTask*> work;
    for (const CollTask& t : sorted) {
        if (IsP2p(t.func)) {
            p2p.push_back(t);
            continue;
        }
        if (t.count == 0) continue;
        if (world_ == 1) {
            // Single rank: the collective is a local copy (plus AVG/scale).
            size_t n = t.count;
            const void* in = t.send_buf ? t.send_buf : t.recv_buf;
            if (t.func == CollFunc::Reduce || t.func == CollFunc::AllReduce || t.func == CollFunc::ReduceScatter) {
                hostmath::Finish(t.dtype, t.op, t.recv_buf, in, n, 1, t.scale);
            } else if (t.recv_buf != in) {
                memmove(t.recv_buf, in, n * DataTypeSize(t.dtype));
            }
            continue;
        }
        work.push_back(&t);
    }
    if (!work.empty()) {
        const std::vector<std::vector<WorkUnit>> plan = PlanChannels(work);
        auto run = [this, &plan](int ch) {
            for (const WorkUnit& u : plan[static_cast<size_t>(ch)])
                if (!RunSlice(ch, *u.task, u.e0, u.e1)) return false;
            return true;
        };
        std::vector<int> busy;
        int last = -1;
        for (int ch = 0; ch < n_channels_; ++ch) {
            if (!plan[static_cast<size_t>(ch)].empty()) {
                busy.push_back(ch);
                last = ch;
            }
        }
        // One busy channel (a small collective, or a small group): run it on this thread, with
        // no hand-off to a worker. Otherwise the workers run the others while this thread runs
        // the last one. The per-channel barriers are in shared memory, so which thread of a rank
        // runs a channel does not matter to the other ranks.
        if (busy.size() == 1) {
            if (!run(last)) return false;
        } else if (!RunOnChannels(run, last, busy)) {
            return false;
        }
    }
    return RunP2p(p2p);
}

// The whole batch becomes one job per channel thread. A collective of at least split_bytes_
// (BCCL_HOST_SPLIT_BYTES; default 256 KiB with four channels, else 1 MiB) is cut into one slice
// per channel; a smaller one goes whole to the channel with the fewest bytes so far (ties: lowest
// index). The plan depends only on the sorted task list,
// which every rank builds identically, so channel c runs the same slices in the same order on
// every rank and the per-channel barriers and connections line up. This is the reference's
// dynamic executor's goal (many small collectives spread over the channels instead of each one
// waking every channel) without its rank-0 in-band broadcast.
std::vector<std::vector<HostEngine::WorkUnit>> HostEngine::PlanChannels(const std::vector<const CollTask*>& work) const {
    std::vector<std::vector<WorkUnit>> plan(static_cast<size_t>(n_channels_));
    std::vector<size_t> load(static_cast<size_t>(n_channels_), 0);
    for (const CollTask* t : work) {
        const size_t bytes = t->count * DataTypeSize(t->dtype);
        if (bytes < split_bytes_ || n_channels_ == 1) {
            size_t best = 0;
            for (size_t c = 1; c < load.size(); ++c)
                if (load[c] < load[best]) best = c;
            plan[best].push_back({t, 0, t->count});
            load[best] += bytes;
            continue;
        }
        for (int ch = 0; ch < n_channels_; ++ch) {
            size_t e0, e1;
            ChannelSlice(t->count, n_channels_, ch, &e0, &e1);
            if (e1 > e0) {
                plan[static_cast<size_t>(ch)].push_back({t, e0, e1});
                load[static_cast<size_t>(ch)] += (e1 - e0) * DataTypeSize(t->dtype);
            }
        }
    }
    return plan;
}

}  // namespace bccl
