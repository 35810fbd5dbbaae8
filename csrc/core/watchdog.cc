#include "core/watchdog.h"

#include <poll.h>
#include <sys/socket.h>
#include <unistd.h>

#include <chrono>

#include "core/bootstrap.h"
#include "core/logger.h"
#include "core/net.h"

namespace bccl {
namespace {

constexpr uint32_t kLiveMagic = 0xBCC10A11u;
constexpr char kBye = 'B';
constexpr char kAbort = 'A';

}  // namespace

bool Watchdog::Start(const CommConfig& cfg, int listen_fd, Bootstrap* bs, std::function<void(int)> on_failure) {
    rank_ = cfg.rank;
    world_ = cfg.world_size;
    on_failure_ = std::move(on_failure);
    if (world_ == 1) return true;
    const int timeout_ms = bs->timeout_ms();
    bool ok = true;
    if (rank_ == 0) {
        fds_.assign(world_, -1);
        int joined = 1;
        auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
        while (ok && joined < world_) {
            const int left = static_cast<int>(std::chrono::duration_cast<std::chrono::milliseconds>(
                                                  deadline - std::chrono::steady_clock::now())
                                                  .count());
            if (left <= 0) {
                LOG_ERROR("watchdog: only %d of %d ranks connected", joined, world_);
                ok = false;
                break;
            }
            int fd = net::Accept(listen_fd, left);
            if (fd < 0) continue;
            std::vector<uint8_t> hello;
            uint32_t magic = 0;
            int32_t rank = -1;
            bool good = net::RecvFrame(fd, &hello, timeout_ms, 64);
            if (good) {
                net::Reader r(hello);
                good = r.U32(&magic) && magic == kLiveMagic && r.I32(&rank) && rank > 0 && rank < world_ &&
                       fds_[rank] < 0;
            }
            if (!good) {
                LOG_ERROR("watchdog: bad liveness hello");
                close(fd);
                ok = false;
                break;
            }
            fds_[rank] = fd;
            ++joined;
        }
    } else {
        fds_.assign(1, -1);
        fds_[0] = net::Connect(cfg.unique_id.ip_addr, cfg.unique_id.port, timeout_ms);
        net::Writer w;
        w.U32(kLiveMagic);
        w.I32(rank_);
        ok = fds_[0] >= 0 && net::SendFrame(fds_[0], w.bytes(), timeout_ms);
        if (!ok) LOG_ERROR("watchdog: rank %d could not connect to rank 0", rank_);
    }
    // Every rank's link exists (or every rank learns that one does not) before anyone watches.
    std::vector<uint8_t> mine(1, ok ? 1 : 0);
    std::vector<std::vector<uint8_t>> all;
    if (!bs->AllGather(mine, &all)) ok = false;
    for (const auto& a : all) ok = ok && !a.empty() && a[0] == 1;
    if (!ok || pipe(wake_) != 0) {
        for (int& fd : fds_) net::CloseFd(&fd);
        return false;
    }
    gone_.assign(fds_.size(), 0);
    running_ = true;
    thread_ = std::thread(&Watchdog::Loop, this);
    return true;
}

void Watchdog::Fail(int peer) {
    if (failed_.exchange(true)) return;
    if (rank_ == 0) {
        LOG_ERROR("watchdog: rank %d ended without finalizing; aborting every rank", peer);
        for (size_t r = 1; r < fds_.size(); ++r) {
            if (fds_[r] >= 0 && !gone_[r] && static_cast<int>(r) != peer) {
                const char a = kAbort;
                (void)send(fds_[r], &a, 1, MSG_NOSIGNAL | MSG_DONTWAIT);
            }
        }
    } else {
        LOG_ERROR("watchdog: rank %d: %s; aborting", rank_,
                  peer == 0 ? "rank 0 ended without finalizing" : "rank 0 reported a failed rank");
    }
    if (on_failure_) on_failure_(peer);
}

void Watchdog::Loop() {
    for (;;) {
        std::vector<pollfd> pf;
        std::vector<int> who;
        pf.push_back({wake_[0], POLLIN, 0});
        who.push_back(-1);
        for (size_t i = 0; i < fds_.size(); ++i) {
            if (fds_[i] >= 0 && !gone_[i]) {
                pf.push_back({fds_[i], POLLIN, 0});
                who.push_back(static_cast<int>(i));
            }
        }
        if (poll(pf.data(), pf.size(), -1) < 0) continue;
        if (pf[0].revents) return;  // Stop()
        for (size_t k = 1; k < pf.size(); ++k) {
            if (!pf[k].revents) continue;
            const int i = who[k];
            char c = 0;
            const ssize_t n = recv(fds_[i], &c, 1, MSG_DONTWAIT);
            if (n == 1 && c == kBye) {
                gone_[i] = 1;
            } else if (n == 1 && c == kAbort) {
                gone_[i] = 1;
                Fail(-1);
            } else if (n == 0 || (n < 0 && errno != EAGAIN && errno != EINTR)) {
                gone_[i] = 1;
                Fail(rank_ == 0 ? i : 0);
            }
        }
    }
}

void Watchdog::Stop() {
    if (!running_) return;
    running_ = false;
    for (size_t i = 0; i < fds_.size(); ++i) {
        if (fds_[i] >= 0) {
            const char b = kBye;
            (void)send(fds_[i], &b, 1, MSG_NOSIGNAL | MSG_DONTWAIT);
        }
    }
    const char x = 1;
    (void)write(wake_[1], &x, 1);
    if (thread_.joinable()) thread_.join();
    for (int& fd : fds_) net::CloseFd(&fd);
    close(wake_[0]);
    close(wake_[1]);
    wake_[0] = wake_[1] = -1;
}

}  // namespace bccl
