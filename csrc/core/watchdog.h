// Liveness watchdog: every rank keeps one extra TCP connection to rank 0 after the bootstrap,
// and a thread per rank watches it. A rank whose process ends without finalizing closes its
// socket without the goodbye byte; rank 0 sees the end of stream, tells every other rank
// ('A'), and every rank aborts its communicator (host waits give up at once, device waits
// within a millisecond). A rank also aborts when rank 0 vanishes. Finalize sends a goodbye
// ('B') first, so an orderly exit is never mistaken for a failure.
//
// The reference has no failure detection beyond timeouts (its executors stop on the first
// error); this turns "a peer died" from a 30 s timeout into a prompt error on every rank.
#pragma once

#include <atomic>
#include <functional>
#include <thread>
#include <vector>

#include "bccl/types.h"

namespace bccl {

class Bootstrap;

class Watchdog {
public:
    ~Watchdog() { Stop(); }

    // Collective over the communicator, right after the bootstrap. listen_fd: rank 0's
    // bootstrap listener (borrowed). on_failure runs on the watchdog thread, at most once.
    bool Start(const CommConfig& cfg, int listen_fd, Bootstrap* bs, std::function<void(int)> on_failure);
    // Sends the goodbye, stops the thread and closes the sockets.
    void Stop();
    bool failed() const { return failed_.load(); }

private:
    void Loop();
    void Fail(int peer);

    int rank_ = 0;
    int world_ = 1;
    std::vector<int> fds_;  // rank 0: per rank (index 0 unused); others: fds_[0] = link to rank 0
    std::vector<char> gone_;  // peer said goodbye
    int wake_[2] = {-1, -1};  // self-pipe to stop the thread
    std::thread thread_;
    std::function<void(int)> on_failure_;
    std::atomic<bool> failed_{false};
    bool running_ = false;
};

}  // namespace bccl
