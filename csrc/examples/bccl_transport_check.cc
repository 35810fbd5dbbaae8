// bccl_transport_check: semantics suite of the host transports (TCP socket, shared-memory ring).
//
//   bccl_transport_check tcp|shm
//
// Two processes (fork): the parent sends, the child receives, over one transport instance each.
// Cases, with the declared differences between the two movers:
//   * poll contract: TCP exposes its socket fd with POLLOUT/POLLIN; the SHM ring has no fd
//     (GetFd() == -1) and is polled;
//   * zero-size transfers are done at once on both ends;
//   * direction: the SHM ring rejects TrySend on the consumer end and TryRecv on the producer end;
//     a TCP socket is bidirectional;
//   * boundaries: 1 B .. 5 MiB around powers of two and the 2 MiB ring capacity, byte-exact,
//     with progress monotone and done <=> progress == size;
//   * back-pressure: a send to a receiver that does not read for 400 ms stalls without error,
//     then completes when the receiver drains (8 MiB over the 2 MiB ring; 64 MiB over TCP, whose
//     loopback socket buffers can absorb several MiB);
//   * close: after the peer closes, TCP reports an error to the receiver once the stream is
//     drained; the SHM ring has no peer-death signal (it just has no data).
// The parent prints one JSON line {"transport", "passed", "failed", "failures"}; exit status is
// non-zero on any failure.
//
// Parity: OriginCCL tests/transport_check.{h,cpp} (one suite for every transport with declared
// differences: direction, poll mask, close; sizes 1 B-5 MiB; 8 MiB back-pressure).
#include <poll.h>
#include <sys/mman.h>
#include <sys/socket.h>
#include <sys/wait.h>
#include <unistd.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "core/net.h"
#include "host/transport.h"

using bccl::ShmRingCtrl;
using bccl::ShmRingTransport;
using bccl::TcpTransport;
using bccl::Transport;

namespace {

constexpr size_t kRingBytes = 2u << 20;

std::vector<size_t> BoundarySizes() {
    std::vector<size_t> s = {1, 2, 7, 8, 63, 64, 65, 4095, 4096, 4097, 65535, 65536, 65537};
    for (size_t b : {size_t(1) << 20, kRingBytes, size_t(4) << 20}) {
        s.push_back(b - 1);
        s.push_back(b);
        s.push_back(b + 1);
    }
    s.push_back(size_t(5) << 20);
    return s;
}

size_t BackPressureBytes(bool tcp) { return tcp ? size_t(16) << 20 : size_t(8) << 20; }

// Loopback TCP autotunes its buffers up to the system maximum, which on some hosts absorbs the
// whole back-pressure message; fixed 256 KiB socket buffers on both ends make the stall certain.
void CapSocketBuffers(int fd) {
    const int bytes = 256 << 10;
    setsockopt(fd, SOL_SOCKET, SO_SNDBUF, &bytes, sizeof(bytes));
    setsockopt(fd, SOL_SOCKET, SO_RCVBUF, &bytes, sizeof(bytes));
}

uint8_t Pattern(size_t size, size_t i) { return static_cast<uint8_t>((i * 131 + size * 7 + (i >> 9)) & 0xff); }

using Clock = std::chrono::steady_clock;

// Drives one transfer to completion (or error / deadline), checking the progress contract.
bool Drive(Transport* t, bool send, void* buf, size_t size, int timeout_ms, std::string* why) {
    size_t progress = 0, last = 0;
    bool done = false;
    auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
    while (true) {
        bool ok = send ? t->TrySend(buf, size, &progress, &done) : t->TryRecv(buf, size, &progress, &done);
        if (!ok) {
            *why = "transport error at " + std::to_string(progress) + "/" + std::to_string(size);
            return false;
        }
        if (progress < last || progress > size || done != (progress == size)) {
            *why = "progress contract broken";
            return false;
        }
        last = progress;
        if (done) return true;
        if (Clock::now() > deadline) {
            *why = "timeout at " + std::to_string(progress) + "/" + std::to_string(size);
            return false;
        }
        if (t->GetFd() >= 0) {
            pollfd p{t->GetFd(), t->GetPollEvents(send), 0};
            poll(&p, 1, 10);
        } else {
            std::this_thread::yield();
        }
    }
}

struct Report {
    int passed = 0, failed = 0;
    std::vector<std::string> failures;
    void Check(bool ok, const std::string& what) {
        if (ok) {
            ++passed;
        } else {
            ++failed;
            if (failures.size() < 10) failures.push_back(what);
        }
    }
};

// Receiver side (child process). Returns the number of failures.
int Receiver(Transport* t, bool tcp) {
    int bad = 0;
    std::string why;
    uint8_t z = 0;
    if (!Drive(t, false, &z, 0, 1000, &why)) ++bad;
    for (size_t size : BoundarySizes()) {
        std::vector<uint8_t> buf(size);
        if (!Drive(t, false, buf.data(), size, 20000, &why)) {
            std::fprintf(stderr, "recv %zu: %s\n", size, why.c_str());
            return bad + 1;
        }
        for (size_t i = 0; i < size; ++i) {
            if (buf[i] != Pattern(size, i)) {
                std::fprintf(stderr, "recv %zu: byte %zu differs\n", size, i);
                ++bad;
                break;
            }
        }
    }
    // Back-pressure: do not read for 400 ms (the sender watches for 100 ms), then drain.
    std::this_thread::sleep_for(std::chrono::milliseconds(400));
    const size_t bp = BackPressureBytes(tcp);
    std::vector<uint8_t> buf(bp);
    if (!Drive(t, false, buf.data(), bp, 20000, &why)) return bad + 1;
    for (size_t i = 0; i < bp; ++i) {
        if (buf[i] != Pattern(bp, i)) {
            ++bad;
            break;
        }
    }
    if (tcp) {
        // The sender closes after its last message: the next receive must fail, not hang.
        std::string msg;
        uint8_t one = 0;
        bool failed_as_expected = !Drive(t, false, &one, 1, 5000, &msg) && msg.find("timeout") == std::string::npos;
        if (!failed_as_expected) {
            std::fprintf(stderr, "close not detected: %s\n", msg.c_str());
            ++bad;
        }
    }
    return bad;
}

int Run(bool tcp) {
    Report rep;
    std::unique_ptr<Transport> tx;
    int listen_fd = -1;
    uint16_t port = 0;
    ShmRingCtrl* ctrl = nullptr;
    char* ring = nullptr;
    if (tcp) {
        listen_fd = bccl::net::Listen(0, &port);
        if (listen_fd < 0) return 2;
    } else {
        void* mem = mmap(nullptr, sizeof(ShmRingCtrl) + kRingBytes, PROT_READ | PROT_WRITE, MAP_SHARED | MAP_ANONYMOUS,
                         -1, 0);
        if (mem == MAP_FAILED) return 2;
        ctrl = new (mem) ShmRingCtrl();
        ctrl->head.store(0);
        ctrl->tail.store(0);
        ring = static_cast<char*>(mem) + sizeof(ShmRingCtrl);
    }
    std::fflush(stdout);
    pid_t child = fork();
    if (child < 0) return 2;
    if (child == 0) {
        std::unique_ptr<Transport> t;
        if (tcp) {
            int fd = bccl::net::Accept(listen_fd, 10000);
            if (fd < 0) _exit(3);
            CapSocketBuffers(fd);
            t.reset(new TcpTransport(fd));
        } else {
            t.reset(new ShmRingTransport(ctrl, ring, kRingBytes, /*producer=*/false));
        }
        int bad = Receiver(t.get(), tcp);
        t->Close();
        _exit(bad == 0 ? 0 : 1);
    }
    if (tcp) {
        int fd = bccl::net::Connect("127.0.0.1", port, 10000);
        if (fd < 0) return 2;
        CapSocketBuffers(fd);
        tx.reset(new TcpTransport(fd));
        rep.Check(tx->GetFd() >= 0 && tx->GetPollEvents(true) == POLLOUT && tx->GetPollEvents(false) == POLLIN,
                  "tcp exposes its fd with POLLOUT/POLLIN");
    } else {
        tx.reset(new ShmRingTransport(ctrl, ring, kRingBytes, /*producer=*/true));
        rep.Check(tx->GetFd() == -1, "shm ring has no readiness fd");
        // A second handle on the same ring, used only to check direction enforcement.
        ShmRingTransport wrong_end(ctrl, ring, kRingBytes, /*producer=*/true);
        size_t pr = 0;
        bool dn = false;
        uint8_t b = 0;
        rep.Check(!wrong_end.TryRecv(&b, 1, &pr, &dn), "shm producer end rejects TryRecv");
        ShmRingTransport consumer_view(ctrl, ring, kRingBytes, /*producer=*/false);
        rep.Check(!consumer_view.TrySend(&b, 1, &pr, &dn), "shm consumer end rejects TrySend");
    }
    std::string why;
    uint8_t z = 0;
    // The back-pressure message is prepared first, so the sender's stall window below starts as
    // soon as the last boundary message is handed over, well inside the receiver's pause (even
    // when an instrumented build makes filling 16 MiB slow).
    const size_t bp = BackPressureBytes(tcp);
    std::vector<uint8_t> buf(bp);
    for (size_t i = 0; i < bp; ++i) buf[i] = Pattern(bp, i);
    rep.Check(Drive(tx.get(), true, &z, 0, 1000, &why), "zero-size send done at once");
    for (size_t size : BoundarySizes()) {
        std::vector<uint8_t> msg(size);
        for (size_t i = 0; i < size; ++i) msg[i] = Pattern(size, i);
        rep.Check(Drive(tx.get(), true, msg.data(), size, 20000, &why), "send " + std::to_string(size) + ": " + why);
    }
    // Back-pressure: while the receiver sleeps, progress must stall below the message size.
    size_t progress = 0;
    bool done = false, ok = true;
    auto until = Clock::now() + std::chrono::milliseconds(100);
    while (ok && Clock::now() < until) {
        ok = tx->TrySend(buf.data(), bp, &progress, &done);
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
    rep.Check(ok && !done && progress < bp, "send stalls without error while the receiver does not read (progress " +
                                                std::to_string(progress) + ")");
    bool finished = ok;
    auto deadline = Clock::now() + std::chrono::seconds(20);
    while (finished && !done && Clock::now() < deadline) {
        finished = tx->TrySend(buf.data(), bp, &progress, &done);
        if (!done) std::this_thread::yield();
    }
    rep.Check(finished && done, "back-pressured send completes once the receiver drains");
    tx->Close();  // TCP receiver must then see the close
    int status = 0;
    waitpid(child, &status, 0);
    rep.Check(WIFEXITED(status) && WEXITSTATUS(status) == 0,
              "receiver saw byte-exact data" + std::string(tcp ? " and the close" : ""));
    if (tcp) bccl::net::CloseFd(&listen_fd);
    std::printf("{\"transport\": \"%s\", \"passed\": %d, \"failed\": %d, \"failures\": [", tcp ? "tcp" : "shm",
                rep.passed, rep.failed);
    for (size_t i = 0; i < rep.failures.size(); ++i) std::printf("%s\"%s\"", i ? ", " : "", rep.failures[i].c_str());
    std::printf("]}\n");
    return rep.failed == 0 ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
    std::string which = argc > 1 ? argv[1] : "";
    if (which != "tcp" && which != "shm") {
        std::fprintf(stderr, "usage: bccl_transport_check tcp|shm\n");
        return 2;
    }
    return Run(which == "tcp");
}
