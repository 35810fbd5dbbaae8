#include "core/net.h"

#include <arpa/inet.h>
#include <cerrno>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <fcntl.h>
#include <ifaddrs.h>
#include <net/if.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <thread>
#include <unistd.h>

#include "core/logger.h"

namespace bccl {
namespace net {
namespace {

using Clock = std::chrono::steady_clock;

int RemainingMs(Clock::time_point deadline) {
    auto left = std::chrono::duration_cast<std::chrono::milliseconds>(deadline - Clock::now()).count();
    return left < 0 ? 0 : static_cast<int>(left);
}

bool WaitFd(int fd, short events, int timeout_ms) {
    struct pollfd p = {fd, events, 0};
    for (;;) {
        int r = poll(&p, 1, timeout_ms);
        if (r > 0) return true;
        if (r == 0) return false;
        if (errno != EINTR) return false;
    }
}

}  // namespace

std::string LocalIpAddress() {
    if (const char* env = std::getenv("BCCL_BOOTSTRAP_ADDR")) {
        if (*env) return env;
    }
    std::string found;
    struct ifaddrs* ifs = nullptr;
    if (getifaddrs(&ifs) == 0) {
        for (struct ifaddrs* it = ifs; it != nullptr; it = it->ifa_next) {
            if (it->ifa_addr == nullptr || it->ifa_addr->sa_family != AF_INET) continue;
            if ((it->ifa_flags & IFF_UP) == 0 || (it->ifa_flags & IFF_LOOPBACK) != 0) continue;
            char buf[INET_ADDRSTRLEN] = {0};
            auto* sin = reinterpret_cast<struct sockaddr_in*>(it->ifa_addr);
            if (inet_ntop(AF_INET, &sin->sin_addr, buf, sizeof(buf)) != nullptr) {
                found = buf;
                break;
            }
        }
        freeifaddrs(ifs);
    }
    return found.empty() ? std::string("127.0.0.1") : found;
}

std::string Hostname() {
    char buf[256] = {0};
    if (gethostname(buf, sizeof(buf) - 1) != 0) return "localhost";
    return buf;
}

int Listen(uint16_t port, uint16_t* bound_port, int backlog) {
    int fd = socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (fd < 0) {
        LOG_ERROR("socket() failed: %s", strerror(errno));
        return -1;
    }
    int one = 1;
    setsockopt(fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    struct sockaddr_in addr;
    memset(&addr, 0, sizeof(addr));
    addr.sin_family = AF_INET;
    addr.sin_addr.s_addr = htonl(INADDR_ANY);
    addr.sin_port = htons(port);
    if (bind(fd, reinterpret_cast<struct sockaddr*>(&addr), sizeof(addr)) != 0 || listen(fd, backlog) != 0) {
        LOG_ERROR("bind/listen on port %u failed: %s", port, strerror(errno));
        close(fd);
        return -1;
    }
    socklen_t len = sizeof(addr);
    getsockname(fd, reinterpret_cast<struct sockaddr*>(&addr), &len);
    if (bound_port) *bound_port = ntohs(addr.sin_port);
    return fd;
}

int Connect(const std::string& ip, uint16_t port, int timeout_ms, int retry_ms) {
    struct sockaddr_in addr;
    memset(&addr, 0, sizeof(addr));
    addr.sin_family = AF_INET;
    addr.sin_port = htons(port);
    if (inet_pton(AF_INET, ip.c_str(), &addr.sin_addr) != 1) {
        LOG_ERROR("invalid IPv4 address '%s'", ip.c_str());
        return -1;
    }
    auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
    for (;;) {
        int fd = socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
        if (fd < 0) return -1;
        if (connect(fd, reinterpret_cast<struct sockaddr*>(&addr), sizeof(addr)) == 0) {
            SetNoDelay(fd);
            return fd;
        }
        int err = errno;
        close(fd);
        if (Clock::now() >= deadline) {
            LOG_ERROR("connect to %s:%u timed out after %d ms: %s", ip.c_str(), port, timeout_ms, strerror(err));
            return -1;
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(retry_ms));
    }
}

int Accept(int listen_fd, int timeout_ms) {
    if (!WaitFd(listen_fd, POLLIN, timeout_ms)) return -1;
    int fd = accept4(listen_fd, nullptr, nullptr, SOCK_CLOEXEC);
    if (fd >= 0) SetNoDelay(fd);
    return fd;
}

bool SendAll(int fd, const void* buf, size_t len, int timeout_ms) {
    const char* p = static_cast<const char*>(buf);
    auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms < 0 ? 1000000000 : timeout_ms);
    while (len > 0) {
        ssize_t n = send(fd, p, len, MSG_NOSIGNAL | MSG_DONTWAIT);
        if (n > 0) {
            p += n;
            len -= static_cast<size_t>(n);
            continue;
        }
        if (n < 0 && errno == EINTR) continue;
        if (n < 0 && (errno == EAGAIN || errno == EWOULDBLOCK)) {
            if (!WaitFd(fd, POLLOUT, RemainingMs(deadline))) return false;
            continue;
        }
        return false;
    }
    return true;
}

bool RecvAll(int fd, void* buf, size_t len, int timeout_ms) {
    char* p = static_cast<char*>(buf);
    auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms < 0 ? 1000000000 : timeout_ms);
    while (len > 0) {
        ssize_t n = recv(fd, p, len, MSG_DONTWAIT);
        if (n > 0) {
            p += n;
            len -= static_cast<size_t>(n);
            continue;
        }
        if (n == 0) return false;  // peer closed
        if (errno == EINTR) continue;
        if (errno == EAGAIN || errno == EWOULDBLOCK) {
            if (!WaitFd(fd, POLLIN, RemainingMs(deadline))) return false;
            continue;
        }
        return false;
    }
    return true;
}

bool SendFrame(int fd, const std::vector<uint8_t>& payload, int timeout_ms) {
    uint64_t n = payload.size();
    return SendAll(fd, &n, sizeof(n), timeout_ms) && (n == 0 || SendAll(fd, payload.data(), n, timeout_ms));
}

bool RecvFrame(int fd, std::vector<uint8_t>* payload, int timeout_ms, size_t max_len) {
    uint64_t n = 0;
    if (!RecvAll(fd, &n, sizeof(n), timeout_ms)) return false;
    if (n > max_len) return false;
    payload->resize(n);
    return n == 0 || RecvAll(fd, payload->data(), n, timeout_ms);
}

bool SetNonBlocking(int fd, bool on) {
    int flags = fcntl(fd, F_GETFL, 0);
    if (flags < 0) return false;
    flags = on ? (flags | O_NONBLOCK) : (flags & ~O_NONBLOCK);
    return fcntl(fd, F_SETFL, flags) == 0;
}

void SetNoDelay(int fd) {
    int one = 1;
    setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
}

void CloseFd(int* fd) {
    if (fd && *fd >= 0) {
        close(*fd);
        *fd = -1;
    }
}

}  // namespace net
}  // namespace bccl
