#include "core/fdpass.h"

#include <cerrno>
#include <chrono>
#include <cstring>
#include <poll.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <thread>
#include <unistd.h>

#include "core/logger.h"

namespace bccl {
namespace {

constexpr uint32_t kFdMagic = 0xBCC1FD00u;

struct FdMsg {
    uint32_t magic;
    uint32_t tag;
    int32_t src;
};

socklen_t MakeAddr(const std::string& name, struct sockaddr_un* addr) {
    memset(addr, 0, sizeof(*addr));
    addr->sun_family = AF_UNIX;
    // Abstract namespace: leading NUL, no file to clean up.
    size_t n = std::min(name.size(), sizeof(addr->sun_path) - 2);
    memcpy(addr->sun_path + 1, name.data(), n);
    return static_cast<socklen_t>(offsetof(struct sockaddr_un, sun_path) + 1 + n);
}

}  // namespace

std::string FdPasser::Name(int rank) const { return "bccl." + ns_ + "." + std::to_string(rank); }

bool FdPasser::Listen(const std::string& ns, int rank) {
    ns_ = ns;
    rank_ = rank;
    listen_fd_ = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (listen_fd_ < 0) {
        LOG_ERROR("fdpass: socket failed: %s", strerror(errno));
        return false;
    }
    struct sockaddr_un addr;
    socklen_t len = MakeAddr(Name(rank), &addr);
    if (bind(listen_fd_, reinterpret_cast<struct sockaddr*>(&addr), len) != 0 || listen(listen_fd_, 256) != 0) {
        LOG_ERROR("fdpass: bind %s failed: %s", Name(rank).c_str(), strerror(errno));
        close(listen_fd_);
        listen_fd_ = -1;
        return false;
    }
    return true;
}

bool FdPasser::SendFd(int peer, uint32_t tag, int fd, int timeout_ms) {
    struct sockaddr_un addr;
    socklen_t len = MakeAddr(Name(peer), &addr);
    auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
    int s = -1;
    for (;;) {
        s = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
        if (s < 0) return false;
        if (connect(s, reinterpret_cast<struct sockaddr*>(&addr), len) == 0) break;
        close(s);
        s = -1;
        if (std::chrono::steady_clock::now() > deadline) {
            LOG_ERROR("fdpass: rank %d cannot reach rank %d", rank_, peer);
            return false;
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(5));
    }
    FdMsg msg{kFdMagic, tag, rank_};
    struct iovec iov = {&msg, sizeof(msg)};
    char ctrl[CMSG_SPACE(sizeof(int))];
    memset(ctrl, 0, sizeof(ctrl));
    struct msghdr mh;
    memset(&mh, 0, sizeof(mh));
    mh.msg_iov = &iov;
    mh.msg_iovlen = 1;
    mh.msg_control = ctrl;
    mh.msg_controllen = sizeof(ctrl);
    struct cmsghdr* cm = CMSG_FIRSTHDR(&mh);
    cm->cmsg_level = SOL_SOCKET;
    cm->cmsg_type = SCM_RIGHTS;
    cm->cmsg_len = CMSG_LEN(sizeof(int));
    memcpy(CMSG_DATA(cm), &fd, sizeof(int));
    ssize_t n = sendmsg(s, &mh, MSG_NOSIGNAL);
    close(s);
    if (n != static_cast<ssize_t>(sizeof(msg))) {
        LOG_ERROR("fdpass: sendmsg to rank %d failed: %s", peer, strerror(errno));
        return false;
    }
    return true;
}

bool FdPasser::RecvFd(int src, uint32_t tag, int* fd, int timeout_ms) {
    auto key = std::make_pair(tag, src);
    auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
    for (;;) {
        auto it = stash_.find(key);
        if (it != stash_.end()) {
            *fd = it->second;
            stash_.erase(it);
            return true;
        }
        int left = static_cast<int>(
            std::chrono::duration_cast<std::chrono::milliseconds>(deadline - std::chrono::steady_clock::now()).count());
        if (left <= 0) {
            LOG_ERROR("fdpass: rank %d timed out waiting for fd tag %u from rank %d", rank_, tag, src);
            return false;
        }
        struct pollfd p = {listen_fd_, POLLIN, 0};
        if (poll(&p, 1, left) <= 0) continue;
        int s = accept4(listen_fd_, nullptr, nullptr, SOCK_CLOEXEC);
        if (s < 0) continue;
        struct pollfd ps = {s, POLLIN, 0};
        if (poll(&ps, 1, left) <= 0) {
            close(s);
            continue;
        }
        FdMsg msg{};
        struct iovec iov = {&msg, sizeof(msg)};
        char ctrl[CMSG_SPACE(sizeof(int))];
        struct msghdr mh;
        memset(&mh, 0, sizeof(mh));
        mh.msg_iov = &iov;
        mh.msg_iovlen = 1;
        mh.msg_control = ctrl;
        mh.msg_controllen = sizeof(ctrl);
        ssize_t n = recvmsg(s, &mh, MSG_CMSG_CLOEXEC);
        close(s);
        struct cmsghdr* cm = CMSG_FIRSTHDR(&mh);
        if (n != static_cast<ssize_t>(sizeof(msg)) || msg.magic != kFdMagic || cm == nullptr ||
            cm->cmsg_type != SCM_RIGHTS) {
            LOG_WARN("fdpass: rank %d dropped a malformed message", rank_);
            continue;
        }
        int got = -1;
        memcpy(&got, CMSG_DATA(cm), sizeof(int));
        auto k = std::make_pair(msg.tag, static_cast<int>(msg.src));
        auto old = stash_.find(k);
        if (old != stash_.end()) close(old->second);
        stash_[k] = got;
    }
}

void FdPasser::Close() {
    for (auto& kv : stash_) close(kv.second);
    stash_.clear();
    if (listen_fd_ >= 0) {
        close(listen_fd_);
        listen_fd_ = -1;
    }
}

}  // namespace bccl
