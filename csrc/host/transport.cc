#include "host/transport.h"

#include <cerrno>
#include <cstring>
#include <sys/socket.h>
#include <unistd.h>

#include "core/logger.h"
#include "core/net.h"

namespace bccl {

TcpTransport::TcpTransport(int fd) : fd_(fd) { net::SetNonBlocking(fd_, true); }

void TcpTransport::Close() { net::CloseFd(&fd_); }

bool TcpTransport::TrySend(const void* data, size_t size, size_t* progress, bool* done) {
    const char* p = static_cast<const char*>(data);
    while (*progress < size) {
        ssize_t n = send(fd_, p + *progress, size - *progress, MSG_NOSIGNAL | MSG_DONTWAIT);
        if (n > 0) {
            *progress += static_cast<size_t>(n);
            continue;
        }
        if (n < 0 && errno == EINTR) continue;
        if (n < 0 && (errno == EAGAIN || errno == EWOULDBLOCK)) break;
        LOG_ERROR("tcp send failed: %s", n == 0 ? "closed" : strerror(errno));
        return false;
    }
    *done = *progress == size;
    return true;
}

bool TcpTransport::TryRecv(void* data, size_t size, size_t* progress, bool* done) {
    char* p = static_cast<char*>(data);
    while (*progress < size) {
        ssize_t n = recv(fd_, p + *progress, size - *progress, MSG_DONTWAIT);
        if (n > 0) {
            *progress += static_cast<size_t>(n);
            continue;
        }
        if (n == 0) {
            LOG_ERROR("tcp peer closed the connection");
            return false;
        }
        if (errno == EINTR) continue;
        if (errno == EAGAIN || errno == EWOULDBLOCK) break;
        LOG_ERROR("tcp recv failed: %s", strerror(errno));
        return false;
    }
    *done = *progress == size;
    return true;
}

bool ShmRingTransport::TrySend(const void* data, size_t size, size_t* progress, bool* done) {
    if (!producer_) {
        LOG_ERROR("shm ring: TrySend on the consumer endpoint");
        return false;
    }
    const char* src = static_cast<const char*>(data);
    uint64_t head = ctrl_->head.load(std::memory_order_relaxed);
    const uint64_t tail = ctrl_->tail.load(std::memory_order_acquire);
    size_t space = cap_ - static_cast<size_t>(head - tail);
    size_t todo = std::min(space, size - *progress);
    while (todo > 0) {
        size_t pos = static_cast<size_t>(head % cap_);
        size_t n = std::min(todo, cap_ - pos);
        memcpy(data_ + pos, src + *progress, n);
        head += n;
        *progress += n;
        todo -= n;
    }
    ctrl_->head.store(head, std::memory_order_release);
    *done = *progress == size;
    return true;
}

bool ShmRingTransport::TryRecv(void* data, size_t size, size_t* progress, bool* done) {
    if (producer_) {
        LOG_ERROR("shm ring: TryRecv on the producer endpoint");
        return false;
    }
    char* dst = static_cast<char*>(data);
    uint64_t tail = ctrl_->tail.load(std::memory_order_relaxed);
    const uint64_t head = ctrl_->head.load(std::memory_order_acquire);
    size_t avail = static_cast<size_t>(head - tail);
    size_t todo = std::min(avail, size - *progress);
    while (todo > 0) {
        size_t pos = static_cast<size_t>(tail % cap_);
        size_t n = std::min(todo, cap_ - pos);
        memcpy(dst + *progress, data_ + pos, n);
        tail += n;
        *progress += n;
        todo -= n;
    }
    ctrl_->tail.store(tail, std::memory_order_release);
    *done = *progress == size;
    return true;
}

}  // namespace bccl
