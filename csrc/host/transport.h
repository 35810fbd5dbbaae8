// Host byte movers with a non-blocking data-plane contract.
//
// Parity: the reference's Transport interface (OriginCCL include/transport/transport.h:19-56):
// TrySend/TryRecv(data, size, *progress, *done) move as many bytes as possible without
// blocking, progress is monotone in [0, size] and done <=> progress == size; GetFd()
// exposes a readiness fd for event-driven waiting (-1 when the transport must be polled).
// Two movers exist: a TCP socket (across logical machines) and an SPSC byte ring in the
// machine's shared-memory segment (between processes of one machine).
#pragma once

#include <atomic>
#include <cstddef>
#include <cstdint>

namespace bccl {

class Transport {
public:
    virtual ~Transport() = default;
    virtual bool TrySend(const void* data, size_t size, size_t* progress, bool* done) = 0;
    virtual bool TryRecv(void* data, size_t size, size_t* progress, bool* done) = 0;
    virtual int GetFd() const { return -1; }
    virtual short GetPollEvents(bool sending) const { return sending ? 0x004 /*POLLOUT*/ : 0x001 /*POLLIN*/; }
    virtual void Close() {}
    virtual const char* Name() const = 0;
};

class TcpTransport : public Transport {
public:
    explicit TcpTransport(int fd);
    ~TcpTransport() override { Close(); }
    bool TrySend(const void* data, size_t size, size_t* progress, bool* done) override;
    bool TryRecv(void* data, size_t size, size_t* progress, bool* done) override;
    int GetFd() const override { return fd_; }
    void Close() override;
    const char* Name() const override { return "tcp"; }

private:
    int fd_;
};

// Shared-memory control block of one directed ring (lives inside the segment).
struct alignas(64) ShmRingCtrl {
    std::atomic<uint64_t> head;  // bytes produced
    char pad0[56];
    std::atomic<uint64_t> tail;  // bytes consumed
    char pad1[56];
};

class ShmRingTransport : public Transport {
public:
    // One endpoint of the ring; the producer only calls TrySend, the consumer only TryRecv.
    ShmRingTransport(ShmRingCtrl* ctrl, char* data, size_t capacity, bool producer)
        : ctrl_(ctrl), data_(data), cap_(capacity), producer_(producer) {}
    bool TrySend(const void* data, size_t size, size_t* progress, bool* done) override;
    bool TryRecv(void* data, size_t size, size_t* progress, bool* done) override;
    const char* Name() const override { return "shm"; }
    size_t capacity() const { return cap_; }

private:
    ShmRingCtrl* ctrl_;
    char* data_;
    size_t cap_;
    bool producer_;
};

}  // namespace bccl
