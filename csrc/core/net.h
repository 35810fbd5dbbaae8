// Socket and host helpers used by the bootstrap, the host TCP transport and the fd passer.
//
// Parity: the reference's Utils socket helpers (OriginCCL src/utils.cpp:16-261): local IP
// and hostname discovery, listen/connect/accept and length-prefixed framing. Every blocking
// call here takes a timeout so that a missing peer ends in an error, not a hang.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace bccl {
namespace net {

std::string LocalIpAddress();   // BCCL_BOOTSTRAP_ADDR, else first up non-loopback IPv4, else 127.0.0.1
std::string Hostname();

// Binds 0.0.0.0:port (0 = ephemeral). Returns the fd and writes the bound port.
int Listen(uint16_t port, uint16_t* bound_port, int backlog = 128);
// Connects with retries every retry_ms until timeout_ms has passed. Returns fd or -1.
int Connect(const std::string& ip, uint16_t port, int timeout_ms, int retry_ms = 100);
// Waits up to timeout_ms (<0: forever) for a connection. Returns fd or -1.
int Accept(int listen_fd, int timeout_ms);

bool SendAll(int fd, const void* buf, size_t len, int timeout_ms);
bool RecvAll(int fd, void* buf, size_t len, int timeout_ms);
// Frame = u64 length + payload.
bool SendFrame(int fd, const std::vector<uint8_t>& payload, int timeout_ms);
bool RecvFrame(int fd, std::vector<uint8_t>* payload, int timeout_ms, size_t max_len = (1ull << 30));

bool SetNonBlocking(int fd, bool on);
void SetNoDelay(int fd);
void CloseFd(int* fd);

// Byte-buffer codec used for NodeInfo and control messages.
class Writer {
public:
    void U8(uint8_t v) { buf_.push_back(v); }
    void U16(uint16_t v) { Raw(&v, sizeof(v)); }
    void U32(uint32_t v) { Raw(&v, sizeof(v)); }
    void U64(uint64_t v) { Raw(&v, sizeof(v)); }
    void I32(int32_t v) { Raw(&v, sizeof(v)); }
    void Str(const std::string& s) {
        U32(static_cast<uint32_t>(s.size()));
        Raw(s.data(), s.size());
    }
    void Raw(const void* p, size_t n) {
        const uint8_t* b = static_cast<const uint8_t*>(p);
        buf_.insert(buf_.end(), b, b + n);
    }
    std::vector<uint8_t>& bytes() { return buf_; }

private:
    std::vector<uint8_t> buf_;
};

class Reader {
public:
    Reader(const uint8_t* p, size_t n) : p_(p), n_(n) {}
    explicit Reader(const std::vector<uint8_t>& v) : p_(v.data()), n_(v.size()) {}
    bool U8(uint8_t* v) { return Raw(v, sizeof(*v)); }
    bool U16(uint16_t* v) { return Raw(v, sizeof(*v)); }
    bool U32(uint32_t* v) { return Raw(v, sizeof(*v)); }
    bool U64(uint64_t* v) { return Raw(v, sizeof(*v)); }
    bool I32(int32_t* v) { return Raw(v, sizeof(*v)); }
    bool Str(std::string* s) {
        uint32_t n = 0;
        if (!U32(&n) || n > n_ - off_) return false;
        s->assign(reinterpret_cast<const char*>(p_ + off_), n);
        off_ += n;
        return true;
    }
    bool Raw(void* dst, size_t n) {
        if (n > n_ - off_) return false;
        for (size_t i = 0; i < n; ++i) static_cast<uint8_t*>(dst)[i] = p_[off_ + i];
        off_ += n;
        return true;
    }
    bool Done() const { return off_ == n_; }

private:
    const uint8_t* p_;
    size_t n_;
    size_t off_ = 0;
};

}  // namespace net
}  // namespace bccl
