// Chunk schedule of the native device Send/Recv, shared by the kernel (p2p_native.cu), the host
// side that builds its launch (DeviceEngine::RunNativeP2p) and the CPU checks of the schedule
// (bcclP2pPlan in the C API).
//
// The operations of one directed pair (sender -> receiver) in one group form a FIFO sequence;
// each is cut into chunks of kP2pChunkBytes, numbered across the sequence, and chunk g travels
// on channel g % nch. nch depends only on the pair's total bytes, so sender and receiver, each
// looking at its own side of the matched operations, derive the same channels and the same
// message order per channel without exchanging anything. The reference keeps one FIFO per
// directed pair too (sends and receives of a pair are matched in issue order, one TrySend /
// TryRecv per task on the pair's transport: OriginCCL src/topology/topology_p2p.cpp:50-58).
#pragma once

#include <stdint.h>

#include "device/dev_types.h"

#if defined(__CUDACC__)
#define BCCL_HD __host__ __device__
#else
#define BCCL_HD
#endif

namespace bccl {

// One Send (buf = its source) or Recv (buf = its destination) of a native P2P launch.
struct P2pNativeOp {
    char* buf;
    unsigned long long bytes;
};

// The work of one CTA: one channel of one directed pair.
struct P2pNativeRole {
    short peer;
    short dir;       // 0 send to peer, 1 receive from peer
    short channel;
    short nch;       // channels of this pair
    int op_begin;    // the pair's operations: ops[op_begin, op_end) in FIFO order
    int op_end;
};

constexpr int kP2pMaxRoles = 2 * (kMaxRanks - 1) * kP2pMaxChannels;
constexpr int kP2pMaxOps = 1536;

BCCL_HD inline int P2pChannels(unsigned long long pair_bytes) {
    const unsigned long long n = (pair_bytes + kP2pBytesPerChannel - 1) / kP2pBytesPerChannel;
    return n < 1 ? 1 : (n > static_cast<unsigned long long>(kP2pMaxChannels) ? kP2pMaxChannels : static_cast<int>(n));
}

BCCL_HD inline unsigned long long P2pChunks(unsigned long long bytes) {
    return (bytes + kP2pChunkBytes - 1) / kP2pChunkBytes;
}

// Byte offset, inside a receiver's P2P region, of the inbox slot of (source rank, channel, slot).
BCCL_HD constexpr unsigned long long P2pSlotOffset(int src, int channel, int slot) {
    return ((static_cast<unsigned long long>(src) * kP2pMaxChannels + channel) * kP2pSlots + slot) * kP2pChunkBytes;
}
static_assert(P2pSlotOffset(kMaxRanks - 1, kP2pMaxChannels - 1, kP2pSlots - 1) + kP2pChunkBytes == kP2pRegionBytes,
              "the last inbox slot ends at the end of the P2P region");

// Walks the chunks that one channel carries, in message order.
struct P2pCursor {
    int op;                  // current operation
    int nch, ch;
    unsigned long long g0;   // pair-wide number of the current operation's first chunk
    unsigned long long k;    // next chunk of the current operation (~0: not positioned yet)

    BCCL_HD P2pCursor(int op_begin, int nch_, int ch_) : op(op_begin), nch(nch_), ch(ch_), g0(0), k(~0ull) {}

    // The next chunk: operation index, byte offset in it and length. False when done.
    BCCL_HD bool next(const P2pNativeOp* ops, int op_end, int* i, unsigned long long* off, unsigned long long* len) {
        while (op < op_end) {
            const unsigned long long nck = P2pChunks(ops[op].bytes);
            if (k == ~0ull) {
                const unsigned long long first = g0 % static_cast<unsigned long long>(nch);
                k = (static_cast<unsigned long long>(ch) + nch - first) % static_cast<unsigned long long>(nch);
            }
            if (k < nck) {
                *i = op;
                *off = k * kP2pChunkBytes;
                const unsigned long long rest = ops[op].bytes - *off;
                *len = rest < kP2pChunkBytes ? rest : kP2pChunkBytes;
                k += static_cast<unsigned long long>(nch);
                return true;
            }
            g0 += nck;
            ++op;
            k = ~0ull;
        }
        return false;
    }
};

}  // namespace bccl
