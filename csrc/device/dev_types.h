// Structures shared by host code and the sm_100a kernels.
//
// Memory model of a device communicator (one process per GPU, all GPUs behind one
// NVSwitch). Every rank owns:
//   * a unicast "UC" buffer, created with cuMemCreate, exported as a POSIX fd and mapped by
//     every peer, so kernels address any peer's UC buffer with plain ld/st over NVLink. It
//     holds the control region (cross-rank flags) followed by the data region used as
//     per-source inboxes by the push kernels;
//   * optionally an NVLS buffer bound to an NVSwitch multicast object: one virtual
//     address (mc) whose multimem.ld_reduce reads and reduces all ranks' copies inside the
//     switch and whose multimem.st writes every rank's copy;
//   * a local DevState (sequence counters) and a host-mapped ErrorRecord.
// Sequence counters live on the device so a kernel captured in a CUDA graph stays
// correct on replay: each launch reads the counters left by the previous launch.
#pragma once

#include <cstddef>
#include <cstdint>

namespace bccl {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 256;
constexpr size_t kCtrlBytes = 1u << 20;          // control region at the start of each UC buffer
constexpr size_t kBarrierFlagsOff = 0;            // u64 [kMaxCtas][kMaxRanks]
constexpr size_t kBarrierFlagsBytes = sizeof(uint64_t) * kMaxCtas * kMaxRanks;
constexpr size_t kRingPostedOff = 16u << 10;     // u64 [kMaxCtas]: messages the ring predecessor posted here
constexpr size_t kRingConsumedOff = 32u << 10;   // u64 [kMaxCtas]: messages the ring successor consumed
constexpr size_t kTpFlagsOff = 64u << 10;         // u64 flags of the fused tensor-parallel kernels
constexpr size_t kTpFlagsBytes = 256u << 10;
constexpr size_t kAlign = 256;

// Native device Send/Recv (p2p_native.cu). Every directed pair (src -> dst) has kP2pMaxChannels
// channels; a channel is one CTA on each side with kP2pSlots inbox slots of kP2pChunkBytes in
// the receiver's P2P region, which follows the data region of the UC buffer.
constexpr int kP2pMaxChannels = 8;
constexpr int kP2pSlots = 4;
constexpr size_t kP2pChunkBytes = 64u << 10;
constexpr size_t kP2pBytesPerChannel = 256u << 10;  // one more channel per this many bytes of a pair
constexpr size_t kP2pRegionBytes = static_cast<size_t>(kMaxRanks) * kP2pMaxChannels * kP2pSlots * kP2pChunkBytes;
constexpr size_t kP2pPostedOff = 512u << 10;    // u64 [src][channel]: messages src posted into this rank's inbox
constexpr size_t kP2pConsumedOff = 520u << 10;  // u64 [dst][channel]: messages dst consumed from this rank
static_assert(kTpFlagsOff + kTpFlagsBytes <= kP2pPostedOff, "control region overlap");

// Low-latency AllReduce (ll.cu): 16-byte lines carrying 8 payload bytes and two epoch words,
// [parity 2][source kMaxRanks][kLLMaxLines] per rank, after the native Send/Recv region.
constexpr size_t kLLMaxLines = 262144;  // 2 MiB of payload per rank and launch (64 MiB of lines per rank)
constexpr size_t kLLRegionBytes = 2ull * kMaxRanks * kLLMaxLines * 16;
static_assert(kP2pConsumedOff + sizeof(uint64_t) * kMaxRanks * kP2pMaxChannels <= kCtrlBytes, "control region size");

// Error codes written by kernels (host-mapped, read after the stream synchronises).
enum DevError : int {
    kDevOk = 0,
    kDevTimeout = 1,   // a bounded wait on a peer flag expired
    kDevAborted = 2,   // the host raised the abort word
    kDevBadArgs = 3,   // a kernel rejected its arguments (bounds/alignment)
};

struct ErrorRecord {
    int code;
    int rank;
    int cta;
    int peer;
    int phase;
    int pad;
    unsigned long long seq;
    unsigned long long waited_ns;
};

struct DevState {
    unsigned long long round_seq;    // data-buffer half parity for the UC inboxes
    unsigned long long barrier_seq;  // last barrier value used by every CTA slot
    unsigned long long nvls_round_seq;
    unsigned int done_ctas;          // CTAs finished in the current launch
    unsigned int pad;
    unsigned long long tp_seq;       // fused tensor-parallel kernels: launches so far
    unsigned int tp_done;
    unsigned int pad2;
    unsigned long long ring_seq;     // ring kernel: message numbers used so far (per CTA slot)
    unsigned long long ll_seq;       // low-latency AllReduce: launches so far (its line epoch)
    // Native Send/Recv: messages this rank sent to / received from each peer, per channel.
    unsigned long long p2p_sent[kMaxRanks][kP2pMaxChannels];
    unsigned long long p2p_recvd[kMaxRanks][kP2pMaxChannels];
};

// One device trace record (written when tracing is on): who did what, when.
struct TraceRecord {
    unsigned long long t_ns;  // %globaltimer
    unsigned int cta;
    unsigned short group;     // warp group (0 = whole CTA)
    unsigned short event;     // TraceEvent
    unsigned int round;
    unsigned int kernel;      // launch serial
};

enum TraceEvent : unsigned short {
    kTrBegin = 1,     // kernel start
    kTrStaged = 2,    // a CTA issued its phases of a pipeline iteration (before the barrier)
    kTrReadyWait = 3, // G2: ready flags observed
    kTrReduced = 4,   // G2: reduce done, flag sent
    kTrDoneWait = 5,  // G3: reduced flags observed
    kTrFinished = 6,  // G3: round copied out
    kTrBarrier = 7,   // push engine: barrier passed
    kTrEnd = 8,       // kernel end
    kTrSlotWait = 9,  // G1: slot became free
};

struct DevComm {
    int rank;
    int nranks;
    char* uc[kMaxRanks];        // every rank's UC buffer, mapped here
    char* nvls_uc;              // this rank's NVLS buffer (unicast view), or null
    char* nvls_mc;              // multicast view of the NVLS buffers, or null
    DevState* state;
    ErrorRecord* err;           // host-mapped
    const volatile int* abort;  // host-mapped, set by the host to stop waits
    unsigned long long timeout_ns;
    unsigned long long data_bytes;  // bytes of the UC data region
    unsigned long long nvls_bytes;  // bytes of the NVLS buffer
    TraceRecord* trace;             // null unless tracing is on
    unsigned int* trace_count;
    unsigned int trace_cap;
    unsigned int kernel_serial;     // host launch counter (trace labels only)
    int spin_wait;                  // 1: flag waits poll without __nanosleep (BCCL_SPIN_WAIT)
    unsigned long long ll_off;      // byte offset of the low-latency line buffers in every UC buffer (0: none)
};

// One collective in a push-engine launch. All byte offsets refer to the per-peer stream:
// the concatenation of every item's per-peer payload, each padded to 16 bytes.
struct WorkItem {
    const void* src;
    void* dst;
    unsigned long long count;       // elements of the per-peer payload
    unsigned long long stream_off;  // byte offset of this payload in the per-peer stream
    unsigned char func;             // CollFunc
    unsigned char dtype;            // DataType
    unsigned char op;               // ReduceOp
    unsigned char root;
    float scale;
};

}  // namespace bccl
