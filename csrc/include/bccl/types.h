// Public data model of the library.
//
// Parity with the reference's data model (OriginCCL include/types.h:16-78): the enums
// DataType / ReduceOp / CollFunc, UniqueId, CommConfig (including the injectable
// get_hostname used to emulate several machines on one host), NodeInfo and CollTask keep
// the reference's names and meaning so that a user of the reference finds the same
// vocabulary. Added for the GPU:
//   * DataType::BF16 and DataType::FP16 (reduced in fp32, rounded once at the end);
//   * CommConfig::device selects a CUDA device (-1 keeps the reference's host-memory
//     communicator), CommConfig::stream an optional cudaStream_t;
//   * CollTask::scale, a fused epilogue multiplier (data-parallel gradient scaling).
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace bccl {

enum class DataType : int {
    FLOAT32 = 0,
    FLOAT64 = 1,
    INT32 = 2,
    INT64 = 3,
    BF16 = 4,
    FP16 = 5,
};

enum class ReduceOp : int {
    SUM = 0,
    MAX = 1,
    MIN = 2,
    AVG = 3,
};

enum class CollFunc : int {
    AllReduce = 0,
    Broadcast = 1,
    Reduce = 2,
    AllGather = 3,
    ReduceScatter = 4,
    Send = 5,
    Recv = 6,
};

// Algorithms a device collective can run with. kAuto lets the planner pick from the
// size -> algorithm table.
enum class Algo : int {
    kAuto = 0,
    kOneShot = 1,  // every rank pushes its whole payload to every peer; one sync
    kTwoShot = 2,  // reduce-scatter by push, all-gather by pull
    kNvls = 3,     // NVSwitch multicast: multimem.ld_reduce / multimem.st
    kRing = 4,     // neighbour-only pipeline (parity with the reference's ring)
    kHybrid = 5,   // AllReduce: part of the payload through the switch (NVLS), the rest two-shot
    kLL = 6,       // AllReduce / AllGather / ReduceScatter up to 2 MiB per rank: data and epoch flags in one store, no barrier
};

struct UniqueId {
    char ip_addr[64] = {};
    uint16_t port = 0;
};

std::string DefaultHostname();

struct CommConfig {
    int rank = 0;
    int world_size = 1;
    UniqueId unique_id;
    // Host communicator: worker threads per rank (0 -> 4). Device communicator: upper
    // bound on CTAs per collective (0 -> planner's choice).
    int n_channels = 0;
    std::string (*get_hostname)() = DefaultHostname;

    // ---- device (B200) extensions ----
    int device = -1;             // CUDA device ordinal; -1 = host-memory communicator
    void* stream = nullptr;      // cudaStream_t; nullptr = internal stream, calls block
    size_t buffer_bytes = 0;     // peer-mapped staging per rank (0 -> env / default)
    int timeout_ms = 0;          // bound on every device-side wait (0 -> env / default)
    bool enable_nvls = true;     // use NVSwitch multicast when the GPUs support it
    bool enable_nccl_p2p = true; // Send/Recv over NCCL point-to-point
};

struct NodeInfo {
    int rank = 0;
    std::string ip_addr;
    uint16_t data_port = 0;
    std::string hostname;
    uint64_t boot_id_hash = 0;  // distinguishes containers that share a hostname
    int device = -1;
    int pid = 0;
};

struct CollTask {
    CollFunc func = CollFunc::AllReduce;
    const void* send_buf = nullptr;
    void* recv_buf = nullptr;
    size_t count = 0;
    DataType dtype = DataType::FLOAT32;
    ReduceOp op = ReduceOp::SUM;
    int root = 0;
    int peer = -1;
    float scale = 1.0f;  // fused epilogue multiplier (floating types only)
    Algo algo = Algo::kAuto;
};

size_t DataTypeSize(DataType dtype);
const char* DataTypeName(DataType dtype);
const char* ReduceOpName(ReduceOp op);
const char* CollFuncName(CollFunc func);
const char* AlgoName(Algo algo);

inline bool IsCollective(CollFunc f) {
    return f == CollFunc::AllReduce || f == CollFunc::Broadcast || f == CollFunc::Reduce ||
           f == CollFunc::AllGather || f == CollFunc::ReduceScatter;
}
inline bool IsP2p(CollFunc f) { return f == CollFunc::Send || f == CollFunc::Recv; }
inline bool IsReducing(CollFunc f) {
    return f == CollFunc::AllReduce || f == CollFunc::Reduce || f == CollFunc::ReduceScatter;
}
inline bool IsFloating(DataType d) {
    return d == DataType::FLOAT32 || d == DataType::FLOAT64 || d == DataType::BF16 ||
           d == DataType::FP16;
}

}  // namespace bccl
