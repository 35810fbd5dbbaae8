#include "core/planner.h"

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <limits>
#include <sstream>

#include "core/env.h"
#include "core/logger.h"

namespace bccl {
namespace {

bool ValidDtype(DataType d) {
    int v = static_cast<int>(d);
    return v >= 0 && v <= static_cast<int>(DataType::FP16);
}
bool ValidOp(ReduceOp o) {
    int v = static_cast<int>(o);
    return v >= 0 && v <= static_cast<int>(ReduceOp::AVG);
}
int EffectiveOp(const CollTask& t) { return IsReducing(t.func) ? static_cast<int>(t.op) : 0; }
int EffectiveRoot(const CollTask& t) {
    return (t.func == CollFunc::Broadcast || t.func == CollFunc::Reduce) ? t.root : 0;
}

CollFunc ParseFunc(const std::string& s) {
    if (s == "allreduce") return CollFunc::AllReduce;
    if (s == "broadcast") return CollFunc::Broadcast;
    if (s == "reduce") return CollFunc::Reduce;
    if (s == "allgather") return CollFunc::AllGather;
    if (s == "reducescatter") return CollFunc::ReduceScatter;
    return CollFunc::Send;
}

// Built-in table. Per-rank payload bytes; measured on 8xB200 (NVLink 5 / NVSwitch).
// Small payloads are latency bound: one-shot push (one cross-rank sync). Large reducing
// payloads go to NVLS, which moves S*(1+1/N) bytes per direction instead of 2*S*(N-1)/N.
std::vector<TuningRow> DefaultTable() {
    return {
        // Two ranks (2 x B200): the switch reads the issuing GPU's own copy too, so NVLS moves
        // 1.5*S per direction against S for the peer-to-peer kernels (measured: NVLS and the
        // hybrid lose at every size). One-shot push up to 2 MiB, the pipelined push up to 6 MiB,
        // the ring (fine-grained neighbour flags) up to 48 MiB, two-shot above (64 MiB: two-shot
        // 160.6 us, ring 167.0 us).
        {CollFunc::AllReduce, 2, 2 << 20, Algo::kOneShot, 0},
        {CollFunc::AllReduce, 2, 6 << 20, Algo::kTwoShot, 0},
        {CollFunc::AllReduce, 2, 48 << 20, Algo::kRing, 0},
        {CollFunc::AllReduce, 2, ~size_t(0), Algo::kTwoShot, 0},
        // Four ranks (4 x B200, fp32, plain buffers): two-shot beats NVLS up to 16 MiB (93 vs
        // 102 us there); above, the hybrid (NVLS on part of the payload, two-shot on the rest)
        // wins (64 MiB: 243 us against NVLS 259 and two-shot 263; 256 MiB: 799 against 820 and 837).
        {CollFunc::AllReduce, 4, 1 << 20, Algo::kOneShot, 0},
        {CollFunc::AllReduce, 4, 16 << 20, Algo::kTwoShot, 0},
        {CollFunc::AllReduce, 4, ~size_t(0), Algo::kHybrid, 0},
        // Three or more ranks (8 x B200): one-shot up to 1 MiB, pipelined two-shot up to 8 MiB,
        // NVLS above.
        {CollFunc::AllReduce, 0, 1 << 20, Algo::kOneShot, 0},
        {CollFunc::AllReduce, 0, 8 << 20, Algo::kTwoShot, 0},
        {CollFunc::AllReduce, 0, ~size_t(0), Algo::kNvls, 0},
        {CollFunc::Broadcast, 2, ~size_t(0), Algo::kOneShot, 0},
        {CollFunc::Broadcast, 0, 512 << 10, Algo::kOneShot, 0},
        {CollFunc::Broadcast, 0, ~size_t(0), Algo::kNvls, 0},
        {CollFunc::Reduce, 2, ~size_t(0), Algo::kOneShot, 0},
        {CollFunc::Reduce, 0, 512 << 10, Algo::kOneShot, 0},
        {CollFunc::Reduce, 0, ~size_t(0), Algo::kNvls, 0},
        // AllGather through the switch: a rank's block leaves its GPU once (multimem.st) instead
        // of once per peer; ReduceScatter: the switch reduces, the SMs only stage and store.
        // Two ranks gain nothing (one peer either way).
        {CollFunc::AllGather, 2, ~size_t(0), Algo::kOneShot, 0},
        {CollFunc::AllGather, 0, 256 << 10, Algo::kOneShot, 0},
        {CollFunc::AllGather, 0, ~size_t(0), Algo::kNvls, 0},
        {CollFunc::ReduceScatter, 2, ~size_t(0), Algo::kOneShot, 0},
        {CollFunc::ReduceScatter, 0, 1 << 20, Algo::kOneShot, 0},
        {CollFunc::ReduceScatter, 0, ~size_t(0), Algo::kNvls, 0},
    };
}

// CTAs for a payload: enough memory-level parallelism to cover NVLink latency for large
// payloads, few CTAs for small ones (each CTA pays a cross-rank sync).
int DefaultCtas(Algo algo, size_t bytes) {
    if (algo == Algo::kNvls) {
        if (bytes <= (1u << 20)) return 8;
        if (bytes <= (8u << 20)) return 16;
        return 32;
    }
    if (bytes <= (16u << 10)) return 1;
    if (bytes <= (64u << 10)) return 2;
    if (bytes <= (256u << 10)) return 4;
    if (bytes <= (1u << 20)) return 8;
    if (bytes <= (4u << 20)) return 16;
    return 32;
}

}  // namespace

Planner::Planner() : table_(DefaultTable()), env_max_ctas_(EnvInt("BCCL_MAX_CTAS", 0)) {
    std::string path = EnvStr("BCCL_TUNING_FILE", "");
    if (!path.empty() && !LoadTuningFile(path)) {
        LOG_WARN("planner: could not load tuning file %s, keeping the built-in table", path.c_str());
    }
}

Algo Planner::ParseAlgo(const std::string& s) {
    if (s == "oneshot") return Algo::kOneShot;
    if (s == "twoshot") return Algo::kTwoShot;
    if (s == "nvls") return Algo::kNvls;
    if (s == "ring") return Algo::kRing;
    if (s == "hybrid") return Algo::kHybrid;
    if (s == "ll") return Algo::kLL;
    return Algo::kAuto;
}

bool Planner::LoadTuningFile(const std::string& path) {
    std::ifstream in(path);
    if (!in) return false;
    std::vector<TuningRow> rows;
    std::string line;
    while (std::getline(in, line)) {
        if (line.empty() || line[0] == '#') continue;
        std::istringstream ls(line);
        std::string func, algo;
        int world = 0, ctas = 0;
        unsigned long long max_bytes = 0;
        if (!(ls >> func >> world >> max_bytes >> algo >> ctas)) return false;
        CollFunc f = ParseFunc(func);
        Algo a = ParseAlgo(algo);
        if (f == CollFunc::Send || a == Algo::kAuto) return false;
        rows.push_back({f, world, static_cast<size_t>(max_bytes), a, ctas});
    }
    if (rows.empty()) return false;
    table_ = rows;
    return true;
}

bool Planner::ValidateCollectiveTask(const CollTask& task, int rank, int world_size) const {
    if (!IsCollective(task.func) || world_size <= 0 || rank < 0 || rank >= world_size) {
        LOG_ERROR("rank %d: rejected: not a collective, or rank outside a communicator of %d", rank, world_size);
        return false;
    }
    const size_t es = ValidDtype(task.dtype) ? DataTypeSize(task.dtype) : 0;
    if (es == 0 || task.count > std::numeric_limits<size_t>::max() / es) {
        LOG_ERROR("rank %d: rejected: unknown data type or element count too large for size_t bytes", rank);
        return false;
    }
    if (IsReducing(task.func) && !ValidOp(task.op)) {
        LOG_ERROR("rank %d: rejected: unknown reduction op %d", rank, static_cast<int>(task.op));
        return false;
    }
    const bool has_root = task.func == CollFunc::Broadcast || task.func == CollFunc::Reduce;
    if (has_root && (task.root < 0 || task.root >= world_size)) {
        LOG_ERROR("rank %d: rejected: root %d is not a rank of this communicator", rank, task.root);
        return false;
    }
    if ((task.func == CollFunc::AllGather || task.func == CollFunc::ReduceScatter) && task.count != 0 &&
        task.count > std::numeric_limits<size_t>::max() / static_cast<size_t>(world_size) / es) {
        LOG_ERROR("rank %d: rejected: count x %d ranks does not fit in size_t bytes", rank, world_size);
        return false;
    }
    if (task.count == 0) return true;
    const bool needs_send = task.func != CollFunc::Broadcast;
    const bool needs_recv = task.func != CollFunc::Reduce || rank == task.root;
    if ((needs_send && task.send_buf == nullptr) || (needs_recv && task.recv_buf == nullptr)) {
        LOG_ERROR("rank %d: rejected: null send or receive pointer for a non-empty collective", rank);
        return false;
    }
    return true;
}

bool Planner::ValidateP2p(const CollTask& task, int rank, int world_size) const {
    if (!IsP2p(task.func) || task.peer < 0 || task.peer >= world_size || task.peer == rank) {
        LOG_ERROR("rank %d: rejected: peer %d is this rank or outside the communicator", rank, task.peer);
        return false;
    }
    const size_t es = ValidDtype(task.dtype) ? DataTypeSize(task.dtype) : 0;
    if (es == 0 || task.count > std::numeric_limits<size_t>::max() / es) {
        LOG_ERROR("rank %d: rejected: unknown data type or element count too large for a Send/Recv", rank);
        return false;
    }
    if (task.count != 0 && task.send_buf == nullptr && task.recv_buf == nullptr) {
        LOG_ERROR("rank %d: rejected: null buffer for a non-empty Send/Recv", rank);
        return false;
    }
    return true;
}

int Planner::P2pRoundOf(CollFunc func, int rank, int peer, int world_size) {
    const int forward = (func == CollFunc::Send) ? (peer - rank + world_size) % world_size
                                                 : (rank - peer + world_size) % world_size;
    return world_size - forward;
}

bool Planner::SortTasks(std::vector<CollTask>& tasks, int rank, int world_size) const {
    if (world_size <= 0 || rank < 0 || rank >= world_size) {
        LOG_ERROR("rank %d: cannot order a group for a communicator of %d ranks", rank, world_size);
        return false;
    }
    std::vector<CollTask> colls, p2p;
    for (const CollTask& t : tasks) {
        if (IsP2p(t.func)) {
            if (!ValidateP2p(t, rank, world_size)) return false;
            p2p.push_back(t);
        } else {
            if (!ValidateCollectiveTask(t, rank, world_size)) return false;
            colls.push_back(t);
        }
    }
    std::stable_sort(colls.begin(), colls.end(), [](const CollTask& a, const CollTask& b) {
        if (a.func != b.func) return a.func < b.func;
        const size_t ab = a.count * DataTypeSize(a.dtype), bb = b.count * DataTypeSize(b.dtype);
        if (ab != bb) return ab < bb;
        if (a.dtype != b.dtype) return a.dtype < b.dtype;
        if (EffectiveOp(a) != EffectiveOp(b)) return EffectiveOp(a) < EffectiveOp(b);
        return EffectiveRoot(a) < EffectiveRoot(b);
    });
    std::stable_sort(p2p.begin(), p2p.end(), [rank, world_size](const CollTask& a, const CollTask& b) {
        int ra = P2pRoundOf(a.func, rank, a.peer, world_size), rb = P2pRoundOf(b.func, rank, b.peer, world_size);
        if (ra != rb) return ra < rb;
        return a.func < b.func;
    });
    tasks.clear();
    tasks.insert(tasks.end(), colls.begin(), colls.end());
    tasks.insert(tasks.end(), p2p.begin(), p2p.end());
    return true;
}

bool Planner::IsCollectiveBatch(const std::vector<CollTask>& tasks) const {
    for (const CollTask& t : tasks)
        if (IsP2p(t.func)) return false;
    return true;
}

AlgoChoice Planner::ChooseAlgo(CollFunc func, DataType dtype, ReduceOp op, size_t bytes, int world_size,
                               bool nvls_ok, int max_ctas, Algo forced) const {
    (void)dtype;
    (void)op;
    AlgoChoice c;
    Algo algo = forced;
    int ctas = 0;
    if (algo == Algo::kAuto) {
        algo = Algo::kOneShot;
        for (const TuningRow& row : table_) {
            if (row.func != func || (row.world != 0 && row.world != world_size) || bytes > row.max_bytes) continue;
            algo = row.algo;
            ctas = row.ctas;
            break;
        }
    }
    // Two-shot and ring exist for AllReduce only; the other collectives are already
    // bandwidth-optimal as one-shot pushes.
    if ((algo == Algo::kTwoShot || algo == Algo::kRing) && func != CollFunc::AllReduce) algo = Algo::kOneShot;
    if (algo == Algo::kHybrid && func != CollFunc::AllReduce) algo = Algo::kNvls;
    if (algo == Algo::kLL && (func == CollFunc::Broadcast || func == CollFunc::Reduce || bytes > (2u << 20))) {
        algo = Algo::kOneShot;
    }
    if (algo == Algo::kHybrid && !nvls_ok) algo = Algo::kTwoShot;
    if (algo == Algo::kNvls && !nvls_ok) algo = (func == CollFunc::AllReduce && bytes > (256u << 10))
                                                    ? Algo::kTwoShot : Algo::kOneShot;
    if (ctas <= 0) ctas = DefaultCtas(algo, bytes);
    if (env_max_ctas_ > 0) ctas = std::min<int>(ctas, static_cast<int>(env_max_ctas_));
    if (max_ctas > 0) ctas = std::min(ctas, max_ctas);
    c.algo = algo;
    c.ctas = std::max(1, ctas);
    return c;
}

}  // namespace bccl
