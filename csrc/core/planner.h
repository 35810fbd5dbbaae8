// Planner: validation, cross-rank-consistent ordering and algorithm choice.
//
// Parity with OriginCCL src/planner.cpp:
//   * ValidateCollectiveTask mirrors :68-110 (dtype/op/root, required buffers, size_t
//     overflow, count 0 succeeds with null buffers, Reduce's non-root recv may be null);
//   * SortTasks mirrors :112-163 (collectives first, stable by (func, bytes, dtype,
//     effective op, effective root); P2P after them ordered by round, then func);
//   * P2pRoundOf mirrors :50-54 (round i sends to (rank-i) and receives from (rank+i)).
// These rules have to be identical for every rank to build the same work list, so the
// ordering keys are the reference's. The reference's tree-vs-ring threshold and channel
// slicing become ChooseAlgo(): a per-(func, dtype, op, bytes, world) pick among the device
// kernels driven by a size -> algorithm table, and a CTA count that plays the role of
// the reference's channels.
#pragma once

#include <cstddef>
#include <string>
#include <vector>

#include "bccl/types.h"

namespace bccl {

struct AlgoChoice {
    Algo algo = Algo::kOneShot;
    int ctas = 1;
};

// One row of the size -> algorithm table: applies to ops of `func` on `world` ranks whose
// per-rank payload is <= max_bytes (rows are scanned in order; the first match wins).
struct TuningRow {
    CollFunc func;
    int world;  // 0 = any
    size_t max_bytes;
    Algo algo;
    int ctas;
};

class Planner {
public:
    Planner();

    bool ValidateCollectiveTask(const CollTask& task, int rank, int world_size) const;
    bool ValidateP2p(const CollTask& task, int rank, int world_size) const;
    bool SortTasks(std::vector<CollTask>& tasks, int rank, int world_size) const;
    bool IsCollectiveBatch(const std::vector<CollTask>& tasks) const;
    static int P2pRoundOf(CollFunc func, int rank, int peer, int world_size);

    // Device algorithm choice. nvls_ok says whether the multicast path exists and supports
    // (func, dtype, op); max_ctas bounds the CTA count (0 = no bound).
    AlgoChoice ChooseAlgo(CollFunc func, DataType dtype, ReduceOp op, size_t bytes, int world_size, bool nvls_ok,
                          int max_ctas, Algo forced) const;

    // Replaces the table (BCCL_TUNING_FILE format: "func world max_bytes algo ctas" per line).
    bool LoadTuningFile(const std::string& path);
    const std::vector<TuningRow>& table() const { return table_; }

    static Algo ParseAlgo(const std::string& s);

private:
    std::vector<TuningRow> table_;
    long env_max_ctas_ = 0;  // BCCL_MAX_CTAS, read at construction
};

}  // namespace bccl
