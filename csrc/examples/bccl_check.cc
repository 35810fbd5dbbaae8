// bccl_check: a C++ program on the public bccl::Communicator API — the collective and P2P
// check matrix and the AllReduce benchmark, run under bccl_run.
//
//   bccl_run -np 4 bccl_check check                 # host memory (shared memory / TCP)
//   bccl_run -np 2 --gpus bccl_check check --device # GPU buffers (one GPU per rank)
//   bccl_run -np 4 bccl_check bench --counts 32768,131072 --warmup 20 --iters 100
//   bccl_run -np 4 bccl_check bench-group --messages 64 --message-bytes 262144
//   bccl_run -np 32 bccl_check check --ranks-per-machine 8   # four logical machines
//   bccl_run -np 4 bccl_check fuzz --seed 3 --ops 60          # random checked sequence
//
// check: every collective with exact-valued inputs (integers, and floats that are multiples of
// 1/8), out of place and in place, a sentinel element after every output, nested groups,
// Send/Recv around the ring and the contract cases (count 0 with null buffers, bad root,
// null buffer). Rank 0 prints one JSON line: {"passed": P, "failed": F, ...}; exit status is
// non-zero on any failure.
// bench: int32 SUM AllReduce with rank r's element i = (r*7 + i) mod 1000 (checked), timed on
// the host clock between barriers; the time per call is the max over ranks (an AllReduce of
// the per-rank times with MAX), busbw = algbw * 2(N-1)/N. One JSON line per count.
//
// --ranks-per-machine K injects the hostname "logical-machine-<rank / K>" through
// CommConfig::get_hostname, as OriginCCL tests/regression/test_multi_machine.cpp:14-20 does, so
// one host runs the shared-memory, leader-exchange and TCP paths of several machines.
//
// Parity: OriginCCL tests/test_common.cpp (case generator, oracle, sentinel, contract cases)
// and tests/benchmark/test_allreduce_benchmark.cpp:341-421 (timing as max over ranks).
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <random>
#include <sstream>
#include <string>
#include <thread>
#include <vector>

#include <cuda_runtime.h>

#include "bccl/communicator.h"

using bccl::Communicator;
using bccl::DataType;
using bccl::ReduceOp;

namespace {

int EnvInt(const char* name, int dflt) {
    const char* v = std::getenv(name);
    return v ? std::atoi(v) : dflt;
}

bool ExchangeId(int rank, bccl::UniqueId* id, Communicator* comm) {
    if (const char* m = std::getenv("BCCL_MASTER")) {  // multi-node launch: the id is known
        if (rank == 0) return comm->GetUniqueId(*id);
        std::string s(m);
        size_t colon = s.rfind(':');
        if (colon == std::string::npos) return false;
        std::snprintf(id->ip_addr, sizeof(id->ip_addr), "%s", s.substr(0, colon).c_str());
        id->port = static_cast<uint16_t>(std::atoi(s.substr(colon + 1).c_str()));
        return true;
    }
    const char* path = std::getenv("BCCL_ID_FILE");
    if (path == nullptr) {
        std::fprintf(stderr, "BCCL_ID_FILE is not set (run under bccl_run)\n");
        return false;
    }
    if (rank == 0) {
        if (!comm->GetUniqueId(*id)) return false;
        std::string tmp = std::string(path) + ".tmp";
        {
            std::ofstream f(tmp);
            f << id->ip_addr << ":" << id->port;
        }
        return std::rename(tmp.c_str(), path) == 0;
    }
    auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(60);
    while (access(path, R_OK) != 0) {
        if (std::chrono::steady_clock::now() > deadline) return false;
        std::this_thread::sleep_for(std::chrono::milliseconds(5));
    }
    std::ifstream f(path);
    std::string s;
    f >> s;
    size_t colon = s.rfind(':');
    if (colon == std::string::npos) return false;
    std::snprintf(id->ip_addr, sizeof(id->ip_addr), "%s", s.substr(0, colon).c_str());
    id->port = static_cast<uint16_t>(std::atoi(s.substr(colon + 1).c_str()));
    return true;
}

// Buffers live on the host or on the GPU; values are staged through host vectors.
struct Mem {
    bool device = false;
    void* Alloc(size_t bytes) {
        void* p = nullptr;
        if (device) {
            if (cudaMalloc(&p, std::max<size_t>(bytes, 16)) != cudaSuccess) return nullptr;
        } else {
            p = std::malloc(std::max<size_t>(bytes, 16));
        }
        return p;
    }
    void Free(void* p) {
        if (device) cudaFree(p); else std::free(p);
    }
    void Put(void* dst, const void* src, size_t bytes) {
        if (device) cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice); else std::memcpy(dst, src, bytes);
    }
    void Get(void* dst, const void* src, size_t bytes) {
        if (device) cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost); else std::memcpy(dst, src, bytes);
    }
};

template <typename T>
T Value(int rank, size_t i) {
    long v = static_cast<long>((rank * 7 + i * 13) % 97) - 48;  // small integers
    if (std::is_floating_point<T>::value) return static_cast<T>(v / 8.0);
    return static_cast<T>(v);
}

template <typename T>
T Reduce(ReduceOp op, const std::vector<T>& xs, int n) {
    double acc = xs[0];
    for (size_t r = 1; r < xs.size(); ++r) {
        if (op == ReduceOp::MAX) acc = std::max<double>(acc, xs[r]);
        else if (op == ReduceOp::MIN) acc = std::min<double>(acc, xs[r]);
        else acc += xs[r];
    }
    if (op == ReduceOp::AVG) acc = std::is_floating_point<T>::value ? acc / n : std::trunc(acc / n);
    return static_cast<T>(acc);
}

struct Checker {
    Communicator* comm;
    Mem mem;
    int rank, world;
    int passed = 0, failed = 0;
    std::vector<std::string> failures;

    void Record(bool ok, const std::string& what) {
        if (ok) {
            ++passed;
        } else {
            ++failed;
            if (failures.size() < 8) failures.push_back(what);
        }
    }

    // The communicator's view of machines when ranks are grouped K per (logical) machine in
    // rank order (K = world when every rank shares one host).
    void View(int per_machine) {
        const int k = per_machine > 0 ? std::min(per_machine, world) : world;
        const int machine = rank / k, machines = (world + k - 1) / k;
        const int first = machine * k, size = std::min(k, world - first);
        std::vector<int> locals, leaders;
        for (int r = first; r < first + size; ++r) locals.push_back(r);
        for (int m = 0; m < machines; ++m) leaders.push_back(m * k);
        Record(comm->GetRank() == rank && comm->GetWorldSize() == world, "view: rank/world");
        Record(comm->GetMachineIndex() == machine && comm->GetMachineCount() == machines, "view: machines");
        Record(comm->IsSingleMachine() == (machines == 1), "view: single machine");
        Record(comm->GetLocalRank() == rank - first && comm->GetLocalSize() == size, "view: local rank/size");
        Record(comm->GetLocalRanks() == locals, "view: local ranks");
        Record(comm->GetMachineLeaders() == leaders, "view: machine leaders");
    }

    template <typename T>
    void AllReduce(DataType dt, ReduceOp op, size_t n, bool in_place) {
        std::vector<T> in(n), out(n + 1);
        for (size_t i = 0; i < n; ++i) in[i] = Value<T>(rank, i);
        void* s = mem.Alloc(n * sizeof(T));
        void* d = in_place ? s : mem.Alloc((n + 1) * sizeof(T));
        T sentinel = static_cast<T>(77);
        std::vector<T> init(n + 1, sentinel);
        if (!in_place) mem.Put(d, init.data(), (n + 1) * sizeof(T));
        mem.Put(s, in.data(), n * sizeof(T));
        bool ok = comm->AllReduce(s, d, n, dt, op);
        mem.Get(out.data(), d, (in_place ? n : n + 1) * sizeof(T));
        for (size_t i = 0; ok && i < n; ++i) {
            std::vector<T> xs(world);
            for (int r = 0; r < world; ++r) xs[r] = Value<T>(r, i);
            ok = out[i] == Reduce<T>(op, xs, world);
        }
        if (ok && !in_place) ok = out[n] == sentinel;
        if (ok && !in_place) {  // the input must come back unchanged
            std::vector<T> back(n);
            mem.Get(back.data(), s, n * sizeof(T));
            ok = back == in;
        }
        Record(ok, "allreduce n=" + std::to_string(n) + " op=" + std::to_string(static_cast<int>(op)) +
                       (in_place ? " in-place" : ""));
        if (!in_place) mem.Free(d);
        mem.Free(s);
    }

    void Broadcast(size_t n, int root) {
        std::vector<float> buf(n);
        for (size_t i = 0; i < n; ++i) buf[i] = rank == root ? Value<float>(root, i) : -1.0f;
        void* b = mem.Alloc(n * sizeof(float));
        mem.Put(b, buf.data(), n * sizeof(float));
        bool ok = comm->Broadcast(b, n, DataType::FLOAT32, root);
        mem.Get(buf.data(), b, n * sizeof(float));
        for (size_t i = 0; ok && i < n; ++i) ok = buf[i] == Value<float>(root, i);
        Record(ok, "broadcast n=" + std::to_string(n));
        mem.Free(b);
    }

    void ReduceTo(size_t n, int root, ReduceOp op) {
        std::vector<float> in(n), out(n, -5.0f);
        for (size_t i = 0; i < n; ++i) in[i] = Value<float>(rank, i);
        void* s = mem.Alloc(n * sizeof(float));
        void* d = rank == root ? mem.Alloc(n * sizeof(float)) : nullptr;  // non-roots may pass null
        mem.Put(s, in.data(), n * sizeof(float));
        bool ok = comm->Reduce(s, d, n, DataType::FLOAT32, op, root);
        if (rank == root) {
            mem.Get(out.data(), d, n * sizeof(float));
            for (size_t i = 0; ok && i < n; ++i) {
                std::vector<float> xs(world);
                for (int r = 0; r < world; ++r) xs[r] = Value<float>(r, i);
                ok = out[i] == Reduce<float>(op, xs, world);
            }
            mem.Free(d);
        }
        Record(ok, "reduce n=" + std::to_string(n));
        mem.Free(s);
    }

    void AllGather(size_t n) {
        std::vector<int> in(n), out(n * world + 1, 77);
        for (size_t i = 0; i < n; ++i) in[i] = Value<int>(rank, i);
        void* s = mem.Alloc(n * sizeof(int));
        void* d = mem.Alloc((n * world + 1) * sizeof(int));
        mem.Put(s, in.data(), n * sizeof(int));
        mem.Put(d, out.data(), out.size() * sizeof(int));
        bool ok = comm->AllGather(s, d, n, DataType::INT32);
        mem.Get(out.data(), d, out.size() * sizeof(int));
        for (int r = 0; ok && r < world; ++r)
            for (size_t i = 0; ok && i < n; ++i) ok = out[r * n + i] == Value<int>(r, i);
        ok = ok && out[n * world] == 77;
        Record(ok, "allgather n=" + std::to_string(n));
        mem.Free(s);
        mem.Free(d);
    }

    void ReduceScatter(size_t n) {
        std::vector<int> in(n * world), out(n + 1, 77);
        for (size_t i = 0; i < n * world; ++i) in[i] = Value<int>(rank, i);
        void* s = mem.Alloc(in.size() * sizeof(int));
        void* d = mem.Alloc((n + 1) * sizeof(int));
        mem.Put(s, in.data(), in.size() * sizeof(int));
        mem.Put(d, out.data(), out.size() * sizeof(int));
        bool ok = comm->ReduceScatter(s, d, n, DataType::INT32, ReduceOp::SUM);
        mem.Get(out.data(), d, out.size() * sizeof(int));
        for (size_t i = 0; ok && i < n; ++i) {
            int want = 0;
            for (int r = 0; r < world; ++r) want += Value<int>(r, rank * n + i);
            ok = out[i] == want;
        }
        ok = ok && out[n] == 77;
        Record(ok, "reducescatter n=" + std::to_string(n));
        mem.Free(s);
        mem.Free(d);
    }

    // Inputs staged with a plain (pageable) copy right before each call, new values every
    // iteration: a pageable host-to-device cudaMemcpy may return before its DMA lands, so a
    // collective that is not ordered after the caller's default-stream work reads stale input.
    void StagedLoop(size_t n, int iters) {
        std::vector<float> in(n), out(n);
        void* s = mem.Alloc(n * sizeof(float));
        void* d = mem.Alloc(n * sizeof(float));
        bool ok = s != nullptr && d != nullptr;
        for (int it = 0; ok && it < iters; ++it) {
            for (size_t i = 0; i < n; ++i) in[i] = Value<float>(rank + 3 * it, i);
            mem.Put(s, in.data(), n * sizeof(float));
            ok = comm->AllReduce(s, d, n, DataType::FLOAT32, ReduceOp::SUM);
            ok = ok && comm->AllReduce(d, d, n, DataType::FLOAT32, ReduceOp::MAX);  // in place as well
            mem.Get(out.data(), d, n * sizeof(float));
            for (size_t i = 0; ok && i < n; ++i) {
                std::vector<float> xs(world);
                for (int r = 0; r < world; ++r) xs[r] = Value<float>(r + 3 * it, i);
                ok = out[i] == Reduce<float>(ReduceOp::SUM, xs, world);
            }
        }
        Record(ok, "staged inputs n=" + std::to_string(n) + " x" + std::to_string(iters));
        mem.Free(s);
        mem.Free(d);
    }

    // A nested group of four independent collectives; only the outer GroupEnd runs them.
    void Group(size_t n) {
        std::vector<void*> bufs;
        std::vector<std::vector<float>> host(4, std::vector<float>(n));
        for (int k = 0; k < 4; ++k) {
            for (size_t i = 0; i < n; ++i) host[k][i] = Value<float>(rank + k, i);
            void* b = mem.Alloc(n * sizeof(float));
            mem.Put(b, host[k].data(), n * sizeof(float));
            bufs.push_back(b);
        }
        comm->GroupStart();
        comm->GroupStart();
        bool ok = comm->AllReduce(bufs[0], bufs[0], n, DataType::FLOAT32, ReduceOp::SUM);
        ok = ok && comm->AllReduce(bufs[1], bufs[1], n, DataType::FLOAT32, ReduceOp::MAX);
        ok = ok && comm->GroupEnd();  // inner: must not execute
        ok = ok && comm->AllReduce(bufs[2], bufs[2], n, DataType::FLOAT32, ReduceOp::MIN);
        ok = ok && comm->Broadcast(bufs[3], n, DataType::FLOAT32, 0);
        ok = comm->GroupEnd() && ok;
        const ReduceOp ops[3] = {ReduceOp::SUM, ReduceOp::MAX, ReduceOp::MIN};
        for (int k = 0; ok && k < 4; ++k) {
            std::vector<float> out(n);
            mem.Get(out.data(), bufs[k], n * sizeof(float));
            for (size_t i = 0; ok && i < n; ++i) {
                float want;
                if (k < 3) {
                    std::vector<float> xs(world);
                    for (int r = 0; r < world; ++r) xs[r] = Value<float>(r + k, i);
                    want = Reduce<float>(ops[k], xs, world);
                } else {
                    want = Value<float>(0 + k, i);
                }
                ok = out[i] == want;
            }
        }
        Record(ok, "nested group n=" + std::to_string(n));
        for (void* b : bufs) mem.Free(b);
    }

    void SendRecvRing(size_t n) {
        if (world < 2) return;
        const int next = (rank + 1) % world, prev = (rank + world - 1) % world;
        std::vector<int> out(n), in(n, -1);
        for (size_t i = 0; i < n; ++i) out[i] = Value<int>(rank, i);
        void* s = mem.Alloc(n * sizeof(int));
        void* d = mem.Alloc(n * sizeof(int));
        mem.Put(s, out.data(), n * sizeof(int));
        comm->GroupStart();
        bool ok = comm->Send(s, n, DataType::INT32, next);
        ok = ok && comm->Recv(d, n, DataType::INT32, prev);
        ok = comm->GroupEnd() && ok;
        mem.Get(in.data(), d, n * sizeof(int));
        for (size_t i = 0; ok && i < n; ++i) ok = in[i] == Value<int>(prev, i);
        Record(ok, "send/recv ring n=" + std::to_string(n));
        mem.Free(s);
        mem.Free(d);
    }

    // Split: ranks of equal parity form a child communicator ranked in reverse (key = -rank);
    // an AllReduce in the child sums exactly its members. Host buffers only.
    void Split() {
        if (mem.device) return;
        Communicator child;
        bool ok = comm->Split(rank % 2, -rank, &child);
        int members = 0, expect = 0;
        for (int r = rank % 2; r < world; r += 2) {
            ++members;
            expect += r + 1;
        }
        ok = ok && child.GetWorldSize() == members && child.GetRank() == (members - 1 - rank / 2);
        int v = rank + 1;
        ok = ok && child.AllReduce(&v, &v, 1, DataType::INT32, ReduceOp::SUM) && v == expect;
        child.Finalize();
        Record(ok, "split by parity");
    }

    void Contract() {
        Record(comm->AllReduce(nullptr, nullptr, 0, DataType::FLOAT32, ReduceOp::SUM), "count 0 with null buffers");
        void* b = mem.Alloc(64);
        Record(!comm->Broadcast(b, 4, DataType::FLOAT32, world), "bad root rejected");
        Record(!comm->AllReduce(nullptr, b, 4, DataType::FLOAT32, ReduceOp::SUM), "null send buffer rejected");
        Record(!comm->Send(b, 4, DataType::FLOAT32, rank), "send to self rejected");
        comm->GroupStart();
        Record(!comm->Reduce(b, b, 4, DataType::FLOAT32, ReduceOp::SUM, -1), "bad root rejected inside a group");
        Record(comm->GroupEnd(), "group with only rejected work ends cleanly");
        mem.Free(b);
    }
};

std::vector<size_t> ParseCounts(const std::string& s) {
    std::vector<size_t> out;
    std::stringstream ss(s);
    std::string tok;
    while (std::getline(ss, tok, ',')) out.push_back(static_cast<size_t>(std::atoll(tok.c_str())));
    return out;
}

int RunBench(Communicator* comm, Mem mem, int rank, int world, const std::vector<size_t>& counts, int warmup,
             int iters) {
    int rc = 0;
    for (size_t n : counts) {
        std::vector<int> in(n), out(n);
        for (size_t i = 0; i < n; ++i) in[i] = static_cast<int>((rank * 7 + i) % 1000);
        void* s = mem.Alloc(n * sizeof(int));
        void* d = mem.Alloc(n * sizeof(int));
        mem.Put(s, in.data(), n * sizeof(int));
        bool ok = true;
        for (int w = 0; w < warmup && ok; ++w) ok = comm->AllReduce(s, d, n, DataType::INT32, ReduceOp::SUM);
        mem.Get(out.data(), d, n * sizeof(int));
        for (size_t i = 0; ok && i < n; ++i) {
            long want = 0;
            for (int r = 0; r < world; ++r) want += static_cast<long>((r * 7 + i) % 1000);
            ok = out[i] == want;
        }
        ok = ok && comm->Barrier();
        auto t0 = std::chrono::steady_clock::now();
        for (int it = 0; it < iters && ok; ++it) ok = comm->AllReduce(s, d, n, DataType::INT32, ReduceOp::SUM);
        double us = std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count() / iters;
        double tmax = us;
        void* tb = mem.Alloc(sizeof(double));
        mem.Put(tb, &us, sizeof(double));
        ok = ok && comm->AllReduce(tb, tb, 1, DataType::FLOAT64, ReduceOp::MAX);
        mem.Get(&tmax, tb, sizeof(double));
        mem.Free(tb);
        const double bytes = static_cast<double>(n) * sizeof(int);
        const double algbw = bytes / tmax / 1e3;  // GB/s
        const double busbw = world > 1 ? algbw * 2.0 * (world - 1) / world : algbw;
        if (rank == 0) {
            std::printf("{\"op\": \"allreduce\", \"dtype\": \"int32\", \"path\": \"%s\", \"ranks\": %d, "
                        "\"count\": %zu, \"bytes\": %.0f, \"time_us\": %.2f, \"algbw_gbs\": %.3f, "
                        "\"busbw_gbs\": %.3f, \"check\": %s, \"warmup\": %d, \"iters\": %d}\n",
                        mem.device ? "device" : "host", world, n, bytes, tmax, algbw, busbw, ok ? "true" : "false",
                        warmup, iters);
            std::fflush(stdout);
        }
        rc |= ok ? 0 : 1;
        mem.Free(s);
        mem.Free(d);
    }
    return rc;
}

// Many small AllReduces in one group (the reference's --group-small benchmark,
// tests/benchmark/test_allreduce_benchmark.cpp:423-490): messages per second, max over ranks.
int RunGroupBench(Communicator* comm, Mem mem, int rank, int world, int nmsg, size_t bytes, int warmup, int iters) {
    const size_t n = bytes / sizeof(float);
    std::vector<void*> bufs;
    std::vector<float> host(n);
    for (int k = 0; k < nmsg; ++k) {
        for (size_t i = 0; i < n; ++i) host[i] = Value<float>(rank + k, i);
        void* b = mem.Alloc(n * sizeof(float));
        mem.Put(b, host.data(), n * sizeof(float));
        bufs.push_back(b);
    }
    auto one = [&]() {
        comm->GroupStart();
        bool ok = true;
        for (int k = 0; k < nmsg && ok; ++k) ok = comm->AllReduce(bufs[k], bufs[k], n, DataType::FLOAT32, ReduceOp::MAX);
        return comm->GroupEnd() && ok;
    };
    bool ok = true;
    for (int w = 0; w < warmup && ok; ++w) ok = one();
    // MAX of identical-per-rank inputs is idempotent: check the first buffer after the warm-up.
    std::vector<float> out(n);
    mem.Get(out.data(), bufs[0], n * sizeof(float));
    for (size_t i = 0; ok && i < n; ++i) {
        float want = Value<float>(0, i);
        for (int r = 1; r < world; ++r) want = std::max(want, Value<float>(r, i));
        ok = out[i] == want;
    }
    ok = ok && comm->Barrier();
    auto t0 = std::chrono::steady_clock::now();
    for (int it = 0; it < iters && ok; ++it) ok = one();
    double us = std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count() / iters;
    double tmax = us;
    void* tb = mem.Alloc(sizeof(double));
    mem.Put(tb, &us, sizeof(double));
    ok = ok && comm->AllReduce(tb, tb, 1, DataType::FLOAT64, ReduceOp::MAX);
    mem.Get(&tmax, tb, sizeof(double));
    mem.Free(tb);
    if (rank == 0) {
        std::printf("{\"op\": \"allreduce_group\", \"path\": \"%s\", \"ranks\": %d, \"messages\": %d, "
                    "\"bytes_per_message\": %zu, \"us_per_group\": %.1f, \"msgs_per_s\": %.0f, \"check\": %s}\n",
                    mem.device ? "device" : "host", world, nmsg, bytes, tmax, nmsg / tmax * 1e6, ok ? "true" : "false");
        std::fflush(stdout);
    }
    for (void* b : bufs) mem.Free(b);
    return ok ? 0 : 1;
}

}  // namespace

std::string g_logical_host;
std::string LogicalHost() { return g_logical_host; }

int main(int argc, char** argv) {
    std::string mode = argc > 1 ? argv[1] : "check";
    bool device = false;
    std::vector<size_t> counts = {32768, 131072};
    int warmup = 20, iters = 100, channels = 0, nmsg = 64, per_machine = 0, fuzz_seed = 1, fuzz_ops = 50;
    size_t msg_bytes = 256u << 10;
    for (int i = 2; i < argc; ++i) {
        std::string a = argv[i];
        if (a == "--device") device = true;
        else if (a == "--counts" && i + 1 < argc) counts = ParseCounts(argv[++i]);
        else if (a == "--warmup" && i + 1 < argc) warmup = std::atoi(argv[++i]);
        else if (a == "--iters" && i + 1 < argc) iters = std::atoi(argv[++i]);
        else if (a == "--channels" && i + 1 < argc) channels = std::atoi(argv[++i]);
        else if (a == "--messages" && i + 1 < argc) nmsg = std::atoi(argv[++i]);
        else if (a == "--message-bytes" && i + 1 < argc) msg_bytes = static_cast<size_t>(std::atoll(argv[++i]));
        else if (a == "--ranks-per-machine" && i + 1 < argc) per_machine = std::atoi(argv[++i]);
        else if (a == "--seed" && i + 1 < argc) fuzz_seed = std::atoi(argv[++i]);
        else if (a == "--ops" && i + 1 < argc) fuzz_ops = std::atoi(argv[++i]);
    }
    const int rank = EnvInt("BCCL_RANK", 0), world = EnvInt("BCCL_WORLD_SIZE", 1);
    Communicator comm;
    bccl::CommConfig cfg;
    cfg.rank = rank;
    cfg.world_size = world;
    cfg.n_channels = channels;
    if (per_machine > 0) {
        g_logical_host = "logical-machine-" + std::to_string(rank / per_machine);
        cfg.get_hostname = LogicalHost;
    }
    if (device) {
        cfg.device = EnvInt("BCCL_DEVICE", EnvInt("BCCL_LOCAL_RANK", rank));
        if (cudaSetDevice(cfg.device) != cudaSuccess) {
            std::fprintf(stderr, "rank %d: no CUDA device %d\n", rank, cfg.device);
            return 3;
        }
    }
    if (!ExchangeId(rank, &cfg.unique_id, &comm) || !comm.Init(cfg)) {
        std::fprintf(stderr, "rank %d: init failed\n", rank);
        return 1;
    }
    Mem mem;
    mem.device = device;
    int rc = 0;
    if (mode == "bench") {
        rc = RunBench(&comm, mem, rank, world, counts, warmup, iters);
    } else if (mode == "bench-group") {
        rc = RunGroupBench(&comm, mem, rank, world, nmsg, msg_bytes, warmup, iters);
    } else if (mode == "fuzz") {
        // A random sequence of checked operations, the same on every rank (one seed): every
        // collective and dtype, SUM/MAX/MIN/AVG, in place or not, sizes from 1 element to a few
        // MiB (so channel splitting, alternating buffer sets and single-copy Send/Recv all run),
        // groups and Send/Recv around the ring. Meant for the sanitizer builds.
        Checker c{&comm, mem, rank, world};
        std::mt19937_64 rng(static_cast<uint64_t>(fuzz_seed));
        const size_t sizes[] = {1, 17, 1000, 4097, 40000, 300001, 1u << 20};
        const ReduceOp ops[] = {ReduceOp::SUM, ReduceOp::MAX, ReduceOp::MIN, ReduceOp::AVG};
        for (int k = 0; k < fuzz_ops; ++k) {
            const size_t n = sizes[rng() % 7];
            const ReduceOp op = ops[rng() % 4];
            const int root = static_cast<int>(rng() % static_cast<uint64_t>(world));
            const bool in_place = rng() % 2 == 0;
            switch (rng() % 9) {
            case 0: c.AllReduce<int>(DataType::INT32, op, n, in_place); break;
            case 1: c.AllReduce<float>(DataType::FLOAT32, op, n, in_place); break;
            case 2: c.AllReduce<double>(DataType::FLOAT64, op, n, in_place); break;
            case 3: c.AllReduce<long long>(DataType::INT64, op, n, in_place); break;
            case 4: c.Broadcast(n, root); break;
            case 5: c.ReduceTo(n, root, op == ReduceOp::AVG ? ReduceOp::SUM : op); break;
            case 6: c.AllGather(n); break;
            case 7: c.ReduceScatter(n); break;
            default: (rng() % 2 ? c.Group(n) : c.SendRecvRing(n)); break;
            }
        }
        int fails = c.failed, total_fail = 0;
        void* fb = mem.Alloc(sizeof(int));
        mem.Put(fb, &fails, sizeof(int));
        if (!comm.AllReduce(fb, fb, 1, DataType::INT32, ReduceOp::SUM)) fails = -1;
        mem.Get(&total_fail, fb, sizeof(int));
        mem.Free(fb);
        if (fails < 0) total_fail = world;
        if (rank == 0) {
            std::printf("{\"fuzz_ops\": %d, \"passed\": %d, \"failed_all_ranks\": %d, \"ranks\": %d, \"failures\": [",
                        fuzz_ops, c.passed, total_fail, world);
            for (size_t i = 0; i < c.failures.size(); ++i)
                std::printf("%s\"%s\"", i ? ", " : "", c.failures[i].c_str());
            std::printf("]}\n");
        }
        rc = total_fail == 0 ? 0 : 1;
    } else {
        Checker c{&comm, mem, rank, world};
        c.View(per_machine);
        for (size_t n : {size_t(1), size_t(1000), size_t(32768 + 3)}) {
            for (ReduceOp op : {ReduceOp::SUM, ReduceOp::MAX, ReduceOp::MIN, ReduceOp::AVG}) {
                c.AllReduce<int>(DataType::INT32, op, n, false);
                c.AllReduce<float>(DataType::FLOAT32, op, n, false);
            }
            c.AllReduce<double>(DataType::FLOAT64, ReduceOp::SUM, n, true);
            c.AllReduce<long long>(DataType::INT64, ReduceOp::MAX, n, true);
            c.Broadcast(n, world - 1);
            c.ReduceTo(n, 1 % world, ReduceOp::SUM);
            c.ReduceTo(n, 0, ReduceOp::MAX);
            c.AllGather(n);
            c.ReduceScatter(n);
            c.Group(n);
            c.SendRecvRing(n);
        }
        c.SendRecvRing(300001);  // above the host path's single-copy threshold (256 KiB)
        c.StagedLoop(32768 + 3, 8);
        c.StagedLoop((1u << 18) + 3, 8);  // 1 MiB + 12 bytes
        c.Split();
        c.Contract();
        int fails = c.failed, total_fail = 0;
        void* fb = mem.Alloc(sizeof(int));
        mem.Put(fb, &fails, sizeof(int));
        if (!comm.AllReduce(fb, fb, 1, DataType::INT32, ReduceOp::SUM)) fails = -1;
        mem.Get(&total_fail, fb, sizeof(int));
        mem.Free(fb);
        if (fails < 0) total_fail = world;
        if (rank == 0) {
            std::printf("{\"passed\": %d, \"failed\": %d, \"failed_all_ranks\": %d, \"ranks\": %d, \"machines\": %d, "
                        "\"path\": \"%s\"",
                        c.passed, c.failed, total_fail, world, comm.GetMachineCount(), device ? "device" : "host");
            std::printf(", \"failures\": [");
            for (size_t i = 0; i < c.failures.size(); ++i)
                std::printf("%s\"%s\"", i ? ", " : "", c.failures[i].c_str());
            std::printf("]}\n");
        } else if (c.failed) {
            for (const std::string& f : c.failures) std::fprintf(stderr, "rank %d: FAILED %s\n", rank, f.c_str());
        }
        rc = total_fail == 0 ? 0 : 1;
    }
    comm.Finalize();
    return rc;
}
