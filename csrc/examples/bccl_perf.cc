// bccl_perf: size sweep of one collective through the C++ API, host or device buffers; the
// counterpart of the reference's AllReduce benchmark (OriginCCL
// tests/benchmark/test_allreduce_benchmark.cpp:113-421: --min/max-bytes, --factor, warm-up and
// timed iterations, time = max over ranks, busbw = algbw x 2(N-1)/N, validated) for every
// collective, in the column layout of nccl-tests.
//
//   bccl_run -np 4 bccl_perf --op allreduce -b 8 -e 128M -f 2
//   bccl_run -np 8 --gpus bccl_perf --device --op allgather --dtype bf16 -b 1K -e 1G --json
//
// Host buffers are timed with the host clock between barriers; device buffers with CUDA events
// on the communicator's stream (calls enqueue; one synchronisation per timed batch). Every size
// is checked once against exact small-integer values (float types divide them by 8, so bf16 /
// fp16 sums stay exact for a few ranks). Rank 0 prints one row (or JSON line) per size.
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <string>
#include <thread>
#include <vector>

#include <cuda_runtime.h>

#include "bccl/communicator.h"

using bccl::Communicator;
using bccl::DataType;
using bccl::ReduceOp;

namespace {

struct Options {
    std::string op = "allreduce";
    size_t min_bytes = 8, max_bytes = 64u << 20;
    double factor = 2;
    DataType dtype = DataType::FLOAT32;
    ReduceOp redop = ReduceOp::SUM;
    int warmup = 5, iters = 20, channels = 0, root = 0;
    bool device = false, inplace = false, json = false, check = true;
};

size_t ParseSize(const std::string& s) {
    double v = std::atof(s.c_str());
    const char c = s.empty() ? '\0' : s.back();
    if (c == 'K' || c == 'k') v *= 1024.0;
    if (c == 'M' || c == 'm') v *= 1024.0 * 1024.0;
    if (c == 'G' || c == 'g') v *= 1024.0 * 1024.0 * 1024.0;
    return static_cast<size_t>(v);
}

size_t Size(DataType t) {
    switch (t) {
    case DataType::FLOAT64:
    case DataType::INT64: return 8;
    case DataType::BF16:
    case DataType::FP16: return 2;
    default: return 4;
    }
}

// Exact test values: small integers (divided by 8 for floating-point types).
double Val(int rank, size_t i) { return static_cast<double>(static_cast<long>((rank * 7 + i * 13) % 17) - 8); }

// Writes `n` values of `rank` into `out` as `t`, starting at element index `first`.
void Fill(DataType t, int rank, size_t first, size_t n, void* out) {
    for (size_t i = 0; i < n; ++i) {
        const double v = Val(rank, first + i);
        switch (t) {
        case DataType::FLOAT32: static_cast<float*>(out)[i] = static_cast<float>(v / 8); break;
        case DataType::FLOAT64: static_cast<double*>(out)[i] = v / 8; break;
        case DataType::INT32: static_cast<int32_t*>(out)[i] = static_cast<int32_t>(v); break;
        case DataType::INT64: static_cast<int64_t*>(out)[i] = static_cast<int64_t>(v); break;
        case DataType::BF16: {
            float f = static_cast<float>(v / 8);
            uint32_t u;
            std::memcpy(&u, &f, 4);
            static_cast<uint16_t*>(out)[i] = static_cast<uint16_t>(u >> 16);  // exact: few mantissa bits
            break;
        }
        case DataType::FP16: {
            // v / 8 with |v| <= 8: sign, exponent and up to 3 mantissa bits, built directly.
            const double a = std::fabs(v / 8);
            uint16_t h = 0;
            if (a > 0) {
                int e = static_cast<int>(std::floor(std::log2(a)));
                const double m = a / std::ldexp(1.0, e) - 1.0;
                h = static_cast<uint16_t>(((e + 15) << 10) | static_cast<int>(std::lround(m * 1024)));
            }
            if (v < 0) h |= 0x8000;
            static_cast<uint16_t*>(out)[i] = h;
            break;
        }
        }
    }
}

double Get(DataType t, const void* p, size_t i) {
    switch (t) {
    case DataType::FLOAT32: return static_cast<const float*>(p)[i];
    case DataType::FLOAT64: return static_cast<const double*>(p)[i];
    case DataType::INT32: return static_cast<const int32_t*>(p)[i];
    case DataType::INT64: return static_cast<double>(static_cast<const int64_t*>(p)[i]);
    case DataType::BF16: {
        uint32_t u = static_cast<uint32_t>(static_cast<const uint16_t*>(p)[i]) << 16;
        float f;
        std::memcpy(&f, &u, 4);
        return f;
    }
    case DataType::FP16: {
        const uint16_t h = static_cast<const uint16_t*>(p)[i];
        const int e = (h >> 10) & 31, m = h & 1023;
        double v = e == 0 ? std::ldexp(m, -24) : std::ldexp(1.0 + m / 1024.0, e - 15);
        return (h & 0x8000) ? -v : v;
    }
    }
    return 0;
}

bool IsFloat(DataType t) { return t != DataType::INT32 && t != DataType::INT64; }

// Expected value of element i of rank `r`'s reduction over `world` ranks (the input index is
// `i` for AllReduce/Reduce and `block * count + i` for ReduceScatter).
double Expect(const Options& o, int world, size_t idx) {
    double acc = o.redop == ReduceOp::MAX ? -1e300 : o.redop == ReduceOp::MIN ? 1e300 : 0;
    for (int q = 0; q < world; ++q) {
        const double v = Val(q, idx) / (IsFloat(o.dtype) ? 8 : 1);
        if (o.redop == ReduceOp::MAX) acc = std::max(acc, v);
        else if (o.redop == ReduceOp::MIN) acc = std::min(acc, v);
        else acc += v;
    }
    if (o.redop == ReduceOp::AVG) acc = IsFloat(o.dtype) ? acc / world : std::trunc(acc / world);
    return acc;
}

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

bool ExchangeId(int rank, bccl::UniqueId* id, Communicator* comm) {
    if (const char* m = std::getenv("BCCL_MASTER")) {
        if (rank == 0) return comm->GetUniqueId(*id);
        std::string s(m);
        const size_t colon = s.rfind(':');
        if (colon == std::string::npos) return false;
        std::snprintf(id->ip_addr, sizeof(id->ip_addr), "%s", s.substr(0, colon).c_str());
        id->port = static_cast<uint16_t>(std::atoi(s.substr(colon + 1).c_str()));
        return true;
    }
    const char* path = std::getenv("BCCL_ID_FILE");
    if (path == nullptr) return false;
    if (rank == 0) {
        if (!comm->GetUniqueId(*id)) return false;
        const std::string tmp = std::string(path) + ".tmp";
        {
            std::ofstream f(tmp);
            f << id->ip_addr << ":" << id->port;
        }
        return std::rename(tmp.c_str(), path) == 0;
    }
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(60);
    while (access(path, R_OK) != 0) {
        if (std::chrono::steady_clock::now() > deadline) return false;
        std::this_thread::sleep_for(std::chrono::milliseconds(5));
    }
    std::ifstream f(path);
    std::string s;
    f >> s;
    const size_t colon = s.rfind(':');
    if (colon == std::string::npos) return false;
    std::snprintf(id->ip_addr, sizeof(id->ip_addr), "%s", s.substr(0, colon).c_str());
    id->port = static_cast<uint16_t>(std::atoi(s.substr(colon + 1).c_str()));
    return true;
}

// busbw / algbw factor (the nccl-tests convention the reference's benchmark uses for AllReduce).
double BusFactor(const std::string& op, int n) {
    if (n <= 1) return 1.0;
    if (op == "allreduce") return 2.0 * (n - 1) / n;
    if (op == "allgather" || op == "reducescatter") return static_cast<double>(n - 1) / n;
    return 1.0;
}

}  // namespace

int main(int argc, char** argv) {
    Options o;
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        auto next = [&]() { return i + 1 < argc ? std::string(argv[++i]) : std::string(); };
        if (a == "--op") o.op = next();
        else if (a == "-b" || a == "--min-bytes") o.min_bytes = ParseSize(next());
        else if (a == "-e" || a == "--max-bytes") o.max_bytes = ParseSize(next());
        else if (a == "-f" || a == "--factor") o.factor = std::atof(next().c_str());
        else if (a == "-w" || a == "--warmup") o.warmup = std::atoi(next().c_str());
        else if (a == "-n" || a == "--iters") o.iters = std::atoi(next().c_str());
        else if (a == "--channels") o.channels = std::atoi(next().c_str());
        else if (a == "--root") o.root = std::atoi(next().c_str());
        else if (a == "--device") o.device = true;
        else if (a == "--inplace") o.inplace = true;
        else if (a == "--json") o.json = true;
        else if (a == "--no-check") o.check = false;
        else if (a == "--dtype") {
            const std::string d = next();
            o.dtype = d == "f64" ? DataType::FLOAT64 : d == "i32" ? DataType::INT32 : d == "i64" ? DataType::INT64
                    : d == "bf16" ? DataType::BF16 : d == "f16" ? DataType::FP16 : DataType::FLOAT32;
        } else if (a == "--redop") {
            const std::string r = next();
            o.redop = r == "max" ? ReduceOp::MAX : r == "min" ? ReduceOp::MIN : r == "avg" ? ReduceOp::AVG : ReduceOp::SUM;
        } else {
            std::fprintf(stderr, "bccl_perf: unknown option %s\n", a.c_str());
            return 2;
        }
    }
    const std::vector<std::string> ops = {"allreduce", "allgather", "reducescatter", "broadcast", "reduce", "sendrecv"};
    if (std::find(ops.begin(), ops.end(), o.op) == ops.end() || o.factor <= 1.0 || o.iters < 1) {
        std::fprintf(stderr, "bccl_perf: bad --op / --factor / --iters\n");
        return 2;
    }
    const int rank = std::atoi(std::getenv("BCCL_RANK") ? std::getenv("BCCL_RANK") : "0");
    const int world = std::atoi(std::getenv("BCCL_WORLD_SIZE") ? std::getenv("BCCL_WORLD_SIZE") : "1");
    if (o.op == "sendrecv" && world < 2) {
        std::fprintf(stderr, "bccl_perf: sendrecv needs at least 2 ranks\n");
        return 2;
    }
    Communicator comm;
    bccl::CommConfig cfg;
    cfg.rank = rank;
    cfg.world_size = world;
    cfg.n_channels = o.channels;
    cudaStream_t stream = nullptr;
    if (o.device) {
        const char* d = std::getenv("BCCL_DEVICE");
        cfg.device = d ? std::atoi(d) : rank;
        if (cudaSetDevice(cfg.device) != cudaSuccess || cudaStreamCreate(&stream) != cudaSuccess) {
            std::fprintf(stderr, "rank %d: no CUDA device %d\n", rank, cfg.device);
            return 3;
        }
    }
    if (!ExchangeId(rank, &cfg.unique_id, &comm) || !comm.Init(cfg)) {
        std::fprintf(stderr, "rank %d: init failed\n", rank);
        return 1;
    }
    if (o.device) comm.SetStream(stream);
    Mem mem;
    mem.device = o.device;
    const size_t es = Size(o.dtype);
    const int root = std::min(std::max(o.root, 0), world - 1);
    if (rank == 0 && !o.json) {
        std::printf("# bccl_perf %s %s, %d ranks, %s buffers, %d warm-up + %d timed iterations, time = max over ranks\n",
                    o.op.c_str(), o.inplace ? "in place" : "out of place", world, o.device ? "device" : "host",
                    o.warmup, o.iters);
        std::printf("%12s %12s %12s %10s %10s %7s\n", "bytes", "count", "time_us", "algbw_GBs", "busbw_GBs", "check");
    }
    int failures = 0;
    for (size_t bytes = std::max(o.min_bytes, es); bytes <= o.max_bytes;
         bytes = std::max(bytes + es, static_cast<size_t>(static_cast<double>(bytes) * o.factor))) {
        const size_t count = bytes / es;
        // Per-rank payload as nccl-tests: AllGather gathers count per rank, ReduceScatter
        // scatters count per rank (input world * count).
        const bool rs = o.op == "reducescatter", ag = o.op == "allgather";
        const size_t in_elems = rs ? count * world : count, out_elems = ag ? count * world : count;
        std::vector<char> host_in(in_elems * es), host_out(out_elems * es);
        Fill(o.dtype, rank, 0, in_elems, host_in.data());
        void* in = mem.Alloc(in_elems * es);
        void* out = (o.inplace && !rs && !ag) ? in : mem.Alloc(out_elems * es);
        mem.Put(in, host_in.data(), in_elems * es);
        const int peer_next = (rank + 1) % world, peer_prev = (rank + world - 1) % world;
        auto call = [&]() -> bool {
            if (o.op == "allreduce") return comm.AllReduce(in, out, count, o.dtype, o.redop);
            if (ag) return comm.AllGather(in, out, count, o.dtype);
            if (rs) return comm.ReduceScatter(in, out, count, o.dtype, o.redop);
            if (o.op == "broadcast") return comm.BroadcastTo(in, out, count, o.dtype, root);
            if (o.op == "reduce") return comm.Reduce(in, out, count, o.dtype, o.redop, root);
            comm.GroupStart();
            bool ok = comm.Send(in, count, o.dtype, peer_next) && comm.Recv(out, count, o.dtype, peer_prev);
            return comm.GroupEnd() && ok;
        };
        bool ok = true;
        // Correctness, once per size (before timing: the timed calls reduce in place repeatedly).
        if (o.check) {
            ok = call() && comm.Synchronize();
            mem.Get(host_out.data(), out, out_elems * es);
            for (size_t i = 0; ok && i < out_elems; ++i) {
                double want;
                if (o.op == "allreduce") want = Expect(o, world, i);
                else if (rs) want = Expect(o, world, static_cast<size_t>(rank) * count + i);
                else if (o.op == "reduce") want = rank == root ? Expect(o, world, i) : Get(o.dtype, host_out.data(), i);
                else if (ag) want = Val(static_cast<int>(i / count), i % count) / (IsFloat(o.dtype) ? 8 : 1);
                else if (o.op == "broadcast") want = Val(root, i) / (IsFloat(o.dtype) ? 8 : 1);
                else want = Val(peer_prev, i) / (IsFloat(o.dtype) ? 8 : 1);
                const double got = Get(o.dtype, host_out.data(), i);
                const double tol = (o.dtype == DataType::BF16 || o.dtype == DataType::FP16) && o.redop == ReduceOp::AVG
                                       ? 1e-2 * std::max(1.0, std::fabs(want)) : 1e-6 * std::max(1.0, std::fabs(want));
                ok = std::fabs(got - want) <= tol;
            }
            if (o.inplace && !rs && !ag) mem.Put(in, host_in.data(), in_elems * es);
        }
        for (int w = 0; w < o.warmup && ok; ++w) ok = call();
        ok = ok && comm.Synchronize() && comm.Barrier();
        double us = 0;
        if (o.device) {
            cudaEvent_t e0, e1;
            cudaEventCreate(&e0);
            cudaEventCreate(&e1);
            cudaEventRecord(e0, stream);
            for (int it = 0; it < o.iters && ok; ++it) ok = call();
            cudaEventRecord(e1, stream);
            ok = ok && comm.Synchronize();
            float ms = 0;
            cudaEventElapsedTime(&ms, e0, e1);
            us = ms * 1e3 / o.iters;
            cudaEventDestroy(e0);
            cudaEventDestroy(e1);
        } else {
            const auto t0 = std::chrono::steady_clock::now();
            for (int it = 0; it < o.iters && ok; ++it) ok = call();
            us = std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count() / o.iters;
        }
        // Max of the per-rank times (and of the failures) over the ranks, through the library.
        double stats[2] = {us, ok ? 0.0 : 1.0};
        void* sbuf = mem.Alloc(sizeof(stats));
        mem.Put(sbuf, stats, sizeof(stats));
        comm.ClearStream();
        const bool reduced = comm.AllReduce(sbuf, sbuf, 2, DataType::FLOAT64, ReduceOp::MAX);
        if (o.device) comm.SetStream(stream);
        mem.Get(stats, sbuf, sizeof(stats));
        mem.Free(sbuf);
        if (!reduced) stats[1] = 1;
        failures += stats[1] != 0;
        const double moved = static_cast<double>(ag || rs ? count * world : count) * es;
        const double algbw = stats[0] > 0 ? moved / (stats[0] * 1e-6) / 1e9 : 0;
        const double busbw = algbw * BusFactor(o.op, world);
        if (rank == 0) {
            if (o.json) {
                std::printf("{\"op\": \"%s\", \"bytes\": %zu, \"count\": %zu, \"ranks\": %d, \"path\": \"%s\", "
                            "\"time_us\": %.3f, \"algbw_gbs\": %.3f, \"busbw_gbs\": %.3f, \"check\": %s}\n",
                            o.op.c_str(), bytes, count, world, o.device ? "device" : "host", stats[0], algbw, busbw,
                            stats[1] == 0 ? "true" : "false");
            } else {
                std::printf("%12zu %12zu %12.2f %10.3f %10.3f %7s\n", bytes, count, stats[0], algbw, busbw,
                            stats[1] == 0 ? "ok" : "FAIL");
            }
            std::fflush(stdout);
        }
        if (out != in) mem.Free(out);
        mem.Free(in);
    }
    comm.Finalize();
    if (stream) cudaStreamDestroy(stream);
    return failures ? 1 : 0;
}
