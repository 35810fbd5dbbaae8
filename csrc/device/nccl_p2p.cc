#include "device/nccl_p2p.h"

#include <dlfcn.h>

#include <cstdio>
#include <cstring>
#include <string>

#include <nccl.h>

#include "core/bootstrap.h"
#include "core/env.h"
#include "core/logger.h"

namespace bccl {
namespace {

struct NcclFns {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*);
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*GroupStart)();
    ncclResult_t (*GroupEnd)();
    const char* (*GetErrorString)(ncclResult_t);
    ncclResult_t (*GetVersion)(int*);
};
NcclFns g_fns;

ncclDataType_t ToNccl(DataType d) {
    switch (d) {
    case DataType::FLOAT32: return ncclFloat32;
    case DataType::FLOAT64: return ncclFloat64;
    case DataType::INT32: return ncclInt32;
    case DataType::INT64: return ncclInt64;
    case DataType::BF16: return ncclBfloat16;
    case DataType::FP16: return ncclFloat16;
    }
    return ncclFloat32;
}

template <typename F>
bool Sym(void* lib, const char* name, F* out) {
    *out = reinterpret_cast<F>(dlsym(lib, name));
    return *out != nullptr;
}

}  // namespace

bool NcclP2p::Init(int rank, int nranks, Bootstrap* bs) {
    std::string path = EnvStr("BCCL_NCCL_LIBRARY", "libnccl.so.2");
    lib_ = dlopen(path.c_str(), RTLD_NOW | RTLD_GLOBAL);
    if (lib_ == nullptr) {
        LOG_ERROR("cannot load NCCL (%s): %s; set BCCL_NCCL_LIBRARY", path.c_str(), dlerror());
        return false;
    }
    bool ok = Sym(lib_, "ncclGetUniqueId", &g_fns.GetUniqueId) && Sym(lib_, "ncclCommInitRank", &g_fns.CommInitRank) &&
              Sym(lib_, "ncclCommDestroy", &g_fns.CommDestroy) && Sym(lib_, "ncclSend", &g_fns.Send) &&
              Sym(lib_, "ncclRecv", &g_fns.Recv) && Sym(lib_, "ncclGroupStart", &g_fns.GroupStart) &&
              Sym(lib_, "ncclGroupEnd", &g_fns.GroupEnd) && Sym(lib_, "ncclGetErrorString", &g_fns.GetErrorString) &&
              Sym(lib_, "ncclGetVersion", &g_fns.GetVersion);
    if (!ok) {
        LOG_ERROR("NCCL library lacks required symbols");
        return false;
    }
    int v = 0;
    g_fns.GetVersion(&v);
    snprintf(version_, sizeof(version_), "%d.%d.%d", v / 10000, (v / 100) % 100, v % 100);
    ncclUniqueId id;
    memset(&id, 0, sizeof(id));
    std::vector<uint8_t> blob;
    bool got = true;
    if (rank == 0) {
        got = g_fns.GetUniqueId(&id) == ncclSuccess;
        blob.assign(reinterpret_cast<uint8_t*>(&id), reinterpret_cast<uint8_t*>(&id) + sizeof(id));
        if (!got) blob.clear();
    }
    if (!bs->Broadcast(0, &blob) || blob.size() != sizeof(id)) {
        LOG_ERROR("rank %d: NCCL unique id exchange failed", rank);
        return false;
    }
    memcpy(&id, blob.data(), sizeof(id));
    ncclComm_t comm = nullptr;
    ncclResult_t r = g_fns.CommInitRank(&comm, nranks, id, rank);
    if (r != ncclSuccess) {
        LOG_ERROR("rank %d: ncclCommInitRank failed: %s", rank, g_fns.GetErrorString(r));
        return false;
    }
    comm_ = comm;
    return true;
}

void NcclP2p::Destroy() {
    if (comm_ != nullptr) {
        g_fns.CommDestroy(static_cast<ncclComm_t>(comm_));
        comm_ = nullptr;
    }
}

bool NcclP2p::Run(const std::vector<CollTask>& tasks, cudaStream_t stream) {
    if (tasks.empty()) return true;
    if (comm_ == nullptr) {
        LOG_ERROR("Send/Recv needs NCCL point-to-point, which is not initialised "
                  "(BCCL_P2P_NATIVE=1 runs it without NCCL)");
        return false;
    }
    ncclComm_t comm = static_cast<ncclComm_t>(comm_);
    g_fns.GroupStart();
    ncclResult_t r = ncclSuccess;
    for (const CollTask& t : tasks) {
        if (t.count == 0) continue;
        if (t.func == CollFunc::Send) {
            r = g_fns.Send(t.send_buf, t.count, ToNccl(t.dtype), t.peer, comm, stream);
        } else {
            r = g_fns.Recv(t.recv_buf, t.count, ToNccl(t.dtype), t.peer, comm, stream);
        }
        if (r != ncclSuccess) break;
    }
    ncclResult_t e = g_fns.GroupEnd();
    if (r != ncclSuccess || e != ncclSuccess) {
        LOG_ERROR("NCCL p2p failed: %s", g_fns.GetErrorString(r != ncclSuccess ? r : e));
        return false;
    }
    return true;
}

}  // namespace bccl
