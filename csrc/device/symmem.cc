#include "device/symmem.h"

#include <algorithm>
#include <cstring>
#include <unistd.h>

#include "core/bootstrap.h"
#include "core/env.h"
#include "core/fdpass.h"
#include "core/logger.h"
#include "device/cuda_driver.h"

namespace bccl {
namespace {

#define DRV_CHECK(call, what)                                                                  \
    do {                                                                                       \
        CUresult _r = (call);                                                                  \
        if (_r != CUDA_SUCCESS) {                                                              \
            LOG_ERROR("%s failed: %s (%d)", what, DriverErrorString(_r), static_cast<int>(_r)); \
            return false;                                                                      \
        }                                                                                      \
    } while (0)

size_t RoundUp(size_t x, size_t a) { return (x + a - 1) / a * a; }

CUmemAllocationProp MakeProp(int device) {
    CUmemAllocationProp prop;
    memset(&prop, 0, sizeof(prop));
    prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    prop.location.id = device;
    prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    return prop;
}

}  // namespace

bool SymmetricMemory::Init(int device, int rank, int nranks, Bootstrap* bs, FdPasser* fp, int timeout_ms,
                           bool want_multicast) {
    device_ = device;
    rank_ = rank;
    nranks_ = nranks;
    bs_ = bs;
    fp_ = fp;
    timeout_ms_ = timeout_ms;
    if (nranks > kMaxRanks) {
        LOG_ERROR("device communicator supports at most %d ranks per node (got %d)", kMaxRanks, nranks);
        return false;
    }
    const DriverApi* d = Driver();
    if (d == nullptr) {
        LOG_ERROR("CUDA driver not available");
        return false;
    }
    DRV_CHECK(d->cuDeviceGet(&cudev_, device), "cuDeviceGet");
    CUmemAllocationProp prop = MakeProp(device);
    DRV_CHECK(d->cuMemGetAllocationGranularity(&gran_, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED),
              "cuMemGetAllocationGranularity");
    int mc = 0;
    if (d->cuMulticastCreate != nullptr) {
        d->cuDeviceGetAttribute(&mc, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, cudev_);
    }
    bool mine = want_multicast && mc != 0 && nranks > 1 && !EnvFlag("BCCL_DISABLE_NVLS");
    if (mine) {
        CUmulticastObjectProp mp;
        memset(&mp, 0, sizeof(mp));
        mp.numDevices = static_cast<unsigned>(nranks);
        mp.size = gran_;
        mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
        if (d->cuMulticastGetGranularity(&mc_gran_, &mp, CU_MULTICAST_GRANULARITY_RECOMMENDED) != CUDA_SUCCESS) {
            mine = false;
        }
    }
    mc_supported_ = AgreeAll(mine);
    LOG_INFO("rank %d: symmetric memory on device %d, granularity %zu, multicast %s", rank, device, gran_,
             mc_supported_ ? "on" : "off");
    return true;
}

bool SymmetricMemory::AgreeAll(bool mine) {
    if (nranks_ == 1) return mine;
    std::vector<std::vector<uint8_t>> all;
    if (!bs_->AllGather({static_cast<uint8_t>(mine ? 1 : 0)}, &all)) return false;
    for (const auto& v : all)
        if (v.empty() || v[0] == 0) return false;
    return true;
}

bool SymmetricMemory::Alloc(size_t bytes, bool with_multicast, SymBuffer* out) {
    const DriverApi* d = Driver();
    *out = SymBuffer();
    const bool mc = with_multicast && mc_supported_;
    size_t g = mc ? std::max(gran_, mc_gran_) : gran_;
    out->bytes = RoundUp(std::max<size_t>(bytes, 1), g);
    const uint32_t tag = (++seq_) * 4u;
    CUmemAllocationProp prop = MakeProp(device_);
    bool ok = d->cuMemCreate(&out->local, out->bytes, &prop, 0) == CUDA_SUCCESS;
    if (!ok) LOG_ERROR("rank %d: cuMemCreate(%zu) failed", rank_, out->bytes);
    int my_fd = -1;
    if (ok && d->cuMemExportToShareableHandle(&my_fd, out->local, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0) !=
                  CUDA_SUCCESS) {
        LOG_ERROR("rank %d: exporting a memory handle failed", rank_);
        ok = false;
    }
    // Exchange handles (every rank sends before receiving; the fd passer stashes out-of-order arrivals).
    const bool drop = FaultActive("handle_drop", rank_);
    for (int p = 0; ok && p < nranks_; ++p) {
        if (p == rank_ || drop) continue;
        ok = fp_->SendFd(p, tag, my_fd, timeout_ms_);
    }
    if (my_fd >= 0) close(my_fd);
    for (int p = 0; ok && p < nranks_; ++p) {
        if (p == rank_) continue;
        int pfd = -1;
        if (!fp_->RecvFd(p, tag, &pfd, timeout_ms_)) {
            ok = false;
            break;
        }
        CUresult r = d->cuMemImportFromShareableHandle(&out->imported[p], reinterpret_cast<void*>(static_cast<intptr_t>(pfd)),
                                                       CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
        close(pfd);
        if (r != CUDA_SUCCESS) {
            LOG_ERROR("rank %d: importing the handle of rank %d failed: %s", rank_, p, DriverErrorString(r));
            ok = false;
        }
    }
    CUdeviceptr base = 0;
    if (ok) ok = d->cuMemAddressReserve(&base, out->bytes * nranks_, g, 0, 0) == CUDA_SUCCESS;
    if (ok) {
        out->base = reinterpret_cast<char*>(base);
        for (int p = 0; ok && p < nranks_; ++p) {
            CUmemGenericAllocationHandle h = (p == rank_) ? out->local : out->imported[p];
            ok = d->cuMemMap(base + out->bytes * p, out->bytes, 0, h, 0) == CUDA_SUCCESS;
            out->ptr[p] = out->base + out->bytes * p;
        }
        CUmemAccessDesc acc;
        memset(&acc, 0, sizeof(acc));
        acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
        acc.location.id = device_;
        acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
        if (ok) ok = d->cuMemSetAccess(base, out->bytes * nranks_, &acc, 1) == CUDA_SUCCESS;
        if (!ok) LOG_ERROR("rank %d: mapping peer memory failed", rank_);
    }
    if (ok && cudaMemset(out->ptr[rank_], 0, out->bytes) != cudaSuccess) ok = false;
    if (ok && cudaDeviceSynchronize() != cudaSuccess) ok = false;
    out->valid = true;  // so Free can release what exists
    if (!AgreeAll(ok)) {
        Free(out);
        LOG_ERROR("rank %d: symmetric allocation of %zu bytes failed on some rank", rank_, bytes);
        return false;
    }
    if (mc && !SetupMulticast(out, tag + 1)) {
        LOG_WARN("rank %d: NVLS multicast setup failed; continuing without it", rank_);
    }
    return true;
}

bool SymmetricMemory::SetupMulticast(SymBuffer* buf, uint32_t tag) {
    const DriverApi* d = Driver();
    bool ok = true;
    CUmulticastObjectProp mp;
    memset(&mp, 0, sizeof(mp));
    mp.numDevices = static_cast<unsigned>(nranks_);
    mp.size = buf->bytes;
    mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    if (rank_ == 0) {
        ok = d->cuMulticastCreate(&buf->mc_handle, &mp) == CUDA_SUCCESS;
        int fd = -1;
        if (ok) ok = d->cuMemExportToShareableHandle(&fd, buf->mc_handle, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0) ==
                     CUDA_SUCCESS;
        // Peers always get a message (fd -1 is not sendable, so on failure we send nothing and
        // the agreement below reports it).
        for (int p = 1; ok && p < nranks_; ++p) ok = fp_->SendFd(p, tag, fd, timeout_ms_);
        if (fd >= 0) close(fd);
    }
    if (!AgreeAll(ok)) return false;
    if (rank_ != 0) {
        int fd = -1;
        ok = fp_->RecvFd(0, tag, &fd, timeout_ms_);
        if (ok) {
            ok = d->cuMemImportFromShareableHandle(&buf->mc_handle, reinterpret_cast<void*>(static_cast<intptr_t>(fd)),
                                                   CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR) == CUDA_SUCCESS;
            close(fd);
        }
    }
    if (ok) ok = d->cuMulticastAddDevice(buf->mc_handle, cudev_) == CUDA_SUCCESS;
    // Every device must be added before any memory is bound.
    if (!AgreeAll(ok)) return false;
    ok = d->cuMulticastBindMem(buf->mc_handle, 0, buf->local, 0, buf->bytes, 0) == CUDA_SUCCESS;
    CUdeviceptr mc = 0;
    if (ok) ok = d->cuMemAddressReserve(&mc, buf->bytes, mc_gran_, 0, 0) == CUDA_SUCCESS;
    if (ok) ok = d->cuMemMap(mc, buf->bytes, 0, buf->mc_handle, 0) == CUDA_SUCCESS;
    if (ok) {
        CUmemAccessDesc acc;
        memset(&acc, 0, sizeof(acc));
        acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
        acc.location.id = device_;
        acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
        ok = d->cuMemSetAccess(mc, buf->bytes, &acc, 1) == CUDA_SUCCESS;
    }
    if (ok) buf->mc = reinterpret_cast<char*>(mc);
    if (!AgreeAll(ok)) {
        if (buf->mc) {
            d->cuMemUnmap(mc, buf->bytes);
            d->cuMemAddressFree(mc, buf->bytes);
            buf->mc = nullptr;
        }
        return false;
    }
    return true;
}

void SymmetricMemory::Free(SymBuffer* buf) {
    if (!buf->valid) return;
    const DriverApi* d = Driver();
    if (buf->mc) {
        d->cuMemUnmap(reinterpret_cast<CUdeviceptr>(buf->mc), buf->bytes);
        d->cuMemAddressFree(reinterpret_cast<CUdeviceptr>(buf->mc), buf->bytes);
        if (d->cuMulticastUnbind) d->cuMulticastUnbind(buf->mc_handle, cudev_, 0, buf->bytes);
        buf->mc = nullptr;
    }
    if (buf->mc_handle) {
        d->cuMemRelease(buf->mc_handle);
        buf->mc_handle = 0;
    }
    if (buf->base) {
        for (int p = 0; p < nranks_; ++p)
            if (buf->ptr[p]) d->cuMemUnmap(reinterpret_cast<CUdeviceptr>(buf->ptr[p]), buf->bytes);
        d->cuMemAddressFree(reinterpret_cast<CUdeviceptr>(buf->base), buf->bytes * nranks_);
    }
    for (int p = 0; p < kMaxRanks; ++p) {
        if (buf->imported[p]) d->cuMemRelease(buf->imported[p]);
        buf->imported[p] = 0;
    }
    if (buf->local) d->cuMemRelease(buf->local);
    *buf = SymBuffer();
}

}  // namespace bccl
