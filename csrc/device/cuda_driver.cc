#include "device/cuda_driver.h"

#include <mutex>

#include "core/logger.h"

namespace bccl {
namespace {

template <typename F>
bool Load(const char* name, F* fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess ||
        p == nullptr) {
        *fn = nullptr;
        return false;
    }
    *fn = reinterpret_cast<F>(p);
    return true;
}

}  // namespace

const DriverApi* Driver() {
    static DriverApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        bool ok = true;
        ok &= Load("cuMemCreate", &api.cuMemCreate);
        ok &= Load("cuMemRelease", &api.cuMemRelease);
        ok &= Load("cuMemExportToShareableHandle", &api.cuMemExportToShareableHandle);
        ok &= Load("cuMemImportFromShareableHandle", &api.cuMemImportFromShareableHandle);
        ok &= Load("cuMemAddressReserve", &api.cuMemAddressReserve);
        ok &= Load("cuMemAddressFree", &api.cuMemAddressFree);
        ok &= Load("cuMemMap", &api.cuMemMap);
        ok &= Load("cuMemUnmap", &api.cuMemUnmap);
        ok &= Load("cuMemSetAccess", &api.cuMemSetAccess);
        ok &= Load("cuMemGetAllocationGranularity", &api.cuMemGetAllocationGranularity);
        ok &= Load("cuDeviceGet", &api.cuDeviceGet);
        ok &= Load("cuDeviceGetAttribute", &api.cuDeviceGetAttribute);
        ok &= Load("cuGetErrorString", &api.cuGetErrorString);
        // Optional (multicast needs a recent driver; the tensor-map encoder is for TMA).
        Load("cuMulticastCreate", &api.cuMulticastCreate);
        Load("cuMulticastAddDevice", &api.cuMulticastAddDevice);
        Load("cuMulticastBindMem", &api.cuMulticastBindMem);
        Load("cuMulticastUnbind", &api.cuMulticastUnbind);
        Load("cuMulticastGetGranularity", &api.cuMulticastGetGranularity);
        Load("cuTensorMapEncodeTiled", &api.cuTensorMapEncodeTiled);
        Load("cuMemGetAddressRange", &api.cuMemGetAddressRange);
        Load("cuCtxGetCurrent", &api.cuCtxGetCurrent);
        api.loaded = ok;
        if (!ok) LOG_WARN("CUDA driver entry points unavailable (no driver?)");
    });
    return api.loaded ? &api : nullptr;
}

const char* DriverErrorString(CUresult r) {
    const DriverApi* d = Driver();
    const char* s = nullptr;
    if (d && d->cuGetErrorString) d->cuGetErrorString(r, &s);
    return s ? s : "unknown CUDA driver error";
}

}  // namespace bccl
