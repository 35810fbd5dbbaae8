// NVTX ranges around the library's host entry points, so a timeline profiler shows each
// collective (or group batch) and each fused TP op by name. NVTX3 is header-only and costs a
// branch when no profiler is attached; BCCL_NVTX=0 turns the ranges off.
#pragma once

#include <nvtx3/nvToolsExt.h>

#include <cstdlib>

namespace bccl {

inline bool NvtxEnabled() {
    static const bool on = [] {
        const char* v = std::getenv("BCCL_NVTX");
        return v == nullptr || v[0] != '0';
    }();
    return on;
}

class NvtxRange {
public:
    explicit NvtxRange(const char* name) : on_(NvtxEnabled()) {
        if (on_) nvtxRangePushA(name);
    }
    ~NvtxRange() {
        if (on_) nvtxRangePop();
    }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;

private:
    bool on_;
};

}  // namespace bccl
