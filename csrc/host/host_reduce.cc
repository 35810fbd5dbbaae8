#include "host/host_reduce.h"

#include <algorithm>
#include <type_traits>

namespace bccl {
namespace hostmath {
namespace {

// Element-wise combiners; the accumulation type is the widened type (fp32 for bf16/fp16).
// Integer sums wrap like two's complement (computed in the unsigned type: no signed-overflow UB).
struct SumOp {
    template <typename A> static A Apply(A a, A b) { return a + b; }
    static int32_t Apply(int32_t a, int32_t b) {
        return static_cast<int32_t>(static_cast<uint32_t>(a) + static_cast<uint32_t>(b));
    }
    static int64_t Apply(int64_t a, int64_t b) {
        return static_cast<int64_t>(static_cast<uint64_t>(a) + static_cast<uint64_t>(b));
    }
};
struct MaxOp {
    template <typename A> static A Apply(A a, A b) { return a < b ? b : a; }
};
struct MinOp {
    template <typename A> static A Apply(A a, A b) { return b < a ? b : a; }
};

template <typename T> struct Plain {
    using Acc = T;
    static T Load(T v) { return v; }
    static T Store(T v) { return v; }
};
struct Bf16 {
    using Acc = float;
    static float Load(uint16_t v) { return Bf16ToFloat(v); }
    static uint16_t Store(float v) { return FloatToBf16(v); }
};
struct Half {
    using Acc = float;
    static float Load(uint16_t v) { return HalfToFloat(v); }
    static uint16_t Store(float v) { return FloatToHalf(v); }
};

// Blocked reduction: a block of kBlock accumulators stays in L1 while every source is folded in
// with one branch-free pass, so each pass is a plain loop over contiguous memory that the
// compiler vectorises (the operator and the type are template parameters, not per-element
// branches). AVG divides the final sum by the rank count (integer division for integers, as in
// the reference); a scale applies to floating-point results only.
template <typename T, typename Conv, typename Op>
void ReduceBlocked(void* dst, const void* const* srcs, int n, size_t count, int nranks, float scale, bool avg,
                   bool final) {
    using Acc = typename Conv::Acc;
    constexpr size_t kBlock = 1024;
    alignas(64) Acc acc[kBlock];
    T* d = static_cast<T*>(dst);
    const bool fp = std::is_floating_point<Acc>::value;
    const bool do_avg = final && avg, do_scale = final && fp && scale != 1.0f;
    for (size_t base = 0; base < count; base += kBlock) {
        const size_t m = std::min(kBlock, count - base);
        const T* s0 = static_cast<const T*>(srcs[0]) + base;
        for (size_t i = 0; i < m; ++i) acc[i] = Conv::Load(s0[i]);
        for (int p = 1; p < n; ++p) {
            const T* sp = static_cast<const T*>(srcs[p]) + base;
            for (size_t i = 0; i < m; ++i) acc[i] = Op::Apply(acc[i], Conv::Load(sp[i]));
        }
        if (do_avg) {
            const Acc div = static_cast<Acc>(nranks);
            for (size_t i = 0; i < m; ++i) acc[i] = static_cast<Acc>(acc[i] / div);
        }
        if (do_scale) {
            const Acc sc = static_cast<Acc>(scale);
            for (size_t i = 0; i < m; ++i) acc[i] = static_cast<Acc>(acc[i] * sc);
        }
        T* dp = d + base;
        for (size_t i = 0; i < m; ++i) dp[i] = Conv::Store(acc[i]);
    }
}

template <typename T, typename Conv>
void ReduceType(ReduceOp op, void* dst, const void* const* srcs, int n, size_t count, int nranks, float scale,
                bool final) {
    switch (op) {
    case ReduceOp::MAX: ReduceBlocked<T, Conv, MaxOp>(dst, srcs, n, count, nranks, scale, false, final); break;
    case ReduceOp::MIN: ReduceBlocked<T, Conv, MinOp>(dst, srcs, n, count, nranks, scale, false, final); break;
    case ReduceOp::AVG: ReduceBlocked<T, Conv, SumOp>(dst, srcs, n, count, nranks, scale, true, final); break;
    default: ReduceBlocked<T, Conv, SumOp>(dst, srcs, n, count, nranks, scale, false, final); break;
    }
}

}  // namespace

void Reduce(DataType dtype, ReduceOp op, void* dst, const void* const* srcs, int n, size_t count, int nranks,
            float scale, bool final) {
    switch (dtype) {
    case DataType::FLOAT32: ReduceType<float, Plain<float>>(op, dst, srcs, n, count, nranks, scale, final); break;
    case DataType::FLOAT64: ReduceType<double, Plain<double>>(op, dst, srcs, n, count, nranks, scale, final); break;
    case DataType::INT32: ReduceType<int32_t, Plain<int32_t>>(op, dst, srcs, n, count, nranks, scale, final); break;
    case DataType::INT64: ReduceType<int64_t, Plain<int64_t>>(op, dst, srcs, n, count, nranks, scale, final); break;
    case DataType::BF16: ReduceType<uint16_t, Bf16>(op, dst, srcs, n, count, nranks, scale, final); break;
    case DataType::FP16: ReduceType<uint16_t, Half>(op, dst, srcs, n, count, nranks, scale, final); break;
    }
}

void Finish(DataType dtype, ReduceOp op, void* dst, const void* src, size_t count, int nranks, float scale) {
    if (op != ReduceOp::AVG && (scale == 1.0f || !IsFloating(dtype))) {
        if (dst != src) memmove(dst, src, count * DataTypeSize(dtype));
        return;
    }
    const void* srcs[1] = {src};
    Reduce(dtype, op, dst, srcs, 1, count, nranks, scale, true);
}

}  // namespace hostmath
}  // namespace bccl
