#include "host/host_reduce.h"

#include <algorithm>

namespace bccl {
namespace hostmath {
namespace {

template <typename T, typename Acc, Acc (*Load)(T), T (*Store)(Acc)>
void ReduceT(ReduceOp op, void* dst, const void* const* srcs, int n, size_t count, int nranks, float scale,
             bool final) {
    T* d = static_cast<T*>(dst);
    for (size_t i = 0; i < count; ++i) {
        Acc acc = Load(static_cast<const T*>(srcs[0])[i]);
        for (int p = 1; p < n; ++p) {
            Acc v = Load(static_cast<const T*>(srcs[p])[i]);
            if (op == ReduceOp::MAX) acc = acc < v ? v : acc;
            else if (op == ReduceOp::MIN) acc = v < acc ? v : acc;
            else acc = static_cast<Acc>(acc + v);
        }
        if (final) {
            if (op == ReduceOp::AVG) acc = static_cast<Acc>(acc / static_cast<Acc>(nranks));
            if (scale != 1.0f && std::is_floating_point<Acc>::value) acc = static_cast<Acc>(acc * static_cast<Acc>(scale));
        }
        d[i] = Store(acc);
    }
}

template <typename T> T Ident(T v) { return v; }
int64_t LoadI64(int64_t v) { return v; }
// Integer sums wrap like two's complement (no signed-overflow UB).
int32_t WrapI32(int64_t v) { return static_cast<int32_t>(static_cast<uint32_t>(static_cast<uint64_t>(v))); }
int64_t LoadI32(int32_t v) { return v; }
uint64_t LoadI64u(int64_t v) { return static_cast<uint64_t>(v); }

}  // namespace

void Reduce(DataType dtype, ReduceOp op, void* dst, const void* const* srcs, int n, size_t count, int nranks,
            float scale, bool final) {
    switch (dtype) {
    case DataType::FLOAT32: ReduceT<float, float, Ident<float>, Ident<float>>(op, dst, srcs, n, count, nranks, scale, final); break;
    case DataType::FLOAT64: ReduceT<double, double, Ident<double>, Ident<double>>(op, dst, srcs, n, count, nranks, scale, final); break;
    case DataType::INT32: {
        // Accumulate in 64 bits so MAX/MIN compare correctly; SUM wraps at the store. AVG of
        // a wrapped sum is computed on the wrapped 32-bit value, as an int32 accumulator would.
        int32_t* d = static_cast<int32_t*>(dst);
        for (size_t i = 0; i < count; ++i) {
            int32_t acc = static_cast<const int32_t*>(srcs[0])[i];
            for (int p = 1; p < n; ++p) {
                int32_t v = static_cast<const int32_t*>(srcs[p])[i];
                if (op == ReduceOp::MAX) acc = std::max(acc, v);
                else if (op == ReduceOp::MIN) acc = std::min(acc, v);
                else acc = static_cast<int32_t>(static_cast<uint32_t>(acc) + static_cast<uint32_t>(v));
            }
            if (final && op == ReduceOp::AVG) acc /= nranks;
            d[i] = acc;
        }
        break;
    }
    case DataType::INT64: {
        int64_t* d = static_cast<int64_t*>(dst);
        for (size_t i = 0; i < count; ++i) {
            int64_t acc = static_cast<const int64_t*>(srcs[0])[i];
            for (int p = 1; p < n; ++p) {
                int64_t v = static_cast<const int64_t*>(srcs[p])[i];
                if (op == ReduceOp::MAX) acc = std::max(acc, v);
                else if (op == ReduceOp::MIN) acc = std::min(acc, v);
                else acc = static_cast<int64_t>(static_cast<uint64_t>(acc) + static_cast<uint64_t>(v));
            }
            if (final && op == ReduceOp::AVG) acc /= nranks;
            d[i] = acc;
        }
        break;
    }
    case DataType::BF16: ReduceT<uint16_t, float, Bf16ToFloat, FloatToBf16>(op, dst, srcs, n, count, nranks, scale, final); break;
    case DataType::FP16: ReduceT<uint16_t, float, HalfToFloat, FloatToHalf>(op, dst, srcs, n, count, nranks, scale, final); break;
    }
    (void)WrapI32;
    (void)LoadI32;
    (void)LoadI64;
    (void)LoadI64u;
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
