// ops.cuh -- binary operators and identities shared by scan and reduce.
#pragma once

#include <cfloat>
#include <climits>
#include <cstdint>

#include "common.cuh"

namespace lcpp {

// Sum / Min / Max as the reference's SumOp / MinOp / MaxOp
// (src/lcpp/common/thread_operators.h:49-75).  Integer sums are computed in
// the unsigned type of the same width so that overflow wraps (two's
// complement) instead of being undefined.
template <typename T>
struct WrapType { using type = T; };
template <> struct WrapType<int32_t> { using type = uint32_t; };
template <> struct WrapType<int64_t> { using type = uint64_t; };

struct SumOp {
    template <typename T>
    __host__ __device__ __forceinline__ T operator()(T a, T b) const
    {
        using W = typename WrapType<T>::type;
        return T(W(a) + W(b));
    }
};
struct MinOp {
    template <typename T>
    __host__ __device__ __forceinline__ T operator()(T a, T b) const { return b < a ? b : a; }
};
struct MaxOp {
    template <typename T>
    __host__ __device__ __forceinline__ T operator()(T a, T b) const { return a < b ? b : a; }
};

// Padding values for out-of-range lanes: they must not change any result.
template <typename T> __host__ __device__ __forceinline__ T lowest_value();
template <typename T> __host__ __device__ __forceinline__ T highest_value();
template <> __host__ __device__ __forceinline__ int32_t lowest_value<int32_t>() { return INT32_MIN; }
template <> __host__ __device__ __forceinline__ int32_t highest_value<int32_t>() { return INT32_MAX; }
template <> __host__ __device__ __forceinline__ uint32_t lowest_value<uint32_t>() { return 0u; }
template <> __host__ __device__ __forceinline__ uint32_t highest_value<uint32_t>() { return UINT32_MAX; }
template <> __host__ __device__ __forceinline__ int64_t lowest_value<int64_t>() { return INT64_MIN; }
template <> __host__ __device__ __forceinline__ int64_t highest_value<int64_t>() { return INT64_MAX; }
template <> __host__ __device__ __forceinline__ uint64_t lowest_value<uint64_t>() { return 0ull; }
template <> __host__ __device__ __forceinline__ uint64_t highest_value<uint64_t>() { return UINT64_MAX; }
template <> __host__ __device__ __forceinline__ float lowest_value<float>() { return -__builtin_huge_valf(); }
template <> __host__ __device__ __forceinline__ float highest_value<float>() { return __builtin_huge_valf(); }
template <> __host__ __device__ __forceinline__ double lowest_value<double>() { return -__builtin_huge_val(); }
template <> __host__ __device__ __forceinline__ double highest_value<double>() { return __builtin_huge_val(); }

template <typename Op, typename T> struct Identity;
template <typename T> struct Identity<SumOp, T> { __host__ __device__ static T value() { return T(0); } };
template <typename T> struct Identity<MinOp, T> { __host__ __device__ static T value() { return highest_value<T>(); } };
template <typename T> struct Identity<MaxOp, T> { __host__ __device__ static T value() { return lowest_value<T>(); } };

// Bit-preserving shuffles for 4- and 8-byte values of any type.
template <typename T>
__device__ __forceinline__ T shfl_up(T v, int delta)
{
    return __shfl_up_sync(0xffffffffu, v, delta);
}
template <typename T>
__device__ __forceinline__ T shfl_idx(T v, int lane)
{
    return __shfl_sync(0xffffffffu, v, lane);
}
template <typename T>
__device__ __forceinline__ T shfl_xor(T v, int mask)
{
    return __shfl_xor_sync(0xffffffffu, v, mask);
}

// Inclusive warp scan (Hillis-Steele over lanes, left operand = lower lane).
template <typename T, typename Op>
__device__ __forceinline__ T warp_inclusive_scan(T v, Op op)
{
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const T y = shfl_up(v, o);
        if (lane >= o) v = op(y, v);
    }
    return v;
}

// Warp reduction with a fixed butterfly tree (deterministic).
template <typename T, typename Op>
__device__ __forceinline__ T warp_reduce(T v, Op op)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, shfl_xor(v, o));
    return v;
}

}  // namespace lcpp
