// select.cuh -- predicates and dtype dispatch for DeviceSelect /
// DevicePartition behind the C ABI (kernels:
// lcpp_b200::device::select_detail in include/lcpp_b200_device.cuh).
#pragma once

#include <cstring>
#include <limits>
#include <type_traits>

#include "../../include/lcpp_b200.h"
#include "../../include/lcpp_b200_device.cuh"
#include "common.cuh"

namespace lcpp {
namespace sel {

namespace sd = lcpp_b200::device::select_detail;
using lcpp_b200::device::NoValue;

// Internal clause kind: x % d == r for a divisor d whose magnitude is a
// power of two, evaluated with a mask instead of a division (a holds
// |d| - 1); C's remainder keeps the sign of x, so a negative signed x with
// low bits set has remainder (x & (|d| - 1)) - |d|.
constexpr int kClauseModPow2 = 100;

// x % (mask + 1) == r with C's remainder (sign of x), mask + 1 a power of two.
template <typename T>
__device__ __forceinline__ bool mod_pow2_eq(T x, T mask, T r)
{
    using W = typename std::make_unsigned<T>::type;
    W rem = W(x) & W(mask);
    if constexpr (std::is_signed<T>::value)
        if (x < T(0) && rem != W(0)) rem -= W(mask) + W(1);
    return T(rem) == r;
}

// AND of up to LCPP_MAX_CLAUSES clauses on a value of type T (the C ABI's
// stand-in for the reference's predicate lambdas).
template <typename T>
struct ClausePick {
    int count;
    int kind[LCPP_MAX_CLAUSES];
    int negate[LCPP_MAX_CLAUSES];
    T a[LCPP_MAX_CLAUSES];
    T b[LCPP_MAX_CLAUSES];
    __device__ __forceinline__ bool operator()(T x) const
    {
#pragma unroll
        for (int c = 0; c < LCPP_MAX_CLAUSES; ++c) {
            if (c >= count) break;
            bool r;
            switch (kind[c]) {
            case LCPP_CLAUSE_LT: r = x < a[c]; break;
            case LCPP_CLAUSE_LE: r = x <= a[c]; break;
            case LCPP_CLAUSE_GT: r = x > a[c]; break;
            case LCPP_CLAUSE_GE: r = x >= a[c]; break;
            case LCPP_CLAUSE_EQ: r = x == a[c]; break;
            case LCPP_CLAUSE_NE: r = x != a[c]; break;
            case LCPP_CLAUSE_MOD_EQ:
                if constexpr (std::is_integral<T>::value) r = x % a[c] == b[c];
                else r = false;
                break;
            case kClauseModPow2:
                if constexpr (std::is_integral<T>::value) r = mod_pow2_eq(x, a[c], b[c]);
                else r = false;
                break;
            default:
                if constexpr (std::is_integral<T>::value) r = (x & a[c]) != 0;
                else r = false;
                break;
            }
            if (negate[c]) r = !r;
            if (!r) return false;
        }
        return true;
    }
};

// The compaction kernels' form: every item of a thread at once (bit
// j * G + e), one dispatch per clause instead of one per item; found by
// argument-dependent lookup.
template <typename T, int C, int G>
__device__ __forceinline__ uint32_t select_mask(const ClausePick<T>& p, const T (&x)[C][G])
{
    auto each = [&](auto test) {
        uint32_t r = 0;
#pragma unroll
        for (int j = 0; j < C; ++j)
#pragma unroll
            for (int e = 0; e < G; ++e) r |= uint32_t(test(x[j][e])) << (j * G + e);
        return r;
    };
    uint32_t m = ~0u;
#pragma unroll
    for (int c = 0; c < LCPP_MAX_CLAUSES; ++c) {
        if (c >= p.count) break;
        const T a = p.a[c], b = p.b[c];
        uint32_t r = 0;
        switch (p.kind[c]) {
        case LCPP_CLAUSE_LT: r = each([&](T v) { return v < a; }); break;
        case LCPP_CLAUSE_LE: r = each([&](T v) { return v <= a; }); break;
        case LCPP_CLAUSE_GT: r = each([&](T v) { return v > a; }); break;
        case LCPP_CLAUSE_GE: r = each([&](T v) { return v >= a; }); break;
        case LCPP_CLAUSE_EQ: r = each([&](T v) { return v == a; }); break;
        case LCPP_CLAUSE_NE: r = each([&](T v) { return v != a; }); break;
        case LCPP_CLAUSE_MOD_EQ:
            if constexpr (std::is_integral<T>::value) r = each([&](T v) { return v % a == b; });
            break;
        case kClauseModPow2:
            if constexpr (std::is_integral<T>::value) r = each([&](T v) { return mod_pow2_eq(v, a, b); });
            break;
        default:
            if constexpr (std::is_integral<T>::value) r = each([&](T v) { return (v & a) != 0; });
            break;
        }
        if (p.negate[c]) r = ~r;
        m &= r;
    }
    return m;
}

template <typename T>
T from_bits(uint64_t bits)
{
    T v;
    if constexpr (sizeof(T) == 1) {
        const uint8_t b = uint8_t(bits);
        memcpy(&v, &b, 1);
    } else if constexpr (sizeof(T) == 4) {
        const uint32_t b = uint32_t(bits);
        memcpy(&v, &b, 4);
    } else {
        memcpy(&v, &bits, 8);
    }
    return v;
}

// Host-side checks and conversion; LCPP_ERR_INVALID_ARG for a bad clause.
template <typename T>
lcpp_status make_pick(const lcpp_clause* clauses, int count, ClausePick<T>& p)
{
    if (count < 0 || count > LCPP_MAX_CLAUSES || (count > 0 && !clauses)) return LCPP_ERR_INVALID_ARG;
    p = ClausePick<T>{};
    p.count = count;
    for (int c = 0; c < count; ++c) {
        const int k = clauses[c].kind;
        if (k < LCPP_CLAUSE_LT || k > LCPP_CLAUSE_BITS_ANY) return LCPP_ERR_INVALID_ARG;
        p.kind[c] = k;
        p.negate[c] = clauses[c].negate != 0;
        p.a[c] = from_bits<T>(clauses[c].a);
        p.b[c] = from_bits<T>(clauses[c].b);
        if (k == LCPP_CLAUSE_MOD_EQ || k == LCPP_CLAUSE_BITS_ANY) {
            if constexpr (!std::is_integral<T>::value) {
                return LCPP_ERR_INVALID_ARG;
            } else {
                if (k == LCPP_CLAUSE_MOD_EQ && p.a[c] == T(0)) return LCPP_ERR_INVALID_ARG;
                if (k == LCPP_CLAUSE_MOD_EQ) {
                    // |d| a power of two (the most negative value excluded): mask
                    using W = typename std::make_unsigned<T>::type;
                    const T d = p.a[c];
                    const bool most_negative = std::is_signed<T>::value && d == std::numeric_limits<T>::min();
                    const W mag = (std::is_signed<T>::value && d < T(0)) ? W(W(0) - W(d)) : W(d);
                    if (!most_negative && (mag & (mag - 1)) == 0) {
                        p.kind[c] = kClauseModPow2;
                        p.a[c] = T(mag - 1);
                        if (p.b[c] == T(0)) {
                            // remainder 0 for either sign exactly when the low bits are
                            // clear: !((x & (|d| - 1)) != 0)
                            p.kind[c] = LCPP_CLAUSE_BITS_ANY;
                            p.negate[c] = !p.negate[c];
                        }
                    }
                }
            }
        }
    }
    return LCPP_OK;
}

inline int flag_bytes(lcpp_dtype dt) { return dt == LCPP_U8 ? 1 : dtype_bytes(dt); }

inline lcpp_status status_of(cudaError_t e)
{
    if (e == cudaSuccess) return LCPP_OK;
    return e == cudaErrorInvalidValue ? LCPP_ERR_INVALID_ARG : LCPP_ERR_CUDA;
}

inline bool misaligned(const void* p, int bytes) { return p && reinterpret_cast<uintptr_t>(p) % unsigned(bytes); }

// Shared checks: counts, pointers, alignment, temp storage.
inline lcpp_status check(void* temp, size_t temp_bytes, const void* in, int item_bytes, uint32_t* num_selected,
                         uint64_t n, bool three)
{
    if (!item_bytes) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (!num_selected || misaligned(num_selected, 4)) return LCPP_ERR_INVALID_ARG;
    if (n > 0xffffffffull) return LCPP_ERR_INVALID_ARG;  // uint32 counts, as the reference
    if (n == 0) return LCPP_OK;
    if (!in || misaligned(in, item_bytes)) return LCPP_ERR_INVALID_ARG;
    if (!temp || (reinterpret_cast<uintptr_t>(temp) & (kTempAlign - 1))) return LCPP_ERR_INVALID_ARG;
    if (temp_bytes < sd::layout(n, three).total) return LCPP_ERR_TEMP_TOO_SMALL;
    return LCPP_OK;
}

// Items that are only moved: dispatched by size.
template <typename Fn>
lcpp_status with_bits_type(lcpp_dtype dt, Fn&& fn)
{
    switch (dtype_bytes(dt)) {
    case 4: return fn(uint32_t{});
    case 8: return fn(uint64_t{});
    default: return LCPP_ERR_UNSUPPORTED_DTYPE;
    }
}

// Items tested by a predicate: the exact type.
template <typename Fn>
lcpp_status with_value_type(lcpp_dtype dt, Fn&& fn)
{
    switch (dt) {
    case LCPP_U32: return fn(uint32_t{});
    case LCPP_I32: return fn(int32_t{});
    case LCPP_F32: return fn(float{});
    case LCPP_U64: return fn(uint64_t{});
    case LCPP_I64: return fn(int64_t{});
    case LCPP_F64: return fn(double{});
    default: return LCPP_ERR_UNSUPPORTED_DTYPE;
    }
}

// Flags tested for != 0: integers by their bits, floats by IEEE (-0.0 is 0).
template <typename Fn>
lcpp_status with_flag_nonzero_type(lcpp_dtype dt, Fn&& fn)
{
    switch (dt) {
    case LCPP_U8: return fn(uint8_t{});
    case LCPP_U32:
    case LCPP_I32: return fn(uint32_t{});
    case LCPP_U64:
    case LCPP_I64: return fn(uint64_t{});
    case LCPP_F32: return fn(float{});
    case LCPP_F64: return fn(double{});
    default: return LCPP_ERR_UNSUPPORTED_DTYPE;
    }
}

// Keys compared for equality (Unique): integers by bits, floats by IEEE.
template <typename Fn>
lcpp_status with_key_type(lcpp_dtype dt, Fn&& fn)
{
    switch (dt) {
    case LCPP_U32:
    case LCPP_I32: return fn(uint32_t{});
    case LCPP_U64:
    case LCPP_I64: return fn(uint64_t{});
    case LCPP_F32: return fn(float{});
    case LCPP_F64: return fn(double{});
    default: return LCPP_ERR_UNSUPPORTED_DTYPE;
    }
}

}  // namespace sel
}  // namespace lcpp
