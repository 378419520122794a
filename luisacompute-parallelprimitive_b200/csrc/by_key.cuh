// by_key.cuh -- dtype / operator dispatch for the by-key scans and
// ReduceByKey (kernels: lcpp_b200::device::bykey_detail in
// include/lcpp_b200_device.cuh).
#pragma once

#include "../../include/lcpp_b200.h"
#include "../../include/lcpp_b200_device.cuh"
#include "common.cuh"
#include "ops.cuh"

namespace lcpp {
namespace bykey {

namespace bd = lcpp_b200::device::bykey_detail;

// Keys are only compared for equality: signed and unsigned integers of one
// width compare alike, floats keep IEEE equality (-0 == +0, NaN != NaN).
template <typename F>
lcpp_status with_key_type(lcpp_dtype kdt, F&& f)
{
    switch (kdt) {
    case LCPP_U32:
    case LCPP_I32: return f(uint32_t{});
    case LCPP_U64:
    case LCPP_I64: return f(uint64_t{});
    case LCPP_F32: return f(float{});
    case LCPP_F64: return f(double{});
    default: return LCPP_ERR_UNSUPPORTED_DTYPE;
    }
}

template <typename F>
lcpp_status with_value_type(lcpp_dtype vdt, F&& f)
{
    switch (vdt) {
    case LCPP_U32: return f(uint32_t{});
    case LCPP_I32: return f(int32_t{});
    case LCPP_F32: return f(float{});
    case LCPP_U64: return f(uint64_t{});
    case LCPP_I64: return f(int64_t{});
    case LCPP_F64: return f(double{});
    default: return LCPP_ERR_UNSUPPORTED_DTYPE;
    }
}

template <typename F>
lcpp_status with_op(lcpp_op op, F&& f)
{
    switch (op) {
    case LCPP_OP_SUM: return f(SumOp{});
    case LCPP_OP_MIN: return f(MinOp{});
    case LCPP_OP_MAX: return f(MaxOp{});
    default: return LCPP_ERR_INVALID_ARG;
    }
}

inline lcpp_status status_of(cudaError_t e)
{
    if (e == cudaSuccess) return LCPP_OK;
    return e == cudaErrorInvalidValue ? LCPP_ERR_INVALID_ARG : LCPP_ERR_CUDA;
}

// Checks shared by the by-key entry points (before any device work).
inline lcpp_status check_common(void* temp, size_t temp_bytes, const void* keys, const void* values, uint64_t n,
                                lcpp_dtype kdt, lcpp_dtype vdt)
{
    const int kb = dtype_bytes(kdt), vb = dtype_bytes(vdt);
    if (!kb || !vb) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (n == 0) return LCPP_OK;
    if (!keys || !values || reinterpret_cast<uintptr_t>(keys) % kb || reinterpret_cast<uintptr_t>(values) % vb)
        return LCPP_ERR_INVALID_ARG;
    if (!temp || (reinterpret_cast<uintptr_t>(temp) & (kTempAlign - 1))) return LCPP_ERR_INVALID_ARG;
    if (temp_bytes < bd::layout(n, size_t(vb)).total) return LCPP_ERR_TEMP_TOO_SMALL;
    if (bd::layout(n, size_t(vb)).tiles > 0xffffffffull) return LCPP_ERR_INVALID_ARG;
    return LCPP_OK;
}

}  // namespace bykey
}  // namespace lcpp
