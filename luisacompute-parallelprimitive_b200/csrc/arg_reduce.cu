// arg_reduce.cu -- DeviceReduce::ArgMin / ArgMax behind the C ABI.
//
// Replaces DeviceReduce::ArgMin / ArgMax (src/lcpp/device/device_reduce.h:
// 310-436): the minimum (maximum) value and the first index holding it
// (ArgMinOp / ArgMaxOp, src/lcpp/common/thread_operators.h:19-47); empty
// input writes max() (lowest()) and index 1 (device_reduce.h:318-323).  The
// reference builds an index-value pair array in temp storage and reduces it
// with its generic multi-level Reduce; here one pass of
// lcpp_b200::device::arg_extremum_kernel (include/lcpp_b200_device.cuh,
// shared with the comparator overloads) keeps each thread's best
// (value, index) while streaming its chunk once, so the only DRAM traffic is
// the input.
#include "../../include/lcpp_b200.h"
#include "../../include/lcpp_b200_device.cuh"
#include "common.cuh"

namespace lcpp {
namespace argred {

using lcpp_b200::device::NaturalOrder;
namespace ad = lcpp_b200::device::arg_detail;

template <typename T, bool IS_MIN>
lcpp_status launch(void* temp, size_t temp_bytes, const void* in, void* out_v, uint32_t* out_i, uint64_t n,
                   cudaStream_t stream)
{
    diag::KernelTimer timer(6 /* LCPP_KERNEL_ARG_REDUCE */, n, stream);
    const cudaError_t e = lcpp_b200::device::arg_extremum<IS_MIN>(temp, temp_bytes, static_cast<const T*>(in),
                                                                  static_cast<T*>(out_v), out_i, n, NaturalOrder{},
                                                                  stream);
    return e == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
}

template <bool IS_MIN>
lcpp_status run(void* temp, size_t temp_bytes, const void* in, void* out_v, uint32_t* out_i, uint64_t n,
                lcpp_dtype dt, cudaStream_t stream)
{
    diag::Range nvtx_range("lcpp DeviceReduce::ArgMin/ArgMax");
    const int tb = dtype_bytes(dt);
    if (!tb) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (!out_v || !out_i) return LCPP_ERR_INVALID_ARG;
    if (n > 0xffffffffull) return LCPP_ERR_INVALID_ARG;  // uint32 indices, as the reference
    if (reinterpret_cast<uintptr_t>(out_v) % tb || reinterpret_cast<uintptr_t>(out_i) % 4) return LCPP_ERR_INVALID_ARG;
    if (n > 0) {
        if (!in || reinterpret_cast<uintptr_t>(in) % tb) return LCPP_ERR_INVALID_ARG;
        if (!temp || (reinterpret_cast<uintptr_t>(temp) & (kTempAlign - 1))) return LCPP_ERR_INVALID_ARG;
        if (temp_bytes < ad::layout(n, device_sm_count()).total) return LCPP_ERR_TEMP_TOO_SMALL;
    }
    switch (dt) {
    case LCPP_U32: return launch<uint32_t, IS_MIN>(temp, temp_bytes, in, out_v, out_i, n, stream);
    case LCPP_I32: return launch<int32_t, IS_MIN>(temp, temp_bytes, in, out_v, out_i, n, stream);
    case LCPP_F32: return launch<float, IS_MIN>(temp, temp_bytes, in, out_v, out_i, n, stream);
    case LCPP_U64: return launch<uint64_t, IS_MIN>(temp, temp_bytes, in, out_v, out_i, n, stream);
    case LCPP_I64: return launch<int64_t, IS_MIN>(temp, temp_bytes, in, out_v, out_i, n, stream);
    case LCPP_F64: return launch<double, IS_MIN>(temp, temp_bytes, in, out_v, out_i, n, stream);
    default: return LCPP_ERR_UNSUPPORTED_DTYPE;
    }
}

}  // namespace argred
}  // namespace lcpp

extern "C" lcpp_status lcpp_reduce_arg_temp_bytes(lcpp_dtype dtype, uint64_t num_items, size_t* temp_bytes)
{
    if (!temp_bytes) return LCPP_ERR_INVALID_ARG;
    if (!lcpp::dtype_bytes(dtype)) return LCPP_ERR_UNSUPPORTED_DTYPE;
    *temp_bytes = num_items ? lcpp::argred::ad::layout(num_items, lcpp::device_sm_count()).total : 0;
    return LCPP_OK;
}

extern "C" lcpp_status lcpp_reduce_argmin(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                                          uint32_t* d_index_out, uint64_t num_items, lcpp_dtype dtype,
                                          lcpp_stream_t stream)
{
    return lcpp::argred::run<true>(temp, temp_bytes, d_in, d_out, d_index_out, num_items, dtype,
                                   reinterpret_cast<cudaStream_t>(stream));
}

extern "C" lcpp_status lcpp_reduce_argmax(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                                          uint32_t* d_index_out, uint64_t num_items, lcpp_dtype dtype,
                                          lcpp_stream_t stream)
{
    return lcpp::argred::run<false>(temp, temp_bytes, d_in, d_out, d_index_out, num_items, dtype,
                                    reinterpret_cast<cudaStream_t>(stream));
}
