// reduce_by_key.cu -- DeviceReduce::ReduceByKey behind the C ABI
// (src/lcpp/device/device_reduce.h:437-491); the kernel is
// lcpp_b200::device::bykey_detail::by_key_kernel in its run-counting form
// (include/lcpp_b200_device.cuh), instantiated for key equality by == and
// the Sum / Min / Max operators.
#include "by_key.cuh"

namespace bd = lcpp::bykey::bd;

extern "C" {

lcpp_status lcpp_reduce_by_key_temp_bytes(lcpp_dtype key_dtype, lcpp_dtype value_dtype, uint64_t num_items,
                                          size_t* temp_bytes)
{
    if (!temp_bytes) return LCPP_ERR_INVALID_ARG;
    if (!lcpp::dtype_bytes(key_dtype) || !lcpp::dtype_bytes(value_dtype)) return LCPP_ERR_UNSUPPORTED_DTYPE;
    *temp_bytes = lcpp_b200::device::by_key_temp_bytes(num_items, size_t(lcpp::dtype_bytes(value_dtype)));
    return LCPP_OK;
}

lcpp_status lcpp_reduce_by_key(void* temp, size_t temp_bytes, const void* d_keys_in, const void* d_values_in,
                               void* d_unique_out, void* d_aggregates_out, uint32_t* d_num_runs_out,
                               uint64_t num_items, lcpp_op op, lcpp_dtype key_dtype, lcpp_dtype value_dtype,
                               lcpp_stream_t stream)
{
    using namespace lcpp;
    using namespace lcpp::bykey;
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (!d_num_runs_out || reinterpret_cast<uintptr_t>(d_num_runs_out) % 4) return LCPP_ERR_INVALID_ARG;
    if (num_items > 0xffffffffull) return LCPP_ERR_INVALID_ARG;  // uint32 run count, as the reference
    const lcpp_status st = check_common(temp, temp_bytes, d_keys_in, d_values_in, num_items, key_dtype, value_dtype);
    if (st != LCPP_OK) return st;
    if (op != LCPP_OP_SUM && op != LCPP_OP_MIN && op != LCPP_OP_MAX) return LCPP_ERR_INVALID_ARG;
    if (num_items == 0)  // the reference writes 0 runs and nothing else (device_reduce.h:449-458)
        return cudaMemsetAsync(d_num_runs_out, 0, 4, s) == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
    const int kb = dtype_bytes(key_dtype), vb = dtype_bytes(value_dtype);
    if (!d_unique_out || !d_aggregates_out || reinterpret_cast<uintptr_t>(d_unique_out) % kb ||
        reinterpret_cast<uintptr_t>(d_aggregates_out) % vb || d_unique_out == d_keys_in)
        return LCPP_ERR_INVALID_ARG;
    return with_key_type(key_dtype, [&](auto k) {
        using K = decltype(k);
        return with_value_type(value_dtype, [&](auto v) {
            using V = decltype(v);
            return with_op(op, [&](auto fn) {
                diag::KernelTimer timer(7 /* LCPP_KERNEL_BY_KEY */, num_items, s);
                return status_of(bd::launch<true>(temp, temp_bytes, static_cast<const K*>(d_keys_in),
                                                  static_cast<const V*>(d_values_in), static_cast<V*>(d_aggregates_out),
                                                  static_cast<K*>(d_unique_out), d_num_runs_out, num_items,
                                                  bd::kModeReduce, V{}, lcpp_b200::device::EqualTo{}, fn, s));
            });
        });
    });
}

}  // extern "C"
