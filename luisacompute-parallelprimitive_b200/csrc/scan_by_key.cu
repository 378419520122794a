// scan_by_key.cu -- DeviceScan::ExclusiveScanByKey / InclusiveScanByKey
// (and the ...SumByKey forms) behind the C ABI; the kernel is
// lcpp_b200::device::bykey_detail::by_key_kernel (include/lcpp_b200_device.cuh),
// instantiated here for key equality by == and the Sum / Min / Max operators.
#include "by_key.cuh"

namespace lcpp {
namespace bykey {

lcpp_status scan(void* temp, size_t temp_bytes, const void* keys, const void* vin, void* vout, uint64_t n,
                 lcpp_op op, const void* init, int mode, lcpp_dtype kdt, lcpp_dtype vdt, cudaStream_t stream)
{
    const lcpp_status s = check_common(temp, temp_bytes, keys, vin, n, kdt, vdt);
    if (s != LCPP_OK || n == 0) return s;
    const int vb = dtype_bytes(vdt);
    if (!vout || reinterpret_cast<uintptr_t>(vout) % vb) return LCPP_ERR_INVALID_ARG;
    if (mode != bd::kModeInclusive && !init) return LCPP_ERR_INVALID_ARG;
    return with_key_type(kdt, [&](auto k) {
        using K = decltype(k);
        return with_value_type(vdt, [&](auto v) {
            using V = decltype(v);
            V init_v{};
            if (mode != bd::kModeInclusive) memcpy(&init_v, init, sizeof(V));
            return with_op(op, [&](auto fn) {
                diag::KernelTimer timer(7 /* LCPP_KERNEL_BY_KEY */, n, stream);
                return status_of(bd::launch<false>(temp, temp_bytes, static_cast<const K*>(keys),
                                                   static_cast<const V*>(vin), static_cast<V*>(vout),
                                                   static_cast<K*>(nullptr), nullptr, n, mode, init_v,
                                                   lcpp_b200::device::EqualTo{}, fn, stream));
            });
        });
    });
}

}  // namespace bykey
}  // namespace lcpp

using lcpp::bykey::scan;
namespace bd = lcpp::bykey::bd;

extern "C" {

lcpp_status lcpp_scan_by_key_temp_bytes(lcpp_dtype key_dtype, lcpp_dtype value_dtype, uint64_t num_items,
                                        size_t* temp_bytes)
{
    if (!temp_bytes) return LCPP_ERR_INVALID_ARG;
    if (!lcpp::dtype_bytes(key_dtype) || !lcpp::dtype_bytes(value_dtype)) return LCPP_ERR_UNSUPPORTED_DTYPE;
    *temp_bytes = lcpp_b200::device::by_key_temp_bytes(num_items, size_t(lcpp::dtype_bytes(value_dtype)));
    return LCPP_OK;
}

lcpp_status lcpp_scan_exclusive_by_key(void* temp, size_t temp_bytes, const void* d_keys_in,
                                       const void* d_values_in, void* d_values_out, uint64_t num_items,
                                       lcpp_op op, const void* init, lcpp_dtype key_dtype,
                                       lcpp_dtype value_dtype, lcpp_stream_t stream)
{
    return scan(temp, temp_bytes, d_keys_in, d_values_in, d_values_out, num_items, op, init, bd::kModeExclusive,
                key_dtype, value_dtype, reinterpret_cast<cudaStream_t>(stream));
}

lcpp_status lcpp_scan_inclusive_by_key(void* temp, size_t temp_bytes, const void* d_keys_in,
                                       const void* d_values_in, void* d_values_out, uint64_t num_items,
                                       lcpp_op op, lcpp_dtype key_dtype, lcpp_dtype value_dtype,
                                       lcpp_stream_t stream)
{
    return scan(temp, temp_bytes, d_keys_in, d_values_in, d_values_out, num_items, op, nullptr,
                bd::kModeInclusive, key_dtype, value_dtype, reinterpret_cast<cudaStream_t>(stream));
}

lcpp_status lcpp_scan_inclusive_by_key_init(void* temp, size_t temp_bytes, const void* d_keys_in,
                                            const void* d_values_in, void* d_values_out, uint64_t num_items,
                                            lcpp_op op, const void* init, lcpp_dtype key_dtype,
                                            lcpp_dtype value_dtype, lcpp_stream_t stream)
{
    return scan(temp, temp_bytes, d_keys_in, d_values_in, d_values_out, num_items, op, init,
                bd::kModeInclusiveInit, key_dtype, value_dtype, reinterpret_cast<cudaStream_t>(stream));
}

lcpp_status lcpp_scan_exclusive_sum_by_key(void* temp, size_t temp_bytes, const void* d_keys_in,
                                           const void* d_values_in, void* d_values_out, uint64_t num_items,
                                           lcpp_dtype key_dtype, lcpp_dtype value_dtype, lcpp_stream_t stream)
{
    const uint64_t zero = 0;  // 0 of every value type
    return scan(temp, temp_bytes, d_keys_in, d_values_in, d_values_out, num_items, LCPP_OP_SUM, &zero,
                bd::kModeExclusive, key_dtype, value_dtype, reinterpret_cast<cudaStream_t>(stream));
}

lcpp_status lcpp_scan_inclusive_sum_by_key(void* temp, size_t temp_bytes, const void* d_keys_in,
                                           const void* d_values_in, void* d_values_out, uint64_t num_items,
                                           lcpp_dtype key_dtype, lcpp_dtype value_dtype, lcpp_stream_t stream)
{
    return scan(temp, temp_bytes, d_keys_in, d_values_in, d_values_out, num_items, LCPP_OP_SUM, nullptr,
                bd::kModeInclusive, key_dtype, value_dtype, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
