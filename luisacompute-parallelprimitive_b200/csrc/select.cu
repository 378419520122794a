// select.cu -- DeviceSelect::Flagged / If / FlaggedIf / Unique / UniqueByKey
// (src/lcpp/device/device_select.h:56-345) behind the C ABI; the kernel is
// lcpp_b200::device::select_detail::compact_kernel
// (include/lcpp_b200_device.cuh).
#include "select.cuh"

using namespace lcpp;
using namespace lcpp::sel;

namespace {

template <int SEL, typename T, typename F, typename V, typename Pick>
lcpp_status go(void* temp, size_t temp_bytes, sd::Args<T, F, V> a, Pick pick, cudaStream_t s)
{
    diag::KernelTimer timer(8 /* LCPP_KERNEL_SELECT */, a.n, s);
    return status_of(sd::launch<SEL, sd::kOutSelect>(temp, temp_bytes, a, pick, sd::Never{},
                                                      lcpp_b200::device::EqualTo{}, s));
}

}  // namespace

extern "C" {

lcpp_status lcpp_select_temp_bytes(uint64_t num_items, size_t* temp_bytes)
{
    if (!temp_bytes) return LCPP_ERR_INVALID_ARG;
    *temp_bytes = lcpp_b200::device::select_temp_bytes(num_items, false);
    return LCPP_OK;
}

lcpp_status lcpp_select_flagged(void* temp, size_t temp_bytes, const void* d_in, const void* d_flags, void* d_out,
                                uint32_t* d_num_selected_out, uint64_t num_items, lcpp_dtype dtype,
                                lcpp_dtype flag_dtype, lcpp_stream_t stream)
{
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    lcpp_status st = check(temp, temp_bytes, d_in, dtype_bytes(dtype), d_num_selected_out, num_items, false);
    if (st != LCPP_OK) return st;
    const int fb = flag_bytes(flag_dtype);
    if (!fb) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (num_items && (!d_flags || !d_out || misaligned(d_flags, fb) || misaligned(d_out, dtype_bytes(dtype))))
        return LCPP_ERR_INVALID_ARG;
    return with_bits_type(dtype, [&](auto t) {
        using T = decltype(t);
        return with_flag_nonzero_type(flag_dtype, [&](auto f) {
            using F = decltype(f);
            sd::Args<T, F, NoValue> a{static_cast<const T*>(d_in), static_cast<const F*>(d_flags), nullptr,
                                      static_cast<T*>(d_out), nullptr, nullptr, nullptr, d_num_selected_out,
                                      num_items, false};
            return go<sd::kSelFlag>(temp, temp_bytes, a, lcpp_b200::device::NonZero{}, s);
        });
    });
}

lcpp_status lcpp_select_flagged_if(void* temp, size_t temp_bytes, const void* d_in, const void* d_flags,
                                   void* d_out, uint32_t* d_num_selected_out, uint64_t num_items, lcpp_dtype dtype,
                                   lcpp_dtype flag_dtype, const lcpp_clause* clauses, int num_clauses,
                                   lcpp_stream_t stream)
{
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    lcpp_status st = check(temp, temp_bytes, d_in, dtype_bytes(dtype), d_num_selected_out, num_items, false);
    if (st != LCPP_OK) return st;
    const int fb = flag_bytes(flag_dtype);
    if (!fb) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (num_items && (!d_flags || !d_out || misaligned(d_flags, fb) || misaligned(d_out, dtype_bytes(dtype))))
        return LCPP_ERR_INVALID_ARG;
    auto with_flag = [&](auto&& fn) -> lcpp_status {
        if (flag_dtype == LCPP_U8) return fn(uint8_t{});
        return with_value_type(flag_dtype, fn);
    };
    return with_bits_type(dtype, [&](auto t) {
        using T = decltype(t);
        return with_flag([&](auto f) {
            using F = decltype(f);
            ClausePick<F> pick;
            const lcpp_status ps = make_pick(clauses, num_clauses, pick);
            if (ps != LCPP_OK) return ps;
            sd::Args<T, F, NoValue> a{static_cast<const T*>(d_in), static_cast<const F*>(d_flags), nullptr,
                                      static_cast<T*>(d_out), nullptr, nullptr, nullptr, d_num_selected_out,
                                      num_items, false};
            return go<sd::kSelFlag>(temp, temp_bytes, a, pick, s);
        });
    });
}

lcpp_status lcpp_select_if(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                           uint32_t* d_num_selected_out, uint64_t num_items, lcpp_dtype dtype,
                           const lcpp_clause* clauses, int num_clauses, lcpp_stream_t stream)
{
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    lcpp_status st = check(temp, temp_bytes, d_in, dtype_bytes(dtype), d_num_selected_out, num_items, false);
    if (st != LCPP_OK) return st;
    if (num_items && (!d_out || misaligned(d_out, dtype_bytes(dtype)))) return LCPP_ERR_INVALID_ARG;
    return with_value_type(dtype, [&](auto t) {
        using T = decltype(t);
        ClausePick<T> pick;
        const lcpp_status ps = make_pick(clauses, num_clauses, pick);
        if (ps != LCPP_OK) return ps;
        sd::Args<T, T, NoValue> a{static_cast<const T*>(d_in), nullptr, nullptr, static_cast<T*>(d_out), nullptr,
                                  nullptr, nullptr, d_num_selected_out, num_items, false};
        return go<sd::kSelIf>(temp, temp_bytes, a, pick, s);
    });
}

lcpp_status lcpp_select_unique(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                               uint32_t* d_num_selected_out, uint64_t num_items, lcpp_dtype dtype,
                               lcpp_stream_t stream)
{
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    lcpp_status st = check(temp, temp_bytes, d_in, dtype_bytes(dtype), d_num_selected_out, num_items, false);
    if (st != LCPP_OK) return st;
    if (num_items && (!d_out || misaligned(d_out, dtype_bytes(dtype)))) return LCPP_ERR_INVALID_ARG;
    return with_key_type(dtype, [&](auto t) {
        using T = decltype(t);
        sd::Args<T, T, NoValue> a{static_cast<const T*>(d_in), nullptr, nullptr, static_cast<T*>(d_out), nullptr,
                                  nullptr, nullptr, d_num_selected_out, num_items, false};
        return go<sd::kSelUnique>(temp, temp_bytes, a, sd::Never{}, s);
    });
}

lcpp_status lcpp_select_unique_by_key(void* temp, size_t temp_bytes, const void* d_keys_in, const void* d_values_in,
                                      void* d_keys_out, void* d_values_out, uint32_t* d_num_selected_out,
                                      uint64_t num_items, lcpp_dtype key_dtype, lcpp_dtype value_dtype,
                                      lcpp_stream_t stream)
{
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    lcpp_status st = check(temp, temp_bytes, d_keys_in, dtype_bytes(key_dtype), d_num_selected_out, num_items, false);
    if (st != LCPP_OK) return st;
    const int vb = dtype_bytes(value_dtype);
    if (!vb) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (num_items && (!d_keys_out || !d_values_in || !d_values_out || misaligned(d_keys_out, dtype_bytes(key_dtype)) ||
                      misaligned(d_values_in, vb) || misaligned(d_values_out, vb)))
        return LCPP_ERR_INVALID_ARG;
    return with_key_type(key_dtype, [&](auto k) {
        using K = decltype(k);
        return with_bits_type(value_dtype, [&](auto v) {
            using V = decltype(v);
            sd::Args<K, K, V> a{static_cast<const K*>(d_keys_in), nullptr, static_cast<const V*>(d_values_in),
                                static_cast<K*>(d_keys_out), nullptr, nullptr, static_cast<V*>(d_values_out),
                                d_num_selected_out, num_items, false};
            return go<sd::kSelUnique>(temp, temp_bytes, a, sd::Never{}, s);
        });
    });
}

lcpp_status lcpp_scan_transform_temp_bytes(uint64_t num_items, size_t* temp_bytes)
{
    if (!temp_bytes) return LCPP_ERR_INVALID_ARG;
    *temp_bytes = lcpp_b200::device::select_temp_bytes(num_items, false);
    return LCPP_OK;
}

lcpp_status lcpp_scan_exclusive_sum_transform(void* temp, size_t temp_bytes, const void* d_in, uint32_t* d_out,
                                              uint64_t num_items, lcpp_dtype dtype, const lcpp_clause* clauses,
                                              int num_clauses, lcpp_stream_t stream)
{
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    // d_out stands in for the count pointer: non-null and 4-byte aligned
    lcpp_status st = check(temp, temp_bytes, d_in, dtype_bytes(dtype), d_out, num_items, false);
    if (st != LCPP_OK || num_items == 0) return st;
    return with_value_type(dtype, [&](auto t) {
        using T = decltype(t);
        ClausePick<T> pick;
        const lcpp_status ps = make_pick(clauses, num_clauses, pick);
        if (ps != LCPP_OK) return ps;
        sd::Args<T, T, NoValue> a{static_cast<const T*>(d_in), nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                                  nullptr, num_items, false, d_out};
        diag::KernelTimer timer(8 /* LCPP_KERNEL_SELECT */, num_items, s);
        return status_of(sd::launch<sd::kSelIf, sd::kOutRanks>(temp, temp_bytes, a, pick, sd::Never{},
                                                                lcpp_b200::device::EqualTo{}, s));
    });
}

lcpp_status lcpp_scan_exclusive_sum_adjacent(void* temp, size_t temp_bytes, const void* d_in, uint32_t* d_out,
                                             uint64_t num_items, lcpp_dtype dtype, lcpp_stream_t stream)
{
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    lcpp_status st = check(temp, temp_bytes, d_in, dtype_bytes(dtype), d_out, num_items, false);
    if (st != LCPP_OK || num_items == 0) return st;
    return with_key_type(dtype, [&](auto t) {
        using T = decltype(t);
        sd::Args<T, T, NoValue> a{static_cast<const T*>(d_in), nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                                  nullptr, num_items, false, d_out};
        diag::KernelTimer timer(8 /* LCPP_KERNEL_SELECT */, num_items, s);
        return status_of(sd::launch<sd::kSelUnique, sd::kOutRanks>(temp, temp_bytes, a, sd::Never{}, sd::Never{},
                                                                    lcpp_b200::device::EqualTo{}, s));
    });
}

}  // extern "C"
