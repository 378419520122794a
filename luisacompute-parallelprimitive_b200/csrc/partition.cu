// partition.cu -- DevicePartition::Flagged / If and the three-way If
// (src/lcpp/device/device_partition.h:55-227) behind the C ABI; the kernel
// is lcpp_b200::device::select_detail::compact_kernel
// (include/lcpp_b200_device.cuh).
#include "select.cuh"

using namespace lcpp;
using namespace lcpp::sel;

namespace {

// True when [out, out + n items) and [in, in + n items) share a byte: the
// partitions write rejected items from the end of the output backwards, so
// any overlap with the input could overwrite items a later tile has not
// read yet (the reference checks the same, device_partition.h:270-285).
bool ranges_overlap(const void* in, const void* out, uint64_t num_items, int item_bytes)
{
    const char *a0 = static_cast<const char*>(in), *b0 = static_cast<const char*>(out);
    const size_t len = size_t(num_items) * size_t(item_bytes);
    return num_items && a0 < b0 + len && b0 < a0 + len;
}

}  // namespace

extern "C" {

lcpp_status lcpp_partition_temp_bytes(uint64_t num_items, size_t* temp_bytes)
{
    if (!temp_bytes) return LCPP_ERR_INVALID_ARG;
    *temp_bytes = lcpp_b200::device::select_temp_bytes(num_items, false);
    return LCPP_OK;
}

lcpp_status lcpp_partition_three_way_temp_bytes(uint64_t num_items, size_t* temp_bytes)
{
    if (!temp_bytes) return LCPP_ERR_INVALID_ARG;
    *temp_bytes = lcpp_b200::device::select_temp_bytes(num_items, true);
    return LCPP_OK;
}

lcpp_status lcpp_partition_flagged(void* temp, size_t temp_bytes, const void* d_in, const void* d_flags, void* d_out,
                                   uint32_t* d_num_selected_out, uint64_t num_items, lcpp_dtype dtype,
                                   lcpp_dtype flag_dtype, lcpp_stream_t stream)
{
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    lcpp_status st = check(temp, temp_bytes, d_in, dtype_bytes(dtype), d_num_selected_out, num_items, false);
    if (st != LCPP_OK) return st;
    const int fb = flag_bytes(flag_dtype);
    if (!fb) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (num_items && (!d_flags || !d_out || ranges_overlap(d_in, d_out, num_items, dtype_bytes(dtype)) ||
                      misaligned(d_flags, fb) || misaligned(d_out, dtype_bytes(dtype))))
        return LCPP_ERR_INVALID_ARG;
    return with_bits_type(dtype, [&](auto t) {
        using T = decltype(t);
        return with_flag_nonzero_type(flag_dtype, [&](auto f) {
            using F = decltype(f);
            sd::Args<T, F, NoValue> a{static_cast<const T*>(d_in), static_cast<const F*>(d_flags), nullptr,
                                      static_cast<T*>(d_out), nullptr, nullptr, nullptr, d_num_selected_out,
                                      num_items, false};
            diag::KernelTimer timer(8 /* LCPP_KERNEL_SELECT */, num_items, s);
            return status_of(sd::launch<sd::kSelFlag, sd::kOutPartition>(temp, temp_bytes, a,
                                                                          lcpp_b200::device::NonZero{}, sd::Never{},
                                                                          lcpp_b200::device::EqualTo{}, s));
        });
    });
}

lcpp_status lcpp_partition_if(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                              uint32_t* d_num_selected_out, uint64_t num_items, lcpp_dtype dtype,
                              const lcpp_clause* clauses, int num_clauses, lcpp_stream_t stream)
{
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    lcpp_status st = check(temp, temp_bytes, d_in, dtype_bytes(dtype), d_num_selected_out, num_items, false);
    if (st != LCPP_OK) return st;
    if (num_items && (!d_out || ranges_overlap(d_in, d_out, num_items, dtype_bytes(dtype)) ||
                      misaligned(d_out, dtype_bytes(dtype))))
        return LCPP_ERR_INVALID_ARG;
    return with_value_type(dtype, [&](auto t) {
        using T = decltype(t);
        ClausePick<T> pick;
        const lcpp_status ps = make_pick(clauses, num_clauses, pick);
        if (ps != LCPP_OK) return ps;
        sd::Args<T, T, NoValue> a{static_cast<const T*>(d_in), nullptr, nullptr, static_cast<T*>(d_out), nullptr,
                                  nullptr, nullptr, d_num_selected_out, num_items, false};
        diag::KernelTimer timer(8 /* LCPP_KERNEL_SELECT */, num_items, s);
        return status_of(sd::launch<sd::kSelIf, sd::kOutPartition>(temp, temp_bytes, a, pick, sd::Never{},
                                                                    lcpp_b200::device::EqualTo{}, s));
    });
}

lcpp_status lcpp_partition_if_three_way(void* temp, size_t temp_bytes, const void* d_in, void* d_first_out,
                                        void* d_second_out, void* d_unselected_out, uint32_t* d_num_selected_out,
                                        uint64_t num_items, lcpp_dtype dtype, const lcpp_clause* first_clauses,
                                        int num_first_clauses, const lcpp_clause* second_clauses,
                                        int num_second_clauses, lcpp_stream_t stream)
{
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    lcpp_status st = check(temp, temp_bytes, d_in, dtype_bytes(dtype), d_num_selected_out, num_items, true);
    if (st != LCPP_OK) return st;
    const int tb = dtype_bytes(dtype);
    if (num_items && (!d_first_out || !d_second_out || !d_unselected_out || misaligned(d_first_out, tb) ||
                      misaligned(d_second_out, tb) || misaligned(d_unselected_out, tb)))
        return LCPP_ERR_INVALID_ARG;
    // the outputs must not overlap the input (device_partition.h:270-285)
    if (ranges_overlap(d_in, d_first_out, num_items, tb) || ranges_overlap(d_in, d_second_out, num_items, tb) ||
        ranges_overlap(d_in, d_unselected_out, num_items, tb))
        return LCPP_ERR_INVALID_ARG;
    return with_value_type(dtype, [&](auto t) {
        using T = decltype(t);
        ClausePick<T> first, second;
        lcpp_status ps = make_pick(first_clauses, num_first_clauses, first);
        if (ps == LCPP_OK) ps = make_pick(second_clauses, num_second_clauses, second);
        if (ps != LCPP_OK) return ps;
        sd::Args<T, T, NoValue> a{static_cast<const T*>(d_in), nullptr, nullptr, static_cast<T*>(d_first_out),
                                  static_cast<T*>(d_second_out), static_cast<T*>(d_unselected_out), nullptr,
                                  d_num_selected_out, num_items, false};
        diag::KernelTimer timer(8 /* LCPP_KERNEL_SELECT */, num_items, s);
        return status_of(sd::launch<sd::kSelIf, sd::kOutThreeWay>(temp, temp_bytes, a, first, second,
                                                                   lcpp_b200::device::EqualTo{}, s));
    });
}

}  // extern "C"
