// capi.cu -- extern "C" entry points of liblcpp_b200 (include/lcpp_b200.h).
#include <cstring>
#include <limits>
#include <mutex>
#include <map>
#include <set>
#include <utility>

#include "common.cuh"
#include "radix_sort.cuh"
#include "reduce.cuh"
#include "scan.cuh"

namespace lcpp {

int device_sm_count()
{
    static std::mutex mu;
    static int cache[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return 148;  // no device: size as for a B200
    }
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 0 && dev < 64 && cache[dev]) return cache[dev];
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
        cudaGetLastError();
        sms = 148;
    }
    if (dev >= 0 && dev < 64) cache[dev] = sms;
    return sms;
}

void set_max_dynamic_smem(const void* kernel, size_t bytes)
{
    static std::mutex mu;
    static std::set<std::pair<std::pair<const void*, int>, size_t>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    auto key = std::make_pair(std::make_pair(kernel, dev), bytes);
    if (done.count(key)) return;
    // Always set: the 48 KB default also has to hold the kernel's static
    // shared memory, so a dynamic size just under it can still need opt-in.
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
    done.insert(key);
}

int resident_blocks(const void* kernel, int block, size_t dynamic_smem)
{
    static std::mutex mu;
    static std::map<std::pair<std::pair<const void*, int>, std::pair<int, size_t>>, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    const auto key = std::make_pair(std::make_pair(kernel, dev), std::make_pair(block, dynamic_smem));
    const auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    int blocks = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, block, dynamic_smem) != cudaSuccess) {
        cudaGetLastError();
        blocks = 1;
    }
    blocks = blocks < 1 ? 1 : blocks;
    cache[key] = blocks;
    return blocks;
}

}  // namespace lcpp

using lcpp::radix::sort;

namespace {

cudaStream_t as_cuda(lcpp_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

template <typename T>
void set_limits(lcpp_op op, void* out)
{
    T v{};
    if (op == LCPP_OP_MIN) v = std::numeric_limits<T>::max();
    if (op == LCPP_OP_MAX) v = std::numeric_limits<T>::lowest();
    std::memcpy(out, &v, sizeof(T));
}

// DeviceReduce's initial values: Sum 0, Min numeric max, Max numeric lowest
// (src/lcpp/device/device_reduce.h:280-308).
bool reduce_init(lcpp_dtype dt, lcpp_op op, unsigned char out[8])
{
    switch (dt) {
    case LCPP_U32: set_limits<uint32_t>(op, out); return true;
    case LCPP_I32: set_limits<int32_t>(op, out); return true;
    case LCPP_F32: set_limits<float>(op, out); return true;
    case LCPP_U64: set_limits<uint64_t>(op, out); return true;
    case LCPP_I64: set_limits<int64_t>(op, out); return true;
    case LCPP_F64: set_limits<double>(op, out); return true;
    default: return false;
    }
}

}  // namespace

extern "C" {

const char* lcpp_status_string(lcpp_status status)
{
    switch (status) {
    case LCPP_OK: return "LCPP_OK";
    case LCPP_ERR_INVALID_ARG: return "LCPP_ERR_INVALID_ARG";
    case LCPP_ERR_TEMP_TOO_SMALL: return "LCPP_ERR_TEMP_TOO_SMALL";
    case LCPP_ERR_UNSUPPORTED_DTYPE: return "LCPP_ERR_UNSUPPORTED_DTYPE";
    case LCPP_ERR_CUDA: return "LCPP_ERR_CUDA";
    case LCPP_ERR_LOOKBACK_TIMEOUT: return "LCPP_ERR_LOOKBACK_TIMEOUT";
    case LCPP_ERR_COMM: return "LCPP_ERR_COMM";
    case LCPP_ERR_INTERNAL: return "LCPP_ERR_INTERNAL";
    default: return "LCPP_ERR_UNKNOWN";
    }
}

int lcpp_version(void) { return 100; }

// ---------------------------------------------------------------- radix sort
lcpp_status lcpp_radix_sort_keys_temp_bytes(lcpp_dtype key_dtype, uint64_t num_items, size_t* temp_bytes)
{
    if (!temp_bytes) return LCPP_ERR_INVALID_ARG;
    const int kb = lcpp::dtype_bytes(key_dtype);
    if (!kb) return LCPP_ERR_UNSUPPORTED_DTYPE;
    *temp_bytes = lcpp::radix::temp_bytes(kb, 0, num_items);
    return LCPP_OK;
}

lcpp_status lcpp_radix_sort_pairs_temp_bytes(lcpp_dtype key_dtype, lcpp_dtype value_dtype,
                                             uint64_t num_items, size_t* temp_bytes)
{
    if (!temp_bytes) return LCPP_ERR_INVALID_ARG;
    const int kb = lcpp::dtype_bytes(key_dtype), vb = lcpp::dtype_bytes(value_dtype);
    if (!kb || !vb) return LCPP_ERR_UNSUPPORTED_DTYPE;
    *temp_bytes = lcpp::radix::temp_bytes(kb, vb, num_items);
    return LCPP_OK;
}

lcpp_status lcpp_radix_sort_keys(void* temp, size_t temp_bytes, const void* keys_in, void* keys_out,
                                 uint64_t num_items, int begin_bit, int end_bit, int descending,
                                 lcpp_dtype key_dtype, lcpp_stream_t stream)
{
    return sort(temp, temp_bytes, keys_in, keys_out, nullptr, nullptr, nullptr, nullptr, nullptr,
                num_items, begin_bit, end_bit, descending, key_dtype, LCPP_NONE, false, false,
                as_cuda(stream));
}

lcpp_status lcpp_radix_sort_pairs(void* temp, size_t temp_bytes, const void* keys_in, void* keys_out,
                                  const void* values_in, void* values_out, uint64_t num_items,
                                  int begin_bit, int end_bit, int descending, lcpp_dtype key_dtype,
                                  lcpp_dtype value_dtype, lcpp_stream_t stream)
{
    return sort(temp, temp_bytes, keys_in, keys_out, values_in, values_out, nullptr, nullptr, nullptr,
                num_items, begin_bit, end_bit, descending, key_dtype, value_dtype, true, false,
                as_cuda(stream));
}

lcpp_status lcpp_radix_sort_keys_double_buffer(void* temp, size_t temp_bytes, void* key_buffers[2],
                                               int* selector, uint64_t num_items, int begin_bit,
                                               int end_bit, int descending, lcpp_dtype key_dtype,
                                               lcpp_stream_t stream)
{
    return sort(temp, temp_bytes, nullptr, nullptr, nullptr, nullptr, key_buffers, nullptr, selector,
                num_items, begin_bit, end_bit, descending, key_dtype, LCPP_NONE, false, true,
                as_cuda(stream));
}

lcpp_status lcpp_radix_sort_pairs_double_buffer(void* temp, size_t temp_bytes, void* key_buffers[2],
                                                void* value_buffers[2], int* selector,
                                                uint64_t num_items, int begin_bit, int end_bit,
                                                int descending, lcpp_dtype key_dtype,
                                                lcpp_dtype value_dtype, lcpp_stream_t stream)
{
    return sort(temp, temp_bytes, nullptr, nullptr, nullptr, nullptr, key_buffers, value_buffers,
                selector, num_items, begin_bit, end_bit, descending, key_dtype, value_dtype, true, true,
                as_cuda(stream));
}

// ---------------------------------------------------------------------- scan
lcpp_status lcpp_scan_temp_bytes(lcpp_dtype dtype, uint64_t num_items, size_t* temp_bytes)
{
    if (!temp_bytes) return LCPP_ERR_INVALID_ARG;
    if (!lcpp::dtype_bytes(dtype)) return LCPP_ERR_UNSUPPORTED_DTYPE;
    *temp_bytes = lcpp::scan::temp_bytes(dtype, num_items);
    return LCPP_OK;
}

lcpp_status lcpp_scan_exclusive(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                                uint64_t num_items, lcpp_op op, const void* init, lcpp_dtype dtype,
                                lcpp_stream_t stream)
{
    return lcpp::scan::run(temp, temp_bytes, d_in, d_out, num_items, op, init, dtype, 0, as_cuda(stream));
}

lcpp_status lcpp_scan_inclusive(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                                uint64_t num_items, lcpp_op op, lcpp_dtype dtype, lcpp_stream_t stream)
{
    return lcpp::scan::run(temp, temp_bytes, d_in, d_out, num_items, op, nullptr, dtype, 1, as_cuda(stream));
}

lcpp_status lcpp_scan_inclusive_init(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                                     uint64_t num_items, lcpp_op op, const void* init,
                                     lcpp_dtype dtype, lcpp_stream_t stream)
{
    return lcpp::scan::run(temp, temp_bytes, d_in, d_out, num_items, op, init, dtype, 2, as_cuda(stream));
}

lcpp_status lcpp_scan_exclusive_sum(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                                    uint64_t num_items, lcpp_dtype dtype, lcpp_stream_t stream)
{
    const unsigned char zero[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    return lcpp::scan::run(temp, temp_bytes, d_in, d_out, num_items, LCPP_OP_SUM, zero, dtype, 0,
                           as_cuda(stream));
}

lcpp_status lcpp_scan_inclusive_sum(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                                    uint64_t num_items, lcpp_dtype dtype, lcpp_stream_t stream)
{
    return lcpp::scan::run(temp, temp_bytes, d_in, d_out, num_items, LCPP_OP_SUM, nullptr, dtype, 1,
                           as_cuda(stream));
}

// -------------------------------------------------------------------- reduce
lcpp_status lcpp_reduce_temp_bytes(lcpp_dtype dtype, uint64_t num_items, size_t* temp_bytes)
{
    if (!temp_bytes) return LCPP_ERR_INVALID_ARG;
    if (!lcpp::dtype_bytes(dtype)) return LCPP_ERR_UNSUPPORTED_DTYPE;
    *temp_bytes = lcpp::reduce::temp_bytes(dtype, num_items);
    return LCPP_OK;
}

lcpp_status lcpp_reduce(void* temp, size_t temp_bytes, const void* d_in, void* d_out, uint64_t num_items,
                        lcpp_op op, const void* init, lcpp_dtype dtype, lcpp_stream_t stream)
{
    return lcpp::reduce::run(temp, temp_bytes, d_in, d_out, num_items, op, init, dtype, as_cuda(stream));
}

static lcpp_status reduce_named(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                                uint64_t num_items, lcpp_op op, lcpp_dtype dtype, lcpp_stream_t stream)
{
    unsigned char init[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (!reduce_init(dtype, op, init)) return LCPP_ERR_UNSUPPORTED_DTYPE;
    return lcpp::reduce::run(temp, temp_bytes, d_in, d_out, num_items, op, init, dtype, as_cuda(stream));
}

lcpp_status lcpp_reduce_sum(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                            uint64_t num_items, lcpp_dtype dtype, lcpp_stream_t stream)
{
    return reduce_named(temp, temp_bytes, d_in, d_out, num_items, LCPP_OP_SUM, dtype, stream);
}

lcpp_status lcpp_reduce_min(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                            uint64_t num_items, lcpp_dtype dtype, lcpp_stream_t stream)
{
    return reduce_named(temp, temp_bytes, d_in, d_out, num_items, LCPP_OP_MIN, dtype, stream);
}

lcpp_status lcpp_reduce_max(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                            uint64_t num_items, lcpp_dtype dtype, lcpp_stream_t stream)
{
    return reduce_named(temp, temp_bytes, d_in, d_out, num_items, LCPP_OP_MAX, dtype, stream);
}

// --------------------------------------------------------------- diagnostics
// Each module keeps its device error word at a fixed offset of its temp
// storage (sort: Ctrl::error; scan and reduce: second word of the control
// block).  All three control blocks start at temp offset 0 and the error
// word is the second 32-bit word in each, so one read serves all modules.
lcpp_status lcpp_device_status(const void* temp, lcpp_stream_t stream)
{
    if (!temp) return LCPP_ERR_INVALID_ARG;
    static_assert(sizeof(uint32_t) == 4, "");
    if (lcpp::radix::error_word_offset() != 4 || lcpp::scan::error_word_offset() != 4) return LCPP_ERR_CUDA;
    if (cudaStreamSynchronize(as_cuda(stream)) != cudaSuccess) return LCPP_ERR_CUDA;
    uint32_t word = 0;
    if (cudaMemcpy(&word, static_cast<const unsigned char*>(temp) + 4, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return LCPP_ERR_CUDA;
    return word == 0 ? LCPP_OK : static_cast<lcpp_status>(word);
}

}  // extern "C"
