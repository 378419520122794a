// radix_sort.cuh -- internal interface of the onesweep radix sort.
#pragma once

#include "common.cuh"

namespace lcpp {
namespace radix {

constexpr int kRadixBits = 8;
constexpr int kDigits = 1 << kRadixBits;
constexpr int kMaxPasses = 8;  // 64-bit keys

// Temp bytes for keys of kb bytes and values of vb bytes (0 = keys only).
size_t temp_bytes(int kb, int vb, uint64_t n);

// Shared implementation of the copy and DoubleBuffer entry points.
lcpp_status sort(void* temp, size_t temp_bytes, const void* keys_in, void* keys_out,
                 const void* vals_in, void* vals_out, void* key_bufs[2], void* val_bufs[2],
                 int* selector, uint64_t n, int begin_bit, int end_bit, int descending,
                 lcpp_dtype kdt, lcpp_dtype vdt, bool pairs, bool double_buffer,
                 cudaStream_t stream);

// Byte offset of the device error word inside the sort's temp storage.
size_t error_word_offset();

// Runs the look-back's bounded wait on a status word nothing publishes
// (lcpp_diag_wait_timeout_probe).
lcpp_status wait_timeout_probe(void* temp, size_t temp_bytes, uint64_t limit_ns, cudaStream_t stream);

}  // namespace radix
}  // namespace lcpp
