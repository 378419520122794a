// scan.cuh -- internal interface of the decoupled look-back scan.
#pragma once

#include "common.cuh"

namespace lcpp {
namespace scan {

size_t temp_bytes(lcpp_dtype dt, uint64_t n);

// mode: 0 exclusive (init required), 1 inclusive, 2 inclusive with init.
lcpp_status run(void* temp, size_t temp_bytes, const void* in, void* out, uint64_t n, lcpp_op op,
                const void* init, lcpp_dtype dt, int mode, cudaStream_t stream);

// run() with the initial value read by the kernels from device memory
// (init_dev, one item of dt) when init_dev is not null; init is then unused.
lcpp_status run_with_init(void* temp, size_t temp_bytes, const void* in, void* out, uint64_t n, lcpp_op op,
                          const void* init, const void* init_dev, lcpp_dtype dt, int mode, cudaStream_t stream);

size_t error_word_offset();

}  // namespace scan
}  // namespace lcpp
