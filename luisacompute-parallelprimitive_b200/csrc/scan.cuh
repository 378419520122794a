// scan.cuh -- internal interface of the decoupled look-back scan.
#pragma once

#include "common.cuh"

namespace lcpp {
namespace scan {

size_t temp_bytes(lcpp_dtype dt, uint64_t n);

// mode: 0 exclusive (init required), 1 inclusive, 2 inclusive with init.
lcpp_status run(void* temp, size_t temp_bytes, const void* in, void* out, uint64_t n, lcpp_op op,
                const void* init, lcpp_dtype dt, int mode, cudaStream_t stream);

size_t error_word_offset();

}  // namespace scan
}  // namespace lcpp
