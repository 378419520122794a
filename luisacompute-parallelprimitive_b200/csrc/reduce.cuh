// reduce.cuh -- internal interface of the deterministic reduction.
#pragma once

#include "common.cuh"

namespace lcpp {
namespace reduce {

size_t temp_bytes(lcpp_dtype dt, uint64_t n);

lcpp_status run(void* temp, size_t temp_bytes, const void* in, void* out, uint64_t n, lcpp_op op,
                const void* init, lcpp_dtype dt, cudaStream_t stream);

}  // namespace reduce
}  // namespace lcpp
