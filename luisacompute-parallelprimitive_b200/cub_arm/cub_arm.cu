// cub_arm.cu -- NVIDIA CUB (the CUDA toolkit's copy) behind a small C ABI,
// for bench.py --impl cub only: the same-box comparison point the
// reference's own benchmark uses (tests/cub_bench_kernels.cu:20-75 of the
// reference runs cub::DeviceRadixSort / DeviceScan / DeviceReduce beside
// LCPP).  Library calls used as they are; not part of liblcpp_b200.
#include <cub/cub.cuh>
#include <cstdint>

extern "C" {

// CUB_VERSION of the headers this was built with (major * 100000 + minor * 100 + patch).
int cub_arm_version() { return CUB_VERSION; }

// op: 0 SortKeys u32 (all bits), 1 SortPairs u32/u32, 2 InclusiveSum i32, 3 Reduce Sum f32.
// temp == nullptr: *temp_bytes receives the size.  Returns the cudaError_t.
int cub_arm_run(int op, void* temp, size_t* temp_bytes, const void* in0, void* out0, const void* in1, void* out1,
                uint64_t n, cudaStream_t stream)
{
    const int ni = int(n);
    switch (op) {
    case 0:
        return int(cub::DeviceRadixSort::SortKeys(temp, *temp_bytes, static_cast<const uint32_t*>(in0),
                                                  static_cast<uint32_t*>(out0), ni, 0, 32, stream));
    case 1:
        return int(cub::DeviceRadixSort::SortPairs(temp, *temp_bytes, static_cast<const uint32_t*>(in0),
                                                   static_cast<uint32_t*>(out0), static_cast<const uint32_t*>(in1),
                                                   static_cast<uint32_t*>(out1), ni, 0, 32, stream));
    case 2:
        return int(cub::DeviceScan::InclusiveSum(temp, *temp_bytes, static_cast<const int32_t*>(in0),
                                                 static_cast<int32_t*>(out0), ni, stream));
    case 3:
        return int(cub::DeviceReduce::Sum(temp, *temp_bytes, static_cast<const float*>(in0),
                                          static_cast<float*>(out0), ni, stream));
    default:
        return int(cudaErrorInvalidValue);
    }
}

}  // extern "C"
