// testgen.cu -- seeded counter-based synthetic inputs (see
// include/lcpp_b200_testgen.h).  Not part of the sort / scan / reduce path.
#include "../../include/lcpp_b200_testgen.h"
#include "common.cuh"

namespace lcpp {
namespace testgen {

__device__ __forceinline__ uint64_t splitmix64(uint64_t x)
{
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ uint64_t counter_rand(uint64_t seed, uint64_t stream, uint64_t i)
{
    return splitmix64((seed << 40) + (stream << 36) + i);
}

// MurmurHash3 32-bit finaliser (a bijection on 32-bit words).
__device__ __forceinline__ uint32_t fmix32(uint32_t h)
{
    h ^= h >> 16;
    h *= 0x85ebca6bu;
    h ^= h >> 13;
    h *= 0xc2b2ae35u;
    h ^= h >> 16;
    return h;
}

// Zipf(s) over ranks [1, N] by rejection-inversion (W. Hormann and
// G. Derflinger, "Rejection-inversion to generate variates from monotone
// discrete distributions", ACM TOMACS 6(3), 1996).  H is an antiderivative
// of the hat function h(x) = x^-s, Hinv its inverse.
struct ZipfParams {
    double s, one_minus_s, h_x1, h_n, accept;
};

__device__ __forceinline__ double zipf_H(double x, double oms)
{
    return (exp(oms * log(x)) - 1.0) / oms;
}
__device__ __forceinline__ double zipf_Hinv(double y, double oms)
{
    return exp(log1p(y * oms) / oms);
}
__device__ __forceinline__ double zipf_h(double x, double s) { return exp(-s * log(x)); }

__device__ uint64_t zipf_sample(uint64_t seed, uint64_t i, const ZipfParams& p, double n_ranks)
{
    uint64_t k = 1;
    for (int attempt = 0; attempt < 64; ++attempt) {
        const uint64_t r = counter_rand(seed, 3 + attempt, i);
        const double u01 = double(r >> 11) * (1.0 / 9007199254740992.0);
        const double u = p.h_n + u01 * (p.h_x1 - p.h_n);
        const double x = zipf_Hinv(u, p.one_minus_s);
        double kd = floor(x + 0.5);
        if (kd < 1.0) kd = 1.0;
        if (kd > n_ranks) kd = n_ranks;
        k = uint64_t(kd);
        if (kd - x <= p.accept || u >= zipf_H(kd + 0.5, p.one_minus_s) - zipf_h(kd, p.s)) return k;
    }
    return k;
}

__global__ void fill_kernel(void* dst, uint64_t n, uint64_t offset, uint64_t seed, int dist,
                            ZipfParams zp)
{
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t j = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += stride) {
        const uint64_t i = offset + j;
        switch (dist) {
        case LCPP_GEN_U32_UNIFORM:
            static_cast<uint32_t*>(dst)[j] = uint32_t(counter_rand(seed, 0, i));
            break;
        case LCPP_GEN_U32_AND3:
            static_cast<uint32_t*>(dst)[j] =
                uint32_t(counter_rand(seed, 0, i) & counter_rand(seed, 1, i) & counter_rand(seed, 2, i));
            break;
        case LCPP_GEN_U32_CONST: static_cast<uint32_t*>(dst)[j] = 0x9E3779B9u; break;
        case LCPP_GEN_U64_UNIFORM: static_cast<uint64_t*>(dst)[j] = counter_rand(seed, 0, i); break;
        case LCPP_GEN_I32_SCAN:
            static_cast<int32_t*>(dst)[j] = int32_t(counter_rand(seed, 0, i) % 2001ull) - 1000;
            break;
        case LCPP_GEN_F32_UNIT:
            static_cast<float*>(dst)[j] = float(counter_rand(seed, 0, i) >> 40) * (1.0f / 16777216.0f);
            break;
        case LCPP_GEN_I64_UNIFORM:
            static_cast<int64_t*>(dst)[j] = int64_t(counter_rand(seed, 0, i));
            break;
        case LCPP_GEN_U32_INDEX: static_cast<uint32_t*>(dst)[j] = uint32_t(i); break;
        case LCPP_GEN_F32_NORMAL: {
            float z;
            if (i % 65536 == 0) {
                z = 0.0f;
            } else if (i % 65536 == 32768) {
                z = -0.0f;
            } else {
                const uint64_t r = counter_rand(seed, 0, i);
                const double u1 = (double(r >> 32) + 0.5) * (1.0 / 4294967296.0);
                const double u2 = double(uint32_t(r)) * (1.0 / 4294967296.0);
                z = float(sqrt(-2.0 * log(u1)) * cospi(2.0 * u2));
            }
            static_cast<float*>(dst)[j] = z;
            break;
        }
        case LCPP_GEN_U32_ZIPF:
            static_cast<uint32_t*>(dst)[j] = fmix32(uint32_t(zipf_sample(seed, i, zp, 4294967296.0)));
            break;
        default: break;
        }
    }
}

}  // namespace testgen
}  // namespace lcpp

extern "C" lcpp_status lcpp_testgen_fill(void* dst, uint64_t n, uint64_t offset, uint64_t seed,
                                         lcpp_testgen_dist dist, lcpp_stream_t stream)
{
    using namespace lcpp;
    using namespace lcpp::testgen;
    if (n == 0) return LCPP_OK;
    if (!dst || int(dist) < 0 || int(dist) > LCPP_GEN_U32_ZIPF) return LCPP_ERR_INVALID_ARG;
    const int eb = (dist == LCPP_GEN_U64_UNIFORM || dist == LCPP_GEN_I64_UNIFORM) ? 8 : 4;
    if (reinterpret_cast<uintptr_t>(dst) % eb) return LCPP_ERR_INVALID_ARG;
    ZipfParams zp{};
    {
        // Host-side constants of the sampler for s = 1.1, N = 2^32.
        const double s = 1.1, oms = 1.0 - s, n_ranks = 4294967296.0;
        auto H = [&](double x) { return (std::exp(oms * std::log(x)) - 1.0) / oms; };
        auto Hinv = [&](double y) { return std::exp(std::log1p(y * oms) / oms); };
        auto h = [&](double x) { return std::exp(-s * std::log(x)); };
        zp.s = s;
        zp.one_minus_s = oms;
        zp.h_x1 = H(1.5) - 1.0;
        zp.h_n = H(n_ranks + 0.5);
        zp.accept = 2.0 - Hinv(H(2.5) - h(2.0));
    }
    const int block = 256;
    const uint64_t blocks = std::min<uint64_t>(ceil_div(n, block), uint64_t(device_sm_count()) * 16);
    fill_kernel<<<unsigned(blocks), block, 0, reinterpret_cast<cudaStream_t>(stream)>>>(dst, n, offset, seed,
                                                                                       int(dist), zp);
    return cudaGetLastError() == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
}
