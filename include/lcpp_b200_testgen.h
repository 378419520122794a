/*
 * lcpp_b200_testgen.h -- synthetic input generators of liblcpp_b200.
 *
 * No counterpart in the reference: these kernels synthesise the seeded,
 * counter-based benchmark and test inputs on the device so that multi-GB
 * workloads need no host generation.  They are not part of the sort / scan /
 * reduce path.  Element i of every distribution is a pure function of
 * (seed, i), so any slice can be regenerated independently:
 *
 *   r(seed, stream, i) = splitmix64(seed * 2^40 + stream * 2^36 + i)
 *
 * with splitmix64 the finaliser of Steele, Lea & Flood's SplitMix generator
 * (z += 0x9E3779B97F4A7C15; z = (z ^ z>>30) * 0xBF58476D1CE4E5B9;
 *  z = (z ^ z>>27) * 0x94D049BB133111EB; z ^ z>>31).
 */
#ifndef LCPP_B200_TESTGEN_H
#define LCPP_B200_TESTGEN_H

#include <stdint.h>

#include "lcpp_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef enum lcpp_testgen_dist {
    LCPP_GEN_U32_UNIFORM = 0, /* u32: low 32 bits of r(seed,0,i) */
    LCPP_GEN_U32_AND3 = 1,    /* u32: r(seed,0,i) & r(seed,1,i) & r(seed,2,i) (low-entropy) */
    LCPP_GEN_U32_CONST = 2,   /* u32: 0x9E3779B9 (all keys equal) */
    LCPP_GEN_U64_UNIFORM = 3, /* u64: r(seed,0,i) */
    LCPP_GEN_I32_SCAN = 4,    /* i32: (r(seed,0,i) % 2001) - 1000 */
    LCPP_GEN_F32_UNIT = 5,    /* f32: (r(seed,0,i) >> 40) * 2^-24, in [0,1) */
    LCPP_GEN_I64_UNIFORM = 6, /* i64: r(seed,0,i) as two's complement */
    LCPP_GEN_U32_INDEX = 7,   /* u32: i (values = original index) */
    LCPP_GEN_F32_NORMAL = 8,  /* f32: Box-Muller N(0,1) from r(seed,0,i); exact +0.0 at
                                 i % 65536 == 0 and -0.0 at i % 65536 == 32768 */
    LCPP_GEN_U32_ZIPF = 9     /* u32: fmix32(rank), rank ~ Zipf(s=1.1) over [1, 2^32],
                                 rejection-inversion sampling (Hormann & Derflinger 1996) */
} lcpp_testgen_dist;

/* Fill dst[j] with element (offset + j) of `dist`, j in [0, n).  dst must be
 * aligned to the element size. */
lcpp_status lcpp_testgen_fill(void* dst, uint64_t n, uint64_t offset, uint64_t seed,
                              lcpp_testgen_dist dist, lcpp_stream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* LCPP_B200_TESTGEN_H */
