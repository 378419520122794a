/*
 * lcpp_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference (LuisaCompute-ParallelPrimitive) semantics
 * for the sort / scan / reduce path.  It is the checker for the CUDA library
 * and the timed CPU baseline; nothing in the product links or calls it.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * this library.
 *
 * Parity is pinned by the golden fixtures under tests/golden/, which were
 * produced by the reference tests' own host oracles (std::sort,
 * std::stable_sort with a selected-bits comparator, std::inclusive_scan,
 * std::exclusive_scan, std::accumulate) on the reference tests' own input
 * generators; see tests/golden/make_golden.cpp.
 *
 * Element type codes match lcpp_dtype in include/lcpp_b200.h.
 */
#include <math.h>
#include <pthread.h>
#include <float.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { DT_U32 = 0, DT_I32 = 1, DT_F32 = 2, DT_U64 = 3, DT_I64 = 4, DT_F64 = 5 };
enum { OP_SUM = 0, OP_MIN = 1, OP_MAX = 2 };
enum { KIND_UNSIGNED = 0, KIND_SIGNED = 1, KIND_FLOAT = 2 };

static int dtype_bytes(int dt)
{
    switch (dt) {
    case DT_U32: case DT_I32: case DT_F32: return 4;
    case DT_U64: case DT_I64: case DT_F64: return 8;
    default: return 0;
    }
}

static int dtype_kind(int dt)
{
    switch (dt) {
    case DT_I32: case DT_I64: return KIND_SIGNED;
    case DT_F32: case DT_F64: return KIND_FLOAT;
    default: return KIND_UNSIGNED;
    }
}

/* ---------------------------------------------------------------------------
 * Key bijection.  Restates Traits<T>::TwiddleIn (src/lcpp/common/util_type.h:
 * 97-175): unsigned keys unchanged; signed keys XOR the high bit; floating keys
 * XOR all bits when the sign bit is set, else XOR the high bit.
 * ------------------------------------------------------------------------- */
static inline uint64_t traits_twiddle_in(uint64_t key, int kind, int bits)
{
    const uint64_t mask = bits == 64 ? ~0ull : ((1ull << bits) - 1ull);
    const uint64_t high = 1ull << (bits - 1);
    key &= mask;
    if (kind == KIND_SIGNED) return key ^ high;
    if (kind == KIND_FLOAT) return (key & high) ? (~key & mask) : (key ^ high);
    return key;
}

/* RadixSortTwiddle<DESC>::In (src/lcpp/agent/radix_rank_sort_operations.h:
 * 123-155): twiddle, then invert every bit for descending order. */
static inline uint64_t sort_twiddle_in(uint64_t key, int kind, int bits, int descending)
{
    const uint64_t mask = bits == 64 ? ~0ull : ((1ull << bits) - 1ull);
    uint64_t t = traits_twiddle_in(key, kind, bits);
    if (descending) t = ~t & mask;
    return t;
}

/* BaseDigitExtractor<float>::ProcessFloatMinusZero
 * (radix_rank_sort_operations.h:31-43): a transformed key equal to
 * TwiddleIn(-0.0 bits) is replaced by TwiddleIn(+0.0 bits) before digits are
 * taken, so that -0.0 and +0.0 always fall into the same bucket. */
static inline uint64_t fold_minus_zero(uint64_t t, int kind, int bits)
{
    if (kind != KIND_FLOAT) return t;
    const uint64_t high = 1ull << (bits - 1);
    const uint64_t tw_minus_zero = traits_twiddle_in(high, kind, bits);
    const uint64_t tw_zero = traits_twiddle_in(0, kind, bits);
    return t == tw_minus_zero ? tw_zero : t;
}

/* ShiftDigitExtractor::Digit (radix_rank_sort_operations.h:46-63). */
static inline uint32_t extract_digit(uint64_t key, int kind, int bits, int descending,
                                     int bit_start, int num_bits)
{
    uint64_t t = fold_minus_zero(sort_twiddle_in(key, kind, bits, descending), kind, bits);
    return (uint32_t)((t >> bit_start) & ((1ull << num_bits) - 1ull));
}

static inline uint64_t load_key(const void* p, uint64_t i, int key_bytes)
{
    if (key_bytes == 4) return ((const uint32_t*)p)[i];
    return ((const uint64_t*)p)[i];
}

static inline void store_raw(void* p, uint64_t i, const void* src, uint64_t j, int bytes)
{
    if (bytes == 4) ((uint32_t*)p)[i] = ((const uint32_t*)src)[j];
    else ((uint64_t*)p)[i] = ((const uint64_t*)src)[j];
}

/* ---------------------------------------------------------------------------
 * Stable LSD radix sort.  Restates the pass loop of
 * DeviceRadixSort::onesweep_radix_sort (src/lcpp/device/device_radix_sort.h:
 * 1380-1471): passes over [begin_bit, end_bit) in 8-bit steps, the last pass
 * taking min(8, end_bit - current_bit) bits; each pass is a stable
 * partition by digit (the onesweep kernel ranks keys in load order,
 * src/lcpp/block/block_radix_rank.h:401-425, and scatters them by digit,
 * src/lcpp/agent/agent_radix_sort_onesweep.h:434-511).  begin_bit == end_bit
 * is a copy (device_radix_sort.h:381-390).  Keys and values keep their
 * original bits.
 * ------------------------------------------------------------------------- */

typedef struct {
    const void* keys_src;
    const void* vals_src;
    void* keys_dst;
    void* vals_dst;
    uint64_t lo, hi;
    int kind, bits, key_bytes, val_bytes, descending, bit_start, num_bits;
    uint64_t* counts; /* [256] for this chunk; in: histogram, out: offsets */
    int phase;        /* 0 = histogram, 1 = scatter */
} pass_job;

static void* pass_worker(void* arg)
{
    pass_job* j = (pass_job*)arg;
    if (j->phase == 0) {
        memset(j->counts, 0, 256 * sizeof(uint64_t));
        for (uint64_t i = j->lo; i < j->hi; ++i) {
            uint64_t k = load_key(j->keys_src, i, j->key_bytes);
            j->counts[extract_digit(k, j->kind, j->bits, j->descending, j->bit_start, j->num_bits)]++;
        }
    } else {
        for (uint64_t i = j->lo; i < j->hi; ++i) {
            uint64_t k = load_key(j->keys_src, i, j->key_bytes);
            uint32_t d = extract_digit(k, j->kind, j->bits, j->descending, j->bit_start, j->num_bits);
            uint64_t pos = j->counts[d]++;
            store_raw(j->keys_dst, pos, j->keys_src, i, j->key_bytes);
            if (j->val_bytes) store_raw(j->vals_dst, pos, j->vals_src, i, j->val_bytes);
        }
    }
    return NULL;
}

static void run_jobs(pass_job* jobs, int threads)
{
    if (threads == 1) {
        pass_worker(&jobs[0]);
        return;
    }
    pthread_t* tid = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
    for (int t = 0; t < threads; ++t) pthread_create(&tid[t], NULL, pass_worker, &jobs[t]);
    for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
    free(tid);
}

/* Returns 0 on success, -1 on bad arguments, -2 on allocation failure.
 * value_bytes == 0 sorts keys only.  threads >= 1 splits every pass into
 * contiguous chunks whose per-digit offsets are laid out digit-major,
 * chunk-minor, so the result is identical for any thread count. */
int oracle_radix_sort(const void* keys_in, void* keys_out, const void* vals_in, void* vals_out,
                      uint64_t n, int begin_bit, int end_bit, int descending, int key_dtype,
                      int value_bytes, int threads)
{
    const int key_bytes = dtype_bytes(key_dtype);
    const int bits = key_bytes * 8;
    if (key_bytes == 0 || begin_bit < 0 || begin_bit > end_bit || end_bit > bits) return -1;
    if (value_bytes != 0 && value_bytes != 4 && value_bytes != 8) return -1;
    if (threads < 1) threads = 1;
    if (n == 0) return 0;
    if ((uint64_t)threads > n) threads = (int)n;
    if (begin_bit == end_bit) {
        memcpy(keys_out, keys_in, n * (uint64_t)key_bytes);
        if (value_bytes) memcpy(vals_out, vals_in, n * (uint64_t)value_bytes);
        return 0;
    }
    const int kind = dtype_kind(key_dtype);
    const int passes = (end_bit - begin_bit + 7) / 8;

    /* Ping-pong so that the last pass writes keys_out / vals_out. */
    void* ktmp = malloc(n * (uint64_t)key_bytes);
    void* vtmp = value_bytes ? malloc(n * (uint64_t)value_bytes) : NULL;
    pass_job* jobs = (pass_job*)calloc((size_t)threads, sizeof(pass_job));
    uint64_t* counts = (uint64_t*)calloc((size_t)threads * 256, sizeof(uint64_t));
    if (!ktmp || (value_bytes && !vtmp) || !jobs || !counts) {
        free(ktmp); free(vtmp); free(jobs); free(counts);
        return -2;
    }

    const void* ksrc = keys_in;
    const void* vsrc = vals_in;
    for (int p = 0; p < passes; ++p) {
        const int bit_start = begin_bit + 8 * p;
        const int num_bits = (end_bit - bit_start) < 8 ? (end_bit - bit_start) : 8;
        const int to_out = ((passes - 1 - p) % 2) == 0;
        void* kdst = to_out ? keys_out : ktmp;
        void* vdst = to_out ? vals_out : vtmp;
        for (int t = 0; t < threads; ++t) {
            pass_job* j = &jobs[t];
            j->keys_src = ksrc; j->vals_src = vsrc; j->keys_dst = kdst; j->vals_dst = vdst;
            j->lo = n * (uint64_t)t / (uint64_t)threads;
            j->hi = n * (uint64_t)(t + 1) / (uint64_t)threads;
            j->kind = kind; j->bits = bits; j->key_bytes = key_bytes; j->val_bytes = value_bytes;
            j->descending = descending; j->bit_start = bit_start; j->num_bits = num_bits;
            j->counts = &counts[(size_t)t * 256];
            j->phase = 0;
        }
        run_jobs(jobs, threads);
        uint64_t running = 0;
        for (int d = 0; d < 256; ++d)
            for (int t = 0; t < threads; ++t) {
                uint64_t c = counts[(size_t)t * 256 + d];
                counts[(size_t)t * 256 + d] = running;
                running += c;
            }
        for (int t = 0; t < threads; ++t) jobs[t].phase = 1;
        run_jobs(jobs, threads);
        ksrc = kdst;
        vsrc = vdst;
    }
    free(ktmp); free(vtmp); free(jobs); free(counts);
    return 0;
}

/* Digit of one key for one pass (exposed so tests can check the device
 * histogram without sorting). */
uint32_t oracle_digit(uint64_t key, int key_dtype, int descending, int bit_start, int num_bits)
{
    const int bits = dtype_bytes(key_dtype) * 8;
    return extract_digit(key, dtype_kind(key_dtype), bits, descending, bit_start, num_bits);
}

/* ---------------------------------------------------------------------------
 * Scan.  Restates DeviceScan's three forms (src/lcpp/device/device_scan.h:
 * 321-369): exclusive with an initial value, inclusive without, inclusive with
 * an initial value.  Integer arithmetic wraps (two's complement, computed in
 * unsigned).  mode: 0 exclusive, 1 inclusive, 2 inclusive with init.
 * ------------------------------------------------------------------------- */
#define SCAN_BODY(T, ACC_T, COMBINE)                                              \
    do {                                                                          \
        const T* in = (const T*)vin;                                              \
        T* out = (T*)vout;                                                        \
        ACC_T acc = init ? (ACC_T)(*(const T*)init) : (ACC_T)0;                   \
        int have = (mode != 1);                                                   \
        for (uint64_t i = 0; i < n; ++i) {                                        \
            ACC_T x = (ACC_T)in[i];                                               \
            if (mode == 0) {                                                      \
                out[i] = (T)acc;                                                  \
                acc = COMBINE(acc, x);                                            \
            } else {                                                              \
                acc = have ? COMBINE(acc, x) : x;                                 \
                have = 1;                                                         \
                out[i] = (T)acc;                                                  \
            }                                                                     \
        }                                                                         \
    } while (0)

#define C_SUM(a, b) ((a) + (b))
#define C_MIN(a, b) ((b) < (a) ? (b) : (a))
#define C_MAX(a, b) ((a) < (b) ? (b) : (a))

int oracle_scan(const void* vin, void* vout, uint64_t n, int dtype, int op, int mode,
                const void* init)
{
    if (mode < 0 || mode > 2 || op < 0 || op > 2) return -1;
    if (mode != 1 && !init) return -1;
    switch (dtype) {
    case DT_I32:
        if (op == OP_SUM) SCAN_BODY(uint32_t, uint32_t, C_SUM);
        else if (op == OP_MIN) SCAN_BODY(int32_t, int32_t, C_MIN);
        else SCAN_BODY(int32_t, int32_t, C_MAX);
        return 0;
    case DT_U32:
        if (op == OP_SUM) SCAN_BODY(uint32_t, uint32_t, C_SUM);
        else if (op == OP_MIN) SCAN_BODY(uint32_t, uint32_t, C_MIN);
        else SCAN_BODY(uint32_t, uint32_t, C_MAX);
        return 0;
    case DT_I64:
        if (op == OP_SUM) SCAN_BODY(uint64_t, uint64_t, C_SUM);
        else if (op == OP_MIN) SCAN_BODY(int64_t, int64_t, C_MIN);
        else SCAN_BODY(int64_t, int64_t, C_MAX);
        return 0;
    case DT_U64:
        if (op == OP_SUM) SCAN_BODY(uint64_t, uint64_t, C_SUM);
        else if (op == OP_MIN) SCAN_BODY(uint64_t, uint64_t, C_MIN);
        else SCAN_BODY(uint64_t, uint64_t, C_MAX);
        return 0;
    case DT_F32:
        if (op == OP_SUM) SCAN_BODY(float, float, C_SUM);
        else if (op == OP_MIN) SCAN_BODY(float, float, C_MIN);
        else SCAN_BODY(float, float, C_MAX);
        return 0;
    case DT_F64:
        if (op == OP_SUM) SCAN_BODY(double, double, C_SUM);
        else if (op == OP_MIN) SCAN_BODY(double, double, C_MIN);
        else SCAN_BODY(double, double, C_MAX);
        return 0;
    default:
        return -1;
    }
}

/* ---------------------------------------------------------------------------
 * Reduce.  Restates DeviceReduce::Reduce/Sum/Min/Max (src/lcpp/device/
 * device_reduce.h:229-308): out = init (+) in[0] (+) ... (+) in[n-1]; n == 0
 * gives init.  Integer sums wrap.  Floating-point sums are accumulated in
 * double here (the fp64 host sum the reference's float tolerance is measured
 * against) and rounded once to the element type.
 * ------------------------------------------------------------------------- */
#define RED_BODY(T, ACC_T, COMBINE)                                               \
    do {                                                                          \
        const T* in = (const T*)vin;                                              \
        ACC_T acc = (ACC_T)(*(const T*)init);                                     \
        for (uint64_t i = 0; i < n; ++i) acc = COMBINE(acc, (ACC_T)in[i]);        \
        *(T*)vout = (T)acc;                                                       \
    } while (0)

int oracle_reduce(const void* vin, void* vout, uint64_t n, int dtype, int op, const void* init)
{
    if (!init || op < 0 || op > 2) return -1;
    switch (dtype) {
    case DT_I32:
        if (op == OP_SUM) RED_BODY(uint32_t, uint32_t, C_SUM);
        else if (op == OP_MIN) RED_BODY(int32_t, int32_t, C_MIN);
        else RED_BODY(int32_t, int32_t, C_MAX);
        return 0;
    case DT_U32:
        if (op == OP_SUM) RED_BODY(uint32_t, uint32_t, C_SUM);
        else if (op == OP_MIN) RED_BODY(uint32_t, uint32_t, C_MIN);
        else RED_BODY(uint32_t, uint32_t, C_MAX);
        return 0;
    case DT_I64:
        if (op == OP_SUM) RED_BODY(uint64_t, uint64_t, C_SUM);
        else if (op == OP_MIN) RED_BODY(int64_t, int64_t, C_MIN);
        else RED_BODY(int64_t, int64_t, C_MAX);
        return 0;
    case DT_U64:
        if (op == OP_SUM) RED_BODY(uint64_t, uint64_t, C_SUM);
        else if (op == OP_MIN) RED_BODY(uint64_t, uint64_t, C_MIN);
        else RED_BODY(uint64_t, uint64_t, C_MAX);
        return 0;
    case DT_F32:
        if (op == OP_SUM) RED_BODY(float, double, C_SUM);
        else if (op == OP_MIN) RED_BODY(float, float, C_MIN);
        else RED_BODY(float, float, C_MAX);
        return 0;
    case DT_F64:
        if (op == OP_SUM) RED_BODY(double, long double, C_SUM);
        else if (op == OP_MIN) RED_BODY(double, double, C_MIN);
        else RED_BODY(double, double, C_MAX);
        return 0;
    default:
        return -1;
    }
}

/* ArgMin / ArgMax: the reference's fold with ArgMinOp / ArgMaxOp
 * (src/lcpp/common/thread_operators.h:19-47) from the identity pair
 * {UINT_MAX, max() or lowest()} (src/lcpp/device/device_reduce.h:346-353,
 * :412-418), taken in index order: item i replaces the best when its value
 * is smaller (larger), or equal with a smaller index -- so the result is the
 * first index of the extreme value.  A NaN compares false both ways and never
 * replaces the best (the reference's tree may keep a NaN it met first; NaN
 * inputs are outside the parity domain).  n == 0 writes the empty-input
 * sentinels max() / lowest() and index 1 (:318-323). */
#define ARG_BODY(T, IS_MIN, EMPTY)                                                   \
    do {                                                                             \
        const T* in = (const T*)vin;                                                 \
        T best = (EMPTY);                                                            \
        uint32_t bi = 0xffffffffu;                                                   \
        if (n == 0) {                                                                \
            *(T*)vout = best;                                                        \
            *index_out = 1u;                                                         \
            return 0;                                                                \
        }                                                                            \
        for (uint64_t i = 0; i < n; ++i) {                                           \
            const T x = in[i];                                                       \
            const int strictly = (IS_MIN) ? (x < best) : (x > best);                 \
            if (strictly || (x == best && (uint32_t)i < bi)) {                       \
                best = x;                                                            \
                bi = (uint32_t)i;                                                    \
            }                                                                        \
        }                                                                            \
        *(T*)vout = best;                                                            \
        *index_out = bi;                                                             \
    } while (0)

int oracle_arg_extremum(const void* vin, void* vout, uint32_t* index_out, uint64_t n, int dtype, int is_min)
{
    if (!vout || !index_out || n > 0xffffffffull) return -1;
    switch (dtype) {
    case DT_I32:
        if (is_min) ARG_BODY(int32_t, 1, INT32_MAX); else ARG_BODY(int32_t, 0, INT32_MIN);
        return 0;
    case DT_U32:
        if (is_min) ARG_BODY(uint32_t, 1, UINT32_MAX); else ARG_BODY(uint32_t, 0, 0u);
        return 0;
    case DT_I64:
        if (is_min) ARG_BODY(int64_t, 1, INT64_MAX); else ARG_BODY(int64_t, 0, INT64_MIN);
        return 0;
    case DT_U64:
        if (is_min) ARG_BODY(uint64_t, 1, UINT64_MAX); else ARG_BODY(uint64_t, 0, 0ull);
        return 0;
    case DT_F32:
        if (is_min) ARG_BODY(float, 1, FLT_MAX); else ARG_BODY(float, 0, -FLT_MAX);
        return 0;
    case DT_F64:
        if (is_min) ARG_BODY(double, 1, DBL_MAX); else ARG_BODY(double, 0, -DBL_MAX);
        return 0;
    default:
        return -1;
    }
}

/* Scans and reductions by key (src/lcpp/device/device_scan.h:425-597,
 * src/lcpp/device/device_reduce.h:437-491), sequentially: a segment (run) is
 * a maximal stretch of consecutive items whose keys compare equal with ==
 * at the key's type (BlockDiscontinuity::FlagHeads with `a != b`,
 * details/reduce_by_key.h).  Integer sums wrap (computed unsigned). */
static void key_heads(const void* keys, int kdt, uint64_t n, uint8_t* heads)
{
    for (uint64_t i = 0; i < n; ++i) {
        int h = i == 0;
        if (!h) {
            switch (kdt) {
            case DT_U32: case DT_I32: h = ((const uint32_t*)keys)[i] != ((const uint32_t*)keys)[i - 1]; break;
            case DT_U64: case DT_I64: h = ((const uint64_t*)keys)[i] != ((const uint64_t*)keys)[i - 1]; break;
            case DT_F32: h = ((const float*)keys)[i] != ((const float*)keys)[i - 1]; break;
            default: h = ((const double*)keys)[i] != ((const double*)keys)[i - 1]; break;
            }
        }
        heads[i] = (uint8_t)h;
    }
}

/* mode 0: exclusive with init, 1: inclusive, 2: inclusive with init */
#define SBK_BODY(T, ACC_T, COMBINE)                                                   \
    do {                                                                              \
        const T* in = (const T*)vin;                                                  \
        T* out = (T*)vout;                                                            \
        const ACC_T init = init_p ? (ACC_T)(*(const T*)init_p) : (ACC_T)0;            \
        ACC_T run = 0;                                                                \
        for (uint64_t i = 0; i < n; ++i) {                                            \
            const ACC_T x = (ACC_T)in[i];                                             \
            if (mode == 0) {                                                          \
                if (heads[i]) { out[i] = (T)init; run = x; }                          \
                else { out[i] = (T)COMBINE(init, run); run = COMBINE(run, x); }       \
            } else {                                                                  \
                run = heads[i] ? x : COMBINE(run, x);                                 \
                out[i] = (T)(mode == 2 ? COMBINE(init, run) : run);                   \
            }                                                                         \
        }                                                                             \
    } while (0)

#define BY_VALUE_TYPE(BODY)                                                           \
    switch (vdt) {                                                                    \
    case DT_I32:                                                                      \
        if (op == OP_SUM) BODY(uint32_t, uint32_t, C_SUM);                            \
        else if (op == OP_MIN) BODY(int32_t, int32_t, C_MIN);                         \
        else BODY(int32_t, int32_t, C_MAX);                                           \
        break;                                                                        \
    case DT_U32:                                                                      \
        if (op == OP_SUM) BODY(uint32_t, uint32_t, C_SUM);                            \
        else if (op == OP_MIN) BODY(uint32_t, uint32_t, C_MIN);                       \
        else BODY(uint32_t, uint32_t, C_MAX);                                         \
        break;                                                                        \
    case DT_I64:                                                                      \
        if (op == OP_SUM) BODY(uint64_t, uint64_t, C_SUM);                            \
        else if (op == OP_MIN) BODY(int64_t, int64_t, C_MIN);                         \
        else BODY(int64_t, int64_t, C_MAX);                                           \
        break;                                                                        \
    case DT_U64:                                                                      \
        if (op == OP_SUM) BODY(uint64_t, uint64_t, C_SUM);                            \
        else if (op == OP_MIN) BODY(uint64_t, uint64_t, C_MIN);                       \
        else BODY(uint64_t, uint64_t, C_MAX);                                         \
        break;                                                                        \
    case DT_F32:                                                                      \
        if (op == OP_SUM) BODY(float, float, C_SUM);                                  \
        else if (op == OP_MIN) BODY(float, float, C_MIN);                             \
        else BODY(float, float, C_MAX);                                               \
        break;                                                                        \
    default:                                                                          \
        if (op == OP_SUM) BODY(double, double, C_SUM);                                \
        else if (op == OP_MIN) BODY(double, double, C_MIN);                           \
        else BODY(double, double, C_MAX);                                             \
        break;                                                                        \
    }

int oracle_scan_by_key(const void* keys, const void* vin, void* vout, uint64_t n, int kdt, int vdt, int op,
                       int mode, const void* init_p)
{
    if (kdt < 0 || kdt > 5 || vdt < 0 || vdt > 5 || op < 0 || op > 2 || mode < 0 || mode > 2) return -1;
    if (mode != 1 && !init_p) return -1;
    if (n == 0) return 0;
    uint8_t* heads = (uint8_t*)malloc(n);
    if (!heads) return -2;
    key_heads(keys, kdt, n, heads);
    BY_VALUE_TYPE(SBK_BODY)
    free(heads);
    return 0;
}

#define RBK_BODY(T, ACC_T, COMBINE)                                                   \
    do {                                                                              \
        const T* in = (const T*)vin;                                                  \
        T* agg = (T*)vagg;                                                            \
        ACC_T run = 0;                                                                \
        uint64_t r = 0;                                                               \
        for (uint64_t i = 0; i < n; ++i) {                                            \
            const ACC_T x = (ACC_T)in[i];                                             \
            if (heads[i]) {                                                           \
                if (i > 0) agg[r++] = (T)run;                                         \
                memcpy((unsigned char*)unique_out + r * kb, (const unsigned char*)keys + i * kb, kb); \
                run = x;                                                              \
            } else {                                                                  \
                run = COMBINE(run, x);                                                \
            }                                                                         \
        }                                                                             \
        agg[r++] = (T)run;                                                            \
        *num_runs = (uint32_t)r;                                                      \
    } while (0)

int oracle_reduce_by_key(const void* keys, const void* vin, void* unique_out, void* vagg, uint32_t* num_runs,
                         uint64_t n, int kdt, int vdt, int op)
{
    if (kdt < 0 || kdt > 5 || vdt < 0 || vdt > 5 || op < 0 || op > 2 || !num_runs) return -1;
    if (n == 0) {
        *num_runs = 0;
        return 0;
    }
    const size_t kb = (kdt == DT_U32 || kdt == DT_I32 || kdt == DT_F32) ? 4 : 8;
    uint8_t* heads = (uint8_t*)malloc(n);
    if (!heads) return -2;
    key_heads(keys, kdt, n, heads);
    BY_VALUE_TYPE(RBK_BODY)
    free(heads);
    return 0;
}

/* fp64 sum of a float32 or float64 array: the reference value for the float
 * reduce tolerance 1e-6 * log2(n) (relative). */
double oracle_sum_f64(const void* vin, uint64_t n, int dtype)
{
    long double acc = 0.0L;
    if (dtype == DT_F32) {
        const float* in = (const float*)vin;
        for (uint64_t i = 0; i < n; ++i) acc += (long double)in[i];
    } else {
        const double* in = (const double*)vin;
        for (uint64_t i = 0; i < n; ++i) acc += (long double)in[i];
    }
    return (double)acc;
}

/* ---------------------------------------------------------------------------
 * Counter-based input generators (independent host restatement of the
 * library's synthetic-input kernels; used to check them and to build inputs
 * for CPU-only tests).  r(seed, stream, i) = splitmix64(seed*2^40 +
 * stream*2^36 + i), splitmix64 being Vigna's public-domain finaliser of the
 * SplitMix generator (Steele, Lea & Flood, OOPSLA 2014).
 * ------------------------------------------------------------------------- */
static inline uint64_t splitmix64(uint64_t x)
{
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static inline uint64_t counter_rand(uint64_t seed, uint64_t stream, uint64_t i)
{
    return splitmix64((seed << 40) + (stream << 36) + i);
}

/* dist codes match lcpp_testgen_dist in the library's testgen.h. */
enum {
    GEN_U32_UNIFORM = 0,
    GEN_U32_AND3 = 1,
    GEN_U32_CONST = 2,
    GEN_U64_UNIFORM = 3,
    GEN_I32_SCAN = 4,     /* (r % 2001) - 1000 */
    GEN_F32_UNIT = 5,     /* (r >> 40) * 2^-24 */
    GEN_I64_UNIFORM = 6,
    GEN_U32_INDEX = 7     /* i (values = original index) */
};

int oracle_generate(void* out, uint64_t n, uint64_t offset, uint64_t seed, int dist)
{
    for (uint64_t j = 0; j < n; ++j) {
        const uint64_t i = offset + j;
        switch (dist) {
        case GEN_U32_UNIFORM: ((uint32_t*)out)[j] = (uint32_t)counter_rand(seed, 0, i); break;
        case GEN_U32_AND3:
            ((uint32_t*)out)[j] = (uint32_t)(counter_rand(seed, 0, i) & counter_rand(seed, 1, i) &
                                             counter_rand(seed, 2, i));
            break;
        case GEN_U32_CONST: ((uint32_t*)out)[j] = 0x9E3779B9u; break;
        case GEN_U64_UNIFORM: ((uint64_t*)out)[j] = counter_rand(seed, 0, i); break;
        case GEN_I32_SCAN: ((int32_t*)out)[j] = (int32_t)(counter_rand(seed, 0, i) % 2001ull) - 1000; break;
        case GEN_F32_UNIT:
            ((float*)out)[j] = (float)(counter_rand(seed, 0, i) >> 40) * (1.0f / 16777216.0f);
            break;
        case GEN_I64_UNIFORM: ((int64_t*)out)[j] = (int64_t)counter_rand(seed, 0, i); break;
        case GEN_U32_INDEX: ((uint32_t*)out)[j] = (uint32_t)i; break;
        default: return -1;
        }
    }
    return 0;
}
