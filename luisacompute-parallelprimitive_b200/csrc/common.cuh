// common.cuh -- shared device helpers for the sm_100a sort / scan / reduce
// kernels: dtype plumbing, relaxed GPU-scope status-word access, bounded
// waits and the radix key bijection.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <type_traits>

#include <nvtx3/nvToolsExt.h>

#include "../../include/lcpp_b200.h"

namespace lcpp {

constexpr int kWarp = 32;
constexpr size_t kTempAlign = 256;  // every temp sub-buffer starts 256-B aligned

__host__ __device__ constexpr size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
__host__ __device__ constexpr uint64_t ceil_div(uint64_t a, uint64_t b) { return (a + b - 1) / b; }

inline int dtype_bytes(lcpp_dtype dt)
{
    switch (dt) {
    case LCPP_U32: case LCPP_I32: case LCPP_F32: return 4;
    case LCPP_U64: case LCPP_I64: case LCPP_F64: return 8;
    default: return 0;
    }
}

// Device-side error word values (written into temp storage; read back by
// lcpp_device_status).
constexpr uint32_t kDevErrTimeout = LCPP_ERR_LOOKBACK_TIMEOUT;
constexpr uint32_t kDevErrInternal = LCPP_ERR_INTERNAL;

// A bounded wait gives up after this many nanoseconds of %globaltimer.  A
// legitimate wait in these kernels is a few microseconds (one predecessor
// tile publishing its partial); the bound only exists so that a broken
// protocol reports an error instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 4000000000ull;

__device__ __forceinline__ uint64_t global_timer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t lanemask_lt()
{
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// Relaxed GPU-scope loads / stores of self-contained status words: each word
// carries its own flag and value, so no ordering with other data is needed.
__device__ __forceinline__ uint32_t ld_relaxed(const uint32_t* p)
{
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t ld_relaxed(const uint64_t* p)
{
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed(uint32_t* p, uint32_t v)
{
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed(uint64_t* p, uint64_t v)
{
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Non-zero once any thread of the call recorded an error.
__device__ __forceinline__ bool error_raised(const uint32_t* err)
{
    return err && ld_relaxed(err) != 0u;
}

// Record a device error once (first writer wins).
__device__ __forceinline__ void report_error(uint32_t* err, uint32_t code)
{
    if (err) atomicCAS(err, 0u, code);
}

// ---------------------------------------------------------------------------
// Radix key bijection.
//
// The reference maps keys to order-preserving unsigned bits with
// Traits<T>::TwiddleIn (src/lcpp/common/util_type.h:97-175), inverts them for
// descending order (src/lcpp/agent/radix_rank_sort_operations.h:123-155) and
// folds -0.0 onto +0.0 before extracting digits (same file, :31-43).  All
// three key kinds and both directions reduce to one formula with two XOR
// masks chosen by the key's sign bit, so one kernel serves every key dtype of
// a given width:
//   unsigned : pos = neg = 0            (descending: ~0)
//   signed   : pos = neg = HIGH         (descending: ~HIGH)
//   float    : pos = HIGH, neg = ~0     (descending: ~HIGH, 0)
// For float keys the reference's fold gives +-0.0 the digits of HIGH in both
// directions (the transformed +0.0 ascending, the folded value descending);
// the kernels apply it when extracting digits only, so stored keys keep
// their bits.
// ---------------------------------------------------------------------------
template <typename U>
struct KeyCodec {
    U xor_pos;
    U xor_neg;
    uint32_t fold_zero;  // 1 for floating-point keys
};

template <typename U>
inline KeyCodec<U> make_codec(lcpp_dtype dt, bool descending)
{
    constexpr int kBits = sizeof(U) * 8;
    constexpr U kHigh = U(1) << (kBits - 1);
    KeyCodec<U> c{};
    switch (dt) {
    case LCPP_I32: case LCPP_I64: c.xor_pos = kHigh; c.xor_neg = kHigh; break;
    case LCPP_F32: case LCPP_F64: c.xor_pos = kHigh; c.xor_neg = U(~U(0)); c.fold_zero = 1; break;
    default: c.xor_pos = 0; c.xor_neg = 0; break;
    }
    if (descending) {
        c.xor_pos = U(~c.xor_pos);
        c.xor_neg = U(~c.xor_neg);
    }
    return c;
}

// ---------------------------------------------------------------------------
// Shared-memory and warp primitives of the ranking loops (inline PTX).
// ---------------------------------------------------------------------------
// Predicated shared-memory atomic add: returns the old value when `pred`,
// else 0, without a branch.
__device__ __forceinline__ uint32_t shared_add_if(bool pred, uint32_t smem_addr, uint32_t inc)
{
    uint32_t old = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "@p atom.shared.add.u32 %0, [%2], %3;\n\t}"
        : "+r"(old)
        : "r"(uint32_t(pred)), "r"(smem_addr), "r"(inc)
        : "memory");
    return old;
}

// Fire-and-forget shared-memory OR.
__device__ __forceinline__ void shared_red_or(uint32_t smem_addr, uint32_t bits)
{
    asm volatile("red.shared.or.b32 [%0], %1;" ::"r"(smem_addr), "r"(bits) : "memory");
}

__device__ __forceinline__ uint32_t shared_load(uint32_t smem_addr)
{
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_addr) : "memory");
    return v;
}

__device__ __forceinline__ void shared_store_if(bool pred, uint32_t smem_addr, uint32_t v)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.u32 p, %0, 0;\n\t"
        "@p st.shared.u32 [%1], %2;\n\t}" ::"r"(uint32_t(pred)), "r"(smem_addr), "r"(v)
        : "memory");
}

// Fire-and-forget shared-memory add.
__device__ __forceinline__ void shared_red_add(uint32_t smem_addr, uint32_t inc)
{
    asm volatile("red.shared.add.u32 [%0], %1;" ::"r"(smem_addr), "r"(inc) : "memory");
}

// Full-warp ballot and warp barrier written as PTX (vote.sync /
// bar.warp.sync with the full member mask).
__device__ __forceinline__ uint32_t warp_ballot(bool pred)
{
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "vote.sync.ballot.b32 %0, p, 0xffffffff;\n\t}"
        : "=r"(r)
        : "r"(uint32_t(pred)));
    return r;
}

__device__ __forceinline__ void warp_barrier() { asm volatile("bar.warp.sync 0xffffffff;" ::: "memory"); }

__device__ __forceinline__ uint32_t warp_shfl(uint32_t v, int src)
{
    uint32_t r;
    asm volatile("shfl.sync.idx.b32 %0, %1, %2, 0x1f, 0xffffffff;" : "=r"(r) : "r"(v), "r"(src));
    return r;
}

// Cached per-device SM count (grid sizing in multiples of the SM count).
int device_sm_count();

// Raise a kernel's dynamic shared-memory limit on the current device (once
// per kernel, device and size).
void set_max_dynamic_smem(const void* kernel, size_t bytes);

// Resident blocks per SM of a kernel at this block size and dynamic shared
// memory on the current device (cached; at least 1).
int resident_blocks(const void* kernel, int block, size_t dynamic_smem);

namespace diag {
// Names the host-side extent of one library call in profiler timelines
// (NVTX; header-only, close to free when no profiler is attached).
class Range {
public:
    explicit Range(const char* name) { nvtxRangePushA(name); }
    ~Range() { nvtxRangePop(); }
    Range(const Range&) = delete;
    Range& operator=(const Range&) = delete;
};

// Brackets one kernel launch with CUDA events when timing is enabled
// (lcpp_diag_timing_enable); otherwise a no-op.
class KernelTimer {
public:
    KernelTimer(int kind, uint64_t items, cudaStream_t stream);
    void stop();
    ~KernelTimer() { stop(); }

private:
    int index_;
    cudaStream_t stream_;
};
}  // namespace diag

}  // namespace lcpp

#define LCPP_CUDA_TRY(expr)                              \
    do {                                                 \
        cudaError_t _e = (expr);                         \
        if (_e != cudaSuccess) return LCPP_ERR_CUDA;     \
    } while (0)
