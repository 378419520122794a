// noalloc.cu -- an InclusiveSum entry point that needs no caller scratch.
//
// Some callers cannot allocate device memory when they want to scan: code
// running inside a custom allocator or a memory-pool callback (allocating
// would re-enter it), a plugin host that hands the plugin fixed buffers and
// no allocation rights, or a real-time loop that must not call cudaMalloc
// (it may synchronise the device) after start-up.  For them this file keeps
// the scan's scratch in a statically sized device array instead of caller
// temp storage.  Nothing here calls cudaMalloc, cudaFree or any allocating
// library routine.
//
// The array is file-scope device memory of the library image: every GPU that
// loads the library holds it until the process exits, and every call on a
// device shares that device's copy.  Its host-side name is only a stand-in,
// so host code passes the device address obtained with cudaGetSymbolAddress.
// That address belongs to the device's current context: it is cached per
// device together with the context's unique ID and looked up again when the
// ID changes (after cudaDeviceReset the library image is loaded again and
// the array may sit elsewhere).
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "scan.cuh"

namespace lcpp {
namespace noalloc {

// 2 MiB + 4 KiB: holds the scan's control block and tile status words for up
// to 1,075,707,904 items of a 4-byte type (a little above 2^30) or
// 215,089,152 items of an 8-byte type.
constexpr size_t kScratchBytes = (2u << 20) + 4096;

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

namespace {

std::mutex g_mu;
struct Cached {
    unsigned long long ctx_id;  // 0: nothing cached
    void* addr;
};
Cached g_cache[64] = {};
PFN_cuCtxGetCurrent g_get_current = nullptr;
PFN_cuCtxGetId g_get_id = nullptr;

// Unique ID of the calling thread's current context, 0 when there is none.
// The two driver functions come through the runtime's entry-point query, so
// the library needs no link-time dependency on the driver library.
unsigned long long current_context_id()
{
    if (!g_get_current || !g_get_id) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_get_current = reinterpret_cast<PFN_cuCtxGetCurrent>(f);
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_get_id = reinterpret_cast<PFN_cuCtxGetId>(f);
        if (!g_get_current || !g_get_id) return 0;
    }
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (g_get_current(&ctx) != CUDA_SUCCESS || !ctx) return 0;
    if (g_get_id(ctx, &id) != CUDA_SUCCESS) return 0;
    return id;
}

// Device address of g_scratch on the current device, with that device
// current: looked up at the first call on the device and again whenever the
// device's context has changed since, else taken from the cache.
cudaError_t scratch_address(void** out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_mu);
    const unsigned long long id = current_context_id();
    if (id == 0 || g_cache[dev].ctx_id != id) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_scratch);  // creates the primary context if none is current
        if (e != cudaSuccess) return e;
        g_cache[dev] = Cached{current_context_id(), p};
    }
    *out = g_cache[dev].addr;
    return cudaSuccess;
}

}  // namespace
}  // namespace noalloc
}  // namespace lcpp

extern "C" lcpp_status lcpp_scan_inclusive_sum_noalloc(const void* d_in, void* d_out, uint64_t num_items,
                                                       lcpp_dtype dtype, lcpp_stream_t stream)
{
    using namespace lcpp;
    if (!dtype_bytes(dtype)) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (num_items == 0) return LCPP_OK;
    // Reject sizes whose scratch would not fit the static array (checked on
    // the host before any device work).
    if (scan::temp_bytes(dtype, num_items) > noalloc::kScratchBytes) return LCPP_ERR_TEMP_TOO_SMALL;
    void* scratch = nullptr;
    if (noalloc::scratch_address(&scratch) != cudaSuccess) {
        cudaGetLastError();
        return LCPP_ERR_CUDA;
    }
    // The scan clears the control block and status words it uses at the
    // start of every call, so the previous call's contents do not matter.
    return scan::run(scratch, noalloc::kScratchBytes, d_in, d_out, num_items, LCPP_OP_SUM, nullptr, dtype, 1,
                     reinterpret_cast<cudaStream_t>(stream));
}
