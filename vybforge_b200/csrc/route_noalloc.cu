// vfmoe_route_noalloc: the router with no device allocation anywhere on its path.
//
// Who needs it: hosts that cannot call cudaMalloc when they route.  cudaMalloc may
// synchronize the whole device, which stalls a latency-critical decode loop, and it fails
// outright once a host has already carved all of device memory into its own pool (the
// reference's drivers size every device buffer up front with cuMemAlloc_v2 and hand out
// sub-ranges).  vfmoe_route needs a caller workspace or grows an internal one;
// this entry point needs neither.
//
// Its scratch (router logit partials + per-expert counts) is the file-scope device array
// below: VFMOE_ROUTE_NOALLOC_SCRATCH_BYTES on every GPU that loads libvfmoe.so, held until
// the process exits.  Host code cannot use the array's name as a device address, so the
// first call on each device (with that device current) fetches the address with
// cudaGetSymbolAddress and caches it together with the device's current context; make that
// first call before any stream capture.  If the context changes (cudaDeviceReset tears the
// primary context down and the module, and with it the array, is loaded again), the next call
// fetches the address again.  The call must be made with the layer's own device current.
// All calls share the one array and it keeps the last call's contents: the counts are
// cleared on every call, and calls whose kernels overlap on the GPU (different streams,
// different threads) race on the array.
#include <cuda.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace vfmoe {

int route_into_scratch(int64_t handle, int64_t x, int64_t T, int64_t idx_out, int64_t w_out, char *scratch,
                       int64_t scratch_bytes, int64_t stream);

static __device__ __align__(256) unsigned char g_route_scratch[VFMOE_ROUTE_NOALLOC_SCRATCH_BYTES];

static std::mutex g_scratch_mu;
static void *g_scratch_addr[256];     // per device ordinal
static CUcontext g_scratch_ctx[256];  // the context the address belongs to

typedef CUresult (*CtxGetCurrentFn)(CUcontext *);

// The calling thread's current driver context (fetched through the runtime's driver entry
// point; the library does not link libcuda).  nullptr if it cannot be read.
static CUcontext current_context() {
    static CtxGetCurrentFn fn = []() -> CtxGetCurrentFn {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<CtxGetCurrentFn>(ptr);
        return nullptr;
    }();
    CUcontext c = nullptr;
    if (!fn || fn(&c) != CUDA_SUCCESS) return nullptr;
    return c;
}

static int scratch_address(void **out) {
    int dev = 0;
    VF_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 256) {
        set_error("vfmoe_route_noalloc: device ordinal %d out of range", dev);
        return VFMOE_ERR_INVALID;
    }
    // No context current on this thread yet (nullptr): the set-up below makes the runtime's
    // context current, and the address is cached against that context.
    CUcontext ctx = current_context();
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_addr[dev] || !ctx || ctx != g_scratch_ctx[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_route_scratch);
        if (e != cudaSuccess || !p) {
            set_error("vfmoe_route_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                      cudaGetErrorString(e));
            return VFMOE_ERR_CUDA;
        }
        if (!ctx) ctx = current_context();
        g_scratch_addr[dev] = p;
        g_scratch_ctx[dev] = ctx;
    }
    *out = g_scratch_addr[dev];
    return VFMOE_OK;
}

}  // namespace vfmoe

extern "C" int vfmoe_route_noalloc(int64_t handle, int64_t x, int64_t T, int64_t idx_out, int64_t w_out,
                                   int64_t stream) {
    using namespace vfmoe;
    if (T < 0 || (T > 0 && (!x || !idx_out || !w_out))) {
        set_error("vfmoe_route_noalloc: bad arguments");
        return VFMOE_ERR_INVALID;
    }
    if (T == 0) return VFMOE_OK;
    void *scratch = nullptr;
    const int rc = scratch_address(&scratch);
    if (rc) return rc;
    return route_into_scratch(handle, x, T, idx_out, w_out, reinterpret_cast<char *>(scratch),
                              VFMOE_ROUTE_NOALLOC_SCRATCH_BYTES, stream);
}
