// static_solve.cu — pp_lmul_static: lmul! on device-resident right-hand sides that allocates nothing.
//
// The scratch of the solve (the right-hand sides in the device layout X[position][rhs] and the counters of
// the persistent sweeps) lives in one file-scope device array of PP_STATIC_SCRATCH_BYTES.  In host code the
// array's name is only a host-side stand-in, so every call asks the CUDA runtime for the array's address on
// the current device (cudaGetSymbolAddress) and passes that address to the solve like any other device
// pointer.  Looking it up per call, rather than caching it, stays correct when the caller's context is torn
// down and created again.  Under lazy module loading (the CUDA 12 default) the runtime places the library's
// device code, and with it the array, on a device at the first lookup there.  The solve is the one pp_lmul
// runs, on the same kernels, so the results are the same.
#include <cuda_runtime.h>

#include "pathpack_b200_internal.h"

namespace {

constexpr size_t kScratchBytes = (size_t)PP_STATIC_SCRATCH_BYTES;

static __device__ __align__(256) unsigned char g_static_scratch[kScratchBytes];

// the array's address on the current device
int32_t scratch_address(void **out) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p) {
        cudaGetLastError();
        return PP_EDEVICE;
    }
    *out = p;
    return PP_OK;
}

}  // namespace

extern "C" int32_t pp_lmul_static(pp_handle *h, void *B, int64_t ldb, int64_t k) {
    const char *who = "pp_lmul_static";
    int device = -1;
    // a null handle, a missing factorization and a size beyond the array are reported by the solve's own
    // checks, which run before any device work
    if (!h || pp_internal_device(h, &device) != PP_OK || pp_internal_lmul_scratch_bytes(h, k) > kScratchBytes)
        return pp_internal_lmul_scratch(h, B, ldb, k, nullptr, kScratchBytes, who);
    if (cudaSetDevice(device) != cudaSuccess)
        return pp_internal_fail(h, PP_EDEVICE, "pp_lmul_static: cudaSetDevice failed");
    void *scratch = nullptr;
    const int32_t rc = scratch_address(&scratch);
    if (rc != PP_OK)
        return pp_internal_fail(h, rc, "pp_lmul_static: no device address for the static scratch array");
    return pp_internal_lmul_scratch(h, B, ldb, k, scratch, kScratchBytes, who);
}
