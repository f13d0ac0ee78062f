// static_solve.cu — pp_lmul_static: lmul! on device-resident right-hand sides that allocates nothing.
//
// The scratch of the solve (the right-hand sides in the device layout X[position][rhs] and the counters of
// the persistent sweeps) lives in one file-scope device array of PP_STATIC_SCRATCH_BYTES, which the CUDA
// runtime places on each device when it loads this library's device image there.  Its address is looked up
// once per device (the first call with that device current) and then passed to the solve like any other
// device pointer.  The solve is the one pp_lmul runs, on the same kernels, so the results are the same.
#include <mutex>

#include <cuda_runtime.h>

#include "pathpack_b200_internal.h"

namespace {

constexpr size_t kScratchBytes = (size_t)PP_STATIC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_static_scratch[kScratchBytes];

std::mutex g_setup_mutex;
void *g_scratch_addr[kMaxDevices] = {};

// the array's address on `device` (which is current), looked up on first use
int32_t scratch_address(int device, void **out) {
    if (device < 0 || device >= kMaxDevices) return PP_EINVAL;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_addr[device]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p) return PP_EDEVICE;
        g_scratch_addr[device] = p;
    }
    *out = g_scratch_addr[device];
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
    const int32_t rc = scratch_address(device, &scratch);
    if (rc != PP_OK)
        return pp_internal_fail(h, rc, "pp_lmul_static: no device address for the static scratch array");
    return pp_internal_lmul_scratch(h, B, ldb, k, scratch, kScratchBytes, who);
}
