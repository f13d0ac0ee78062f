// pathpack_b200_internal.h — shared between the library's translation units.
#pragma once

#include <cstddef>

#include "pathpack_b200.h"

#define PP_INTERNAL __attribute__((visibility("hidden")))

// lmul! on device-resident B (n x k, leading dimension ldb) using `scratch` (cap bytes of device memory)
// for the right-hand-side workspace and the sweep counters instead of the handle's own buffers; allocates
// nothing.  Fails with PP_EINVAL when cap is below pp_internal_lmul_scratch_bytes(h, k).
PP_INTERNAL int32_t pp_internal_lmul_scratch(pp_handle *h, void *B, int64_t ldb, int64_t k, void *scratch, size_t cap,
                                             const char *who);
PP_INTERNAL size_t pp_internal_lmul_scratch_bytes(const pp_handle *h, int64_t k);
// the handle's device; an error return that records `msg` as the handle's last error
PP_INTERNAL int32_t pp_internal_device(const pp_handle *h, int *device);
PP_INTERNAL int32_t pp_internal_fail(pp_handle *h, int32_t code, const char *msg);
// the element size of the handle's semiring and type (0 before pp_assemble / pp_set_values)
PP_INTERNAL size_t pp_internal_esize(const pp_handle *h);
