"""ctypes binding of libpathpack_b200.so (the C ABI declared in include/pathpack_b200.h).

The library is the product: there is no CPU fallback.  Loading fails loudly when the shared library is
missing; calls that need a GPU return PP_EDEVICE on a machine without one.
"""
import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIBPATH = os.environ.get("PATHPACK_B200_LIB", os.path.join(os.path.dirname(_HERE), "lib", "libpathpack_b200.so"))

PP_OK, PP_EINVAL, PP_EUNSUPPORTED, PP_ENOMEM, PP_EDEVICE, PP_ETIMEOUT, PP_ESTATE = 0, -1, -2, -3, -4, -5, -6
PP_HOST, PP_DEVICE = 0, 1
ERRNAMES = {PP_EINVAL: "EINVAL", PP_EUNSUPPORTED: "EUNSUPPORTED", PP_ENOMEM: "ENOMEM", PP_EDEVICE: "EDEVICE",
            PP_ETIMEOUT: "ETIMEOUT", PP_ESTATE: "ESTATE"}


class PPError(RuntimeError):
    """A failed call of the C ABI: `code` is the PP_E* status."""

    def __init__(self, code, msg):
        super().__init__("%s (%s)" % (msg, ERRNAMES.get(code, code)))
        self.code = code


class pp_stats(C.Structure):
    _fields_ = [("n", C.c_int64), ("nf", C.c_int64), ("nB", C.c_int64), ("nlevels", C.c_int64),
                ("nD", C.c_int64), ("nL", C.c_int64), ("nN", C.c_int64), ("max_front", C.c_int64),
                ("pairs_factor", C.c_double), ("ms_factor", C.c_double), ("ms_solve", C.c_double),
                ("pairs_solve", C.c_double), ("device_bytes", C.c_int64), ("kernel_launches", C.c_int64),
                ("plan_fronts", C.c_int64)]


class pp_options(C.Structure):
    _fields_ = [("wait_timeout_us", C.c_int64), ("fail_alloc_after", C.c_int64), ("profile", C.c_int32),
                ("merge_width", C.c_int32), ("trace", C.c_int32), ("reserved", C.c_int32)]


class pp_kernel_class(C.Structure):
    _fields_ = [("name", C.c_char * 32), ("launches", C.c_int64), ("ms", C.c_double), ("bytes", C.c_double),
                ("pairs", C.c_double)]


# every symbol the header declares, with its ctypes signature
_P = C.c_void_p
_I64P = C.POINTER(C.c_int64)
SIGNATURES = {
    "pp_version": (C.c_int32, []),
    "pp_check_semiring": (C.c_int32, [C.c_int32, C.c_int32]),
    "pp_last_error": (C.c_char_p, [_P]),
    "pp_create": (C.c_int32, [C.c_int32, C.POINTER(_P)]),
    "pp_destroy": (C.c_int32, [_P]),
    "pp_default_options": (None, [C.c_void_p]),
    "pp_create_with": (C.c_int32, [C.c_int32, C.c_void_p, C.POINTER(_P)]),
    "pp_set_options": (C.c_int32, [_P, C.c_void_p]),
    "pp_get_options": (C.c_int32, [_P, C.c_void_p]),
    "pp_set_structure": (C.c_int32, [_P, C.c_int64, C.c_int64, C.c_int64] + [_I64P] * 8 + [C.c_int32]),
    "pp_assemble": (C.c_int32, [_P, C.c_int32, C.c_int32, _I64P, _I64P, _P, C.c_int32]),
    "pp_update_values": (C.c_int32, [_P, _P, C.c_int32]),
    "pp_set_values": (C.c_int32, [_P, C.c_int32, C.c_int32, _P, _P, _P, _P, _P]),
    "pp_factor": (C.c_int32, [_P]),
    "pp_get_factor": (C.c_int32, [_P, _P, _P, _P, _P]),
    "pp_lmul": (C.c_int32, [_P, _P, C.c_int64, C.c_int64, C.c_int32]),
    "pp_rmul": (C.c_int32, [_P, _P, C.c_int64, C.c_int64, C.c_int32]),
    "pp_lmul_t": (C.c_int32, [_P, _P, C.c_int64, C.c_int64, C.c_int32]),
    "pp_rmul_t": (C.c_int32, [_P, _P, C.c_int64, C.c_int64, C.c_int32]),
    "pp_lmul_static": (C.c_int32, [_P, _P, C.c_int64, C.c_int64]),
    "pp_star": (C.c_int32, [_P, _P, C.c_int64, C.c_int64, C.c_int64, C.c_int32]),
    "pp_sync": (C.c_int32, [_P]),
    "pp_star_cols": (C.c_int32, [_P, _P, C.c_int64, _I64P, C.c_int64, C.c_int32]),
    "pp_star_rows": (C.c_int32, [_P, _P, C.c_int64, _I64P, C.c_int64, C.c_int32]),
    "pp_comm_id": (C.c_int32, [C.c_void_p]),
    "pp_comm_init": (C.c_int32, [_P, C.c_void_p, C.c_int32, C.c_int32]),
    "pp_multi_create": (C.c_int32, [C.POINTER(C.c_int32), C.c_int32, C.c_void_p, C.POINTER(_P)]),
    "pp_multi_destroy": (C.c_int32, [_P]),
    "pp_multi_handle": (C.c_int32, [_P, C.c_int32, C.POINTER(_P)]),
    "pp_multi_set_structure": (C.c_int32, [_P, C.c_int64, C.c_int64, C.c_int64] + [_I64P] * 8 + [C.c_int32]),
    "pp_multi_assemble": (C.c_int32, [_P, C.c_int32, C.c_int32, _I64P, _I64P, _P, C.c_int32]),
    "pp_multi_factor": (C.c_int32, [_P]),
    "pp_multi_lmul": (C.c_int32, [_P, _P, C.c_int64, C.c_int64, C.c_int32]),
    "pp_multi_rmul": (C.c_int32, [_P, _P, C.c_int64, C.c_int64, C.c_int32]),
    "pp_multi_star": (C.c_int32, [_P, _P, C.c_int64, C.c_int64, C.c_int64]),
    "pp_plan_lmul": (C.c_int32, [_P, _P, _P, _P, C.c_int64, C.c_int64, C.POINTER(_P)]),
    "pp_plan_launch": (C.c_int32, [_P]),
    "pp_plan_launches": (C.c_int32, [_P, C.POINTER(C.c_int64)]),
    "pp_plan_destroy": (C.c_int32, [_P]),
    "pp_get_stats": (C.c_int32, [_P, C.POINTER(pp_stats)]),
    "pp_get_trace": (C.c_int32, [_P, C.c_void_p, C.c_int64, C.POINTER(C.c_int64)]),
    "pp_stream": (_P, [_P]),
    "pp_set_profile": (C.c_int32, [_P, C.c_int32]),
    "pp_get_profile": (C.c_int32, [_P, C.POINTER(pp_kernel_class), C.c_int32, C.POINTER(C.c_int32)]),
    "pp_gemm": (C.c_int32, [C.c_int32, C.c_int32, C.c_int64, C.c_int64, C.c_int64, _P, C.c_int64, _P, C.c_int64,
                            _P, C.c_int64, _P]),
    "pp_getrf_batched": (C.c_int32, [C.c_int32, C.c_int32, C.c_int64, C.c_int64, _P, _P]),
    "pp_symbolic": (C.c_int32, [C.c_int64, _I64P, _I64P, C.c_int32, C.c_int32, C.POINTER(_P)]),
    "pp_symbolic_sizes": (None, [_P, _I64P]),
    "pp_symbolic_get": (None, [_P] + [_I64P] * 8),
    "pp_symbolic_free": (None, [_P]),
}

_lib = None


def lib():
    """The loaded library (loaded once; raises OSError if the build is missing)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIBPATH):
            raise OSError("libpathpack_b200.so not found at %s: run `python pathpack.jl_b200/build.py`" % LIBPATH)
        L = C.CDLL(LIBPATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(code, handle=None):
    """Raise PPError for a non-zero status, with the library's message."""
    if code != PP_OK:
        msg = lib().pp_last_error(handle)
        raise PPError(code, msg.decode() if msg else "error")
    return code


def i64ptr(a):
    """A ctypes int64 pointer to a contiguous numpy int64 array (or NULL for None)."""
    if a is None:
        return None
    return a.ctypes.data_as(_I64P)


def vptr(a):
    """A void pointer to a numpy array, a torch tensor (data_ptr) or an integer address."""
    if a is None:
        return None
    if isinstance(a, int):
        return C.c_void_p(a)
    if hasattr(a, "data_ptr"):
        return C.c_void_p(a.data_ptr())
    return a.ctypes.data_as(C.c_void_p)
