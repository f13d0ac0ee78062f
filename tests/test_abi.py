"""The C ABI without a GPU: the library loads, exports every function include/pathpack_b200.h declares with the
arity the Python binding uses, and its host-side checks answer with the documented status codes."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import pathpack_b200 as pp
from pathpack_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "pathpack_b200.h")


def declared():
    """name -> number of parameters of every function declared in the header."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    out = {}
    for m in re.finditer(r"\b([A-Za-z_][A-Za-z0-9_ \*]*?)\b(pp_[a-z_]+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S):
        params = m.group(3).strip()
        out[m.group(2)] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_header_parses():
    d = declared()
    for name in ("pp_create", "pp_set_structure", "pp_assemble", "pp_factor", "pp_lmul", "pp_rmul", "pp_star",
                 "pp_gemm", "pp_getrf_batched", "pp_symbolic"):
        assert name in d


def test_every_declared_symbol_is_exported_and_bound():
    L = pp.lib()
    for name, arity in declared().items():
        assert hasattr(L, name), "%s is declared but not exported" % name
        assert name in _lib.SIGNATURES, "%s has no Python signature" % name
        assert len(_lib.SIGNATURES[name][1]) == arity, "%s: header has %d parameters, binding %d" % (
            name, arity, len(_lib.SIGNATURES[name][1]))


def test_check_semiring():
    L = pp.lib()
    ok = {(0, 0), (0, 1), (0, 2), (1, 0), (1, 1), (2, 0), (2, 1), (3, 0), (3, 1), (4, 0), (4, 1), (5, 0), (5, 1), (6, 2)}
    for s in range(7):
        for d in range(3):
            r = L.pp_check_semiring(s, d)
            assert (r == 0) == ((s, d) in ok), (s, d, r)
            assert pp.supported(pp.semiring.BY_ID[s], [np.float32, np.float64, np.int32][d]) == ((s, d) in ok)
    assert L.pp_check_semiring(6, 0) == _lib.PP_EUNSUPPORTED
    assert b"not supported" in L.pp_last_error(None)
    assert L.pp_check_semiring(42, 0) == _lib.PP_EUNSUPPORTED


def test_null_handle_and_argument_errors():
    L = pp.lib()
    assert L.pp_destroy(None) == 0
    assert L.pp_factor(None) == _lib.PP_EINVAL
    assert L.pp_lmul(None, None, 1, 1, 0) == _lib.PP_EINVAL
    assert L.pp_create(0, None) == _lib.PP_EINVAL
    assert L.pp_gemm(0, 0, -1, 1, 1, None, 1, None, 1, None, 1, None) == _lib.PP_EINVAL
    assert L.pp_gemm(6, 0, 1, 1, 1, None, 1, None, 1, None, 1, None) == _lib.PP_EUNSUPPORTED
    assert L.pp_gemm(0, 0, 0, 5, 5, None, 1, None, 1, None, 1, None) == 0  # empty product is a no-op
    assert L.pp_getrf_batched(0, 2, 500, 1, None, None) == _lib.PP_EUNSUPPORTED  # block beyond shared memory
    assert L.pp_getrf_batched(0, 2, 0, 1, None, None) == 0


def test_create_without_gpu_fails_loudly():
    from tests.conftest import has_gpu

    if has_gpu():
        pytest.skip("a GPU is present")
    h = C.c_void_p()
    r = pp.lib().pp_create(0, C.byref(h))
    assert r in (_lib.PP_EDEVICE, _lib.PP_EINVAL)
    assert not h.value
    with pytest.raises(pp.PPError):
        pp.B200SLU(pp.MinPlus(), np.float64, pp.ssymbolic(3, np.array([0, 1, 2, 3]), np.array([1, 2, 0])))


def test_default_options():
    """pp_default_options: the default wait bound (0 = 2 s), the allocation hook off, profiling off."""
    L = pp.lib()
    o = _lib.pp_options()
    o.wait_timeout_us, o.fail_alloc_after, o.profile = 7, 7, 7
    L.pp_default_options(C.byref(o))
    assert (o.wait_timeout_us, o.fail_alloc_after, o.profile) == (0, -1, 0)
    assert L.pp_get_options(None, C.byref(o)) == _lib.PP_EINVAL
    assert L.pp_set_options(None, C.byref(o)) == _lib.PP_EINVAL
    with pytest.raises(TypeError):
        pp.api._options({"no_such_option": 1})


def test_multi_device_handle_argument_errors():
    """pp_multi_create refuses bad arguments before touching a device, and reports a device it cannot open."""
    L = pp.lib()
    m = C.c_void_p()
    assert L.pp_multi_create(None, 1, None, C.byref(m)) == _lib.PP_EINVAL and not m.value
    devs = (C.c_int32 * 1)(0)
    assert L.pp_multi_create(devs, 0, None, C.byref(m)) == _lib.PP_EINVAL
    assert L.pp_multi_factor(None) == _lib.PP_EINVAL
    assert L.pp_multi_destroy(None) == 0
    if not __import__("torch").cuda.is_available():
        r = L.pp_multi_create(devs, 1, None, C.byref(m))
        assert r != 0 and not m.value and L.pp_last_error(None)
