"""lmul! on host memory in column panels (pp_lmul / pp_lmul_t with where = PP_HOST and B of 32 MB or more): the
uploads, the per-panel solves and the downloads overlap on three streams.  The results must be those of the
device-memory solve of the whole B and of the oracle's lmul!, bit for bit for the idempotent semirings, for
pageable and page-locked host arrays, a leading dimension larger than n, and panel counts from 2 to 4.
"""
import ctypes as C

import numpy as np
import pytest

import pathpack_b200 as pp
from oracle.oracle import OracleLU
from pathpack_b200 import graphs
from pathpack_b200._lib import PP_HOST, check, lib
from tests.helpers import same, weights

pytestmark = pytest.mark.gpu

SR = {"MinPlus": pp.MinPlus(), "MaxMin": pp.MaxMin(), "PlusProd": pp.PlusProd()}


def factor_pair(name, dtype, side):
    n, I, J, _ = graphs.grid2d(side, side, seed=5)
    W = weights(name, dtype, len(I), 23)
    cp, rv, nz = graphs.csc(n, I, J, W)
    S = pp.ssymbolic(n, cp, rv)
    F = pp.B200SLU(SR[name], dtype, S, device=0).assemble_csc(cp, rv, nz).factor()
    O = OracleLU(name, dtype, S).assemble(cp, rv, nz).factor()
    return n, F, O


def bits(a):
    return np.ascontiguousarray(a).view(np.uint8)


def rhs(name, dtype, n, k, ld, seed):
    rng = np.random.default_rng(seed)
    s = SR[name]
    B = np.full((ld, k), s.zero(dtype), dtype=dtype, order="F")
    B[rng.integers(0, n, size=k), np.arange(k)] = s.one(dtype)
    B[:n][rng.random((n, k)) < 0.002] = s.one(dtype)
    return B


@pytest.mark.parametrize("name,dtype,side,k", [("MinPlus", np.float64, 128, 256), ("MinPlus", np.float64, 128, 384),
                                               ("MaxMin", np.float32, 128, 512), ("PlusProd", np.float64, 96, 512)])
def test_host_lmul_panels(gpu, name, dtype, side, k):
    import torch

    n, F, O = factor_pair(name, dtype, side)
    try:
        assert n * k * np.dtype(dtype).itemsize >= 32 << 20  # the panel path
        B = rhs(name, dtype, n, k, n, seed=k)
        want = O.lmul(B)
        # pageable numpy array
        got = pp.lmul_(F, B.copy(order="F"))
        same(got, want, name, dtype, "pageable host lmul!")
        # the device-memory solve of the whole B
        Bd = torch.from_numpy(B.T.copy()).cuda().T  # column-major CUDA tensor
        pp.lmul_(F, Bd)
        dev = Bd.cpu().numpy()
        if name != "PlusProd":
            assert np.array_equal(bits(got), bits(dev)), "host panels vs device"
        # page-locked host memory with a leading dimension above n
        ld = n + 8
        Bp = rhs(name, dtype, n, k, ld, seed=k)
        pin = torch.from_numpy(Bp.T.copy()).pin_memory()  # rows of pin = columns of Bp
        check(lib().pp_lmul(F._h, C.c_void_p(pin.data_ptr()), ld, k, PP_HOST), F._h)
        got_p = pin.numpy().T
        same(got_p[:n], want, name, dtype, "page-locked host lmul! (ldb = n + 8)")
        assert np.array_equal(bits(got_p[n:]), bits(Bp[n:])), "rows past n were written"
        # lmul!(transpose(F), B) takes the same panel path
        got_t = pp.lmul_(pp.transpose(F), B.copy(order="F"))
        same(got_t, np.asfortranarray(O.rmul(np.asfortranarray(B.T)).T), name, dtype, "host lmul!(F', B)")
        st = F.stats()
        assert st["pairs_solve"] > 0
    finally:
        F.close()
