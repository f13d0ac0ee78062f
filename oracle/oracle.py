"""ctypes wrapper of the oracle (oracle/_build/libpp_oracle.so).

TEST INFRASTRUCTURE ONLY: the CPU restatement of PATHPACK.jl's solver (see pp_oracle.h for the file:line
each routine follows).  Only tests/, __graft_entry__.smoke() and bench.py's CPU legs load it, as the checker
and the timed CPU baseline; the product never does.

A structure is any object with the attributes n, nf, nB, Rptr, Sptr, Stgt, Bptr, Fptr, Nptr, Ntgt, perm
(0-based int64 numpy arrays), such as pathpack_b200.Structure.  Matrices are column-major numpy arrays.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIBPATH = os.path.join(HERE, "_build", "libpp_oracle.so")

SR = {"MinPlus": 0, "MaxPlus": 1, "MaxMin": 2, "MinMax": 3, "MaxProd": 4, "PlusProd": 5, "OrAnd": 6}
DT = {np.dtype(np.float32): 0, np.dtype(np.float64): 1, np.dtype(np.int32): 2}
I32MAX = np.iinfo(np.int32).max

_lib = None
_P = C.c_void_p
_I64P = C.POINTER(C.c_int64)


def build():
    """Compile the oracle with its Makefile (gcc) if needed."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIBPATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIBPATH):
            build()
        L = C.CDLL(LIBPATH)
        L.ppo_struct_new.restype = _P
        L.ppo_struct_new.argtypes = [C.c_int64] * 3 + [_I64P] * 8
        L.ppo_struct_free.argtypes = [_P]
        L.ppo_struct_sizes.argtypes = [_P, _I64P]
        L.ppo_struct_derived.argtypes = [_P, _I64P, _I64P, _I64P, _I64P]
        for name in ("ppo_assemble",):
            getattr(L, name).argtypes = [C.c_int, C.c_int, _P, _I64P, _I64P, _P, _P, _P, _P, _P, _P]
        L.ppo_factor.argtypes = [C.c_int, C.c_int, _P, _P, _P, _P, _P, C.c_int]
        for name in ("ppo_lmul", "ppo_rmul"):
            getattr(L, name).argtypes = [C.c_int, C.c_int, _P, _P, _P, _P, _P, _P, _P, C.c_int64, C.c_int64, C.c_int]
        L.ppo_star.argtypes = [C.c_int, C.c_int, _P, _P, _P, _P, _P, _P, _P, C.c_int]
        L.ppo_gemm.argtypes = [C.c_int, C.c_int, C.c_int64, C.c_int64, C.c_int64, _P, C.c_int64, _P, C.c_int64, _P,
                               C.c_int64, C.c_int]
        L.ppo_getrf.argtypes = [C.c_int, C.c_int, C.c_int64, _P, C.c_int64]
        L.ppo_getrf_batched.argtypes = [C.c_int, C.c_int, C.c_int64, C.c_int64, _P, C.c_int]
        _lib = L
    return _lib


def _i64(a):
    return np.ascontiguousarray(a, dtype=np.int64)


def _p(a):
    return a.ctypes.data_as(C.c_void_p) if a is not None else None


def _check(code, what):
    if code == -1:
        raise TypeError("%s: unsupported semiring / element type" % what)
    if code != 0:
        raise MemoryError("%s: oracle failed with %d" % (what, code))


def srid(s):
    return SR[s if isinstance(s, str) else type(s).__name__]


class OStruct:
    """The oracle's copy of a structure (derived arrays computed in C)."""

    def __init__(self, S):
        self._keep = [_i64(getattr(S, k)) for k in ("Rptr", "Sptr", "Stgt", "Bptr", "Fptr", "Nptr", "Ntgt", "perm")]
        ptrs = [a.ctypes.data_as(_I64P) for a in self._keep]
        self.h = lib().ppo_struct_new(int(S.n), int(S.nf), int(S.nB), *ptrs)
        if not self.h:
            raise ValueError("malformed structure")
        sz = np.zeros(4, np.int64)
        lib().ppo_struct_sizes(self.h, sz.ctypes.data_as(_I64P))
        self.nD, self.nL, self.nN, self.maxfront = (int(x) for x in sz)
        self.n, self.nf = int(S.n), int(S.nf)

    def derived(self):
        pnt = np.zeros(max(self.nf, 1), np.int64)
        rel = np.zeros(max(int(self._keep[1][-1]), 1), np.int64)
        Dp = np.zeros(self.nf + 1, np.int64)
        Lp = np.zeros(self.nf + 1, np.int64)
        lib().ppo_struct_derived(self.h, *(a.ctypes.data_as(_I64P) for a in (pnt, rel, Dp, Lp)))
        return pnt[:self.nf], rel[:int(self._keep[1][-1])], Dp, Lp

    def __del__(self):
        if getattr(self, "h", None):
            lib().ppo_struct_free(self.h)
            self.h = None


class OracleLU:
    """mlu on the CPU restatement: assembly (copyto!) and multifrontal factorization (sgetrf!)."""

    def __init__(self, s, dtype, S):
        self.s, self.dtype, self.S = srid(s), np.dtype(dtype), S
        self.dt = DT[self.dtype]
        self.os = OStruct(S)
        z = self.dtype
        self.LD, self.UD = np.empty(self.os.nD, z), np.empty(self.os.nD, z)
        self.LL, self.UL = np.empty(self.os.nL, z), np.empty(self.os.nL, z)
        self.Nval = np.empty(self.os.nN, z)

    def assemble(self, colptr, rowval, nzval):
        nz = np.ascontiguousarray(nzval, dtype=self.dtype)
        cp, rv = _i64(colptr), _i64(rowval)
        _check(lib().ppo_assemble(self.s, self.dt, self.os.h, cp.ctypes.data_as(_I64P), rv.ctypes.data_as(_I64P),
                                  _p(nz), _p(self.LD), _p(self.LL), _p(self.UD), _p(self.UL), _p(self.Nval)),
               "assemble")
        return self

    def factor(self, nthreads=1):
        _check(lib().ppo_factor(self.s, self.dt, self.os.h, _p(self.LD), _p(self.LL), _p(self.UD), _p(self.UL),
                                nthreads), "factor")
        return self

    def _vals(self):
        return _p(self.LD), _p(self.LL), _p(self.UD), _p(self.UL), _p(self.Nval)

    def lmul(self, B, nthreads=1):
        """B <- A* B (n x k), returns a new Fortran-ordered array."""
        X = np.array(B, dtype=self.dtype, order="F", ndmin=2) if np.ndim(B) == 2 else \
            np.array(np.reshape(B, (-1, 1)), dtype=self.dtype, order="F")
        _check(lib().ppo_lmul(self.s, self.dt, self.os.h, *self._vals(), _p(X), X.shape[0], X.shape[1], nthreads),
               "lmul")
        return X if np.ndim(B) == 2 else X[:, 0]

    def rmul(self, B, nthreads=1):
        """B <- B A* (k x n), returns a new Fortran-ordered array."""
        X = np.array(B, dtype=self.dtype, order="F", ndmin=2)
        _check(lib().ppo_rmul(self.s, self.dt, self.os.h, *self._vals(), _p(X), X.shape[0], X.shape[0], nthreads),
               "rmul")
        return X

    def star(self, nthreads=1):
        n = self.os.n
        Cm = np.empty((n, n), dtype=self.dtype, order="F")
        _check(lib().ppo_star(self.s, self.dt, self.os.h, *self._vals(), _p(Cm), nthreads), "star")
        return Cm


def gemm(s, C_, A, B, nthreads=1):
    """C <- C (+) A (x) B (column-major numpy arrays; C modified in place)."""
    dt = DT[C_.dtype]
    m, n = C_.shape
    k = A.shape[1]
    assert C_.flags.f_contiguous and A.flags.f_contiguous and B.flags.f_contiguous
    _check(lib().ppo_gemm(srid(s), dt, m, n, k, _p(C_), m, _p(A), m, _p(B), k, nthreads), "gemm")
    return C_


def getrf_batched(s, A, nthreads=1):
    """In-place LU of the star of count n x n blocks: A has shape (count, n, n) with each block column-major
    (i.e. A[b] is the transpose of the block in numpy's C order); returns A."""
    count, n, _ = A.shape
    assert A.flags.c_contiguous
    _check(lib().ppo_getrf_batched(srid(s), DT[A.dtype], n, count, _p(A), nthreads), "getrf_batched")
    return A
