"""The reference's user API on the B200 library: mlu, mstar, lu_, lmul_, rmul_, Matrix.

PATHPACK.jl (src/CPU/abstract_slu.jl) exposes
    F = mlu(s, A; alg, nt)   factor the star A* = U* L*          (:44-58)
    mstar(s, A)              Matrix(mlu(s, A))                   (:81-87)
    lu!(F)                   refactor in place                   (:119-121)
    lmul!(F, B)              B <- A* B (columns of the star)     (:131-134)
    rmul!(B, F)              B <- B A* (rows of the star)        (:142-145)
    Matrix(F)                the whole star                      (:10-14)
Python has no `!`: the in-place functions are lmul_, rmul_, lu_.  A factor is a B200SLU (the analogue of
ChordalSLU, src/CPU/chordal_slu.jl:1-26) holding a library handle on one GPU.  Arrays are column-major as
Julia's: numpy arrays are used in Fortran order (copied when they are not); CUDA torch tensors with column
stride 1 are used in place on the device.
"""
import ctypes as C

import numpy as np

from . import semiring as sr
from ._lib import PP_DEVICE, PP_HOST, check, i64ptr, lib, pp_options, pp_stats, vptr
from .symbolic import Structure, ssymbolic


def _csc(A, dtype=None):
    """(n, colptr, rowval, nzval) of a square scipy.sparse matrix or dense array (entries != 0 are arcs for
    dense input only through scipy), duplicates already combined by the caller."""
    import scipy.sparse as sp

    if not sp.issparse(A):
        A = sp.csc_matrix(np.asarray(A))
    A = sp.csc_matrix(A)
    A.sort_indices()
    n, m = A.shape
    if n != m:
        raise ValueError("the matrix must be square, got %s" % (A.shape,))
    data = A.data if dtype is None else A.data.astype(dtype)
    return n, A.indptr.astype(np.int64), A.indices.astype(np.int64), np.ascontiguousarray(data)


def _options(kw):
    o = pp_options()
    lib().pp_default_options(C.byref(o))
    for k, v in kw.items():
        if k not in dict(pp_options._fields_) or k == "reserved":
            raise TypeError("unknown option %r" % k)
        setattr(o, k, int(v))
    return o


class B200SLU:
    """A factorization of the star of A over a semiring, held on one GPU (mlu's result)."""

    def __init__(self, s, dtype, structure, device=0, **options):
        dtype = np.dtype(dtype)
        if not sr.supported(s, dtype):
            raise TypeError("%r over %s is not supported (pp_check_semiring)" % (s, dtype))
        self.s, self.dtype, self.S, self.device = s, dtype, structure, device
        self._dt = sr.DTYPES[dtype]
        L = lib()
        h = C.c_void_p()
        check(L.pp_create_with(device, C.byref(_options(options)) if options else None, C.byref(h)))
        self._h = h
        S = structure
        check(L.pp_set_structure(h, S.n, S.nf, S.nB, i64ptr(S.Rptr), i64ptr(S.Sptr), i64ptr(S.Stgt), i64ptr(S.Bptr),
                                 i64ptr(S.Fptr), i64ptr(S.Nptr), i64ptr(S.Ntgt), i64ptr(S.perm), 0), h)

    # --- options
    def options(self):
        """The handle's pp_options as a dict (wait_timeout_us, fail_alloc_after, profile)."""
        o = pp_options()
        check(lib().pp_get_options(self._h, C.byref(o)), self._h)
        return {k: getattr(o, k) for k, _ in pp_options._fields_ if k != "reserved"}

    def set_options(self, **options):
        """Change options (keywords as in pp_options); the others keep their values."""
        cur = self.options()
        cur.update(options)
        check(lib().pp_set_options(self._h, C.byref(_options(cur))), self._h)
        return self

    # --- several GPUs
    def join(self, comm_id, nranks, rank):
        """Join this factor's handle to a group of `nranks` GPUs as `rank` (pp_comm_init): factor() then splits
        the bottom of the tree across the group and exchanges the parts over NCCL; every rank must set the same
        structure, assemble the same matrix and call factor() the same number of times.  comm_id: the bytes of
        comm_id() made on one rank; nranks = 1 leaves the group."""
        buf = C.create_string_buffer(bytes(comm_id), 128) if comm_id is not None else None
        check(lib().pp_comm_init(self._h, buf, int(nranks), int(rank)), self._h)
        return self

    # --- lifecycle
    def close(self):
        if getattr(self, "_h", None):
            lib().pp_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def shape(self):
        return (self.S.n, self.S.n)

    # --- numeric phase
    def assemble(self, A):
        """copyto!(F, A): scatter A's entries into the factor arrays on the device."""
        n, cp, rv, nz = _csc(A, self.dtype)
        if n != self.S.n:
            raise ValueError("matrix size %d does not match the structure (%d)" % (n, self.S.n))
        check(lib().pp_assemble(self._h, self.s.id, self._dt, i64ptr(cp), i64ptr(rv), vptr(nz), 0), self._h)
        return self

    def assemble_csc(self, colptr, rowval, nzval):
        """copyto!(F, A) from 0-based CSC arrays of A (no duplicates)."""
        cp = np.ascontiguousarray(colptr, dtype=np.int64)
        rv = np.ascontiguousarray(rowval, dtype=np.int64)
        nz = np.ascontiguousarray(nzval, dtype=self.dtype)
        check(lib().pp_assemble(self._h, self.s.id, self._dt, i64ptr(cp), i64ptr(rv), vptr(nz), 0), self._h)
        return self

    def update_values(self, nzval):
        """New weights (host numpy array or CUDA tensor, in the order of the last assemble) for the same
        pattern, re-assembled on the device; then factor() refactorizes."""
        where = PP_DEVICE if hasattr(nzval, "data_ptr") else PP_HOST
        if where == PP_HOST:
            nzval = np.ascontiguousarray(nzval, dtype=self.dtype)
        check(lib().pp_update_values(self._h, vptr(nzval), where), self._h)
        return self

    def set_values(self, LD, LL, UD, UL, Nval):
        c = lambda a: np.ascontiguousarray(a, dtype=self.dtype)
        LD, LL, UD, UL, Nval = (c(a) for a in (LD, LL, UD, UL, Nval))
        check(lib().pp_set_values(self._h, self.s.id, self._dt, vptr(LD), vptr(LL), vptr(UD), vptr(UL), vptr(Nval)),
              self._h)
        return self

    def factor(self, sync=True):
        """lu!(F): the multifrontal factorization of the star on the GPU.  The C call only enqueues the work on
        the handle's stream; with sync=False this returns at once too, and a device error is reported by the next
        call that waits (sync(), a solve into host memory, factors(), stats())."""
        check(lib().pp_factor(self._h), self._h)
        if sync:
            self.sync()
        return self

    def factors(self):
        """(LD, LL, UD, UL) downloaded to the host (the ChordalSLU fields LDval, LLval, UDval, ULval)."""
        nD, nL, _ = self.S.sizes()
        LD, UD = np.empty(nD, self.dtype), np.empty(nD, self.dtype)
        LL, UL = np.empty(nL, self.dtype), np.empty(nL, self.dtype)
        check(lib().pp_get_factor(self._h, vptr(LD), vptr(LL), vptr(UD), vptr(UL)), self._h)
        return LD, LL, UD, UL

    def stats(self):
        st = pp_stats()
        check(lib().pp_get_stats(self._h, C.byref(st)), self._h)
        return {k: getattr(st, k) for k, _ in pp_stats._fields_}

    def set_profile(self, on=True):
        """Time every launch of this handle per kernel class (CUDA events on its stream); resets the totals."""
        check(lib().pp_set_profile(self._h, 1 if on else 0), self._h)

    def profile(self):
        """{class: {launches, ms, bytes, pairs}} accumulated since set_profile."""
        from ._lib import pp_kernel_class

        arr = (pp_kernel_class * 16)()
        cnt = C.c_int32()
        check(lib().pp_get_profile(self._h, arr, 16, C.byref(cnt)), self._h)
        return {arr[i].name.decode(): {"launches": arr[i].launches, "ms": arr[i].ms, "bytes": arr[i].bytes,
                                       "pairs": arr[i].pairs} for i in range(cnt.value)}

    def trace(self):
        """The timeline of the last factorization's top of the tree (option trace=1; pp_get_trace): an
        (ntasks, 6) uint64 array of [taken, assembled, products done, published] (global timer, ns),
        (sm << 32) | front, (I << 32) | J per tile task, in list order."""
        cnt = C.c_int64()
        check(lib().pp_get_trace(self._h, None, 0, C.byref(cnt)), self._h)
        out = np.zeros((cnt.value, 6), dtype=np.uint64)
        if cnt.value:
            check(lib().pp_get_trace(self._h, vptr(out), cnt.value, C.byref(cnt)), self._h)
        return out

    def stream(self):
        """The handle's CUDA stream (cudaStream_t as an integer)."""
        return lib().pp_stream(self._h)

    def sync(self):
        check(lib().pp_sync(self._h), self._h)

    # --- plans
    def plan_lmul(self, nzval, Bin, Bout=None):
        """A Plan replaying one step as a CUDA graph (pp_plan_lmul): new weights from the CUDA tensor nzval
        re-assembled, the factorization, and Bout <- A* Bin (column-major n x k CUDA tensors; Bout = Bin by
        default).  Plan.launch() enqueues a step on the handle's stream."""
        Bout = Bin if Bout is None else Bout
        for t in (nzval, Bin, Bout):
            if not hasattr(t, "data_ptr") or not t.is_cuda or t.dtype.itemsize != self.dtype.itemsize:
                raise TypeError("nzval, Bin and Bout must be CUDA tensors of the factor's element type")
        if Bin.dim() != 2 or Bin.stride(0) != 1 or Bout.shape != Bin.shape or Bout.stride() != Bin.stride():
            raise ValueError("Bin and Bout must be column-major n x k tensors of the same layout")
        return Plan(self, nzval, Bin, Bout)

    # --- solves
    def lmul_static(self, B):
        """B <- A* B for a column-major CUDA tensor B, through pp_lmul_static: the solve allocates nothing and
        uses the library's static per-device scratch (PP_STATIC_SCRATCH_BYTES), so n x k must fit in it."""
        n = self.S.n
        if not hasattr(B, "data_ptr") or not B.is_cuda or B.dtype.itemsize != self.dtype.itemsize:
            raise TypeError("B must be a CUDA tensor of the factor's element type")
        if B.dim() == 1:
            k, ld = 1, n
        else:
            if B.stride(0) != 1:
                raise ValueError("B must be column-major (stride(0) == 1)")
            k, ld = B.shape[1], B.stride(1)
        check(lib().pp_lmul_static(self._h, vptr(B), ld, k), self._h)
        return B

    def _solve(self, B, left, sync=True, trans=False):
        n = self.S.n
        L = lib()
        fn = (L.pp_lmul_t if left else L.pp_rmul_t) if trans else (L.pp_lmul if left else L.pp_rmul)
        if hasattr(B, "data_ptr"):  # a CUDA torch tensor, used in place
            if B.dtype.itemsize != self.dtype.itemsize or not B.is_cuda:
                raise TypeError("B must be a CUDA tensor of the factor's element type")
            if B.dim() == 1:
                k, ld = 1, (n if left else 1)
            else:
                if B.stride(0) != 1:
                    raise ValueError("B must be column-major (stride(0) == 1)")
                k, ld = (B.shape[1], B.stride(1)) if left else (B.shape[0], B.stride(1))
            check(fn(self._h, vptr(B), ld, k, PP_DEVICE), self._h)
            if sync:  # device results are ordered on the handle's stream; make them visible to every stream
                self.sync()
            return B
        X = np.asarray(B)
        vec = X.ndim == 1
        X2 = X.reshape(-1, 1) if (vec and left) else (X.reshape(1, -1) if vec else X)
        if (X2.shape[0] if left else X2.shape[1]) != n:
            raise ValueError("B has %s rows/columns, the factor has %d vertices" % (X2.shape, n))
        W = np.asfortranarray(X2, dtype=self.dtype)
        k = W.shape[1] if left else W.shape[0]
        ld = W.shape[0]
        check(fn(self._h, vptr(W), ld, k, PP_HOST), self._h)
        if isinstance(B, np.ndarray) and B.dtype == self.dtype and (W is B or np.shares_memory(W, B)):
            return B
        if isinstance(B, np.ndarray) and B.flags.writeable:
            B[...] = W.reshape(B.shape)
            return B
        return W.reshape(X.shape)

    def star(self, col0=0, ncols=None, out=None):
        """Columns col0 .. col0+ncols-1 of A* (original labels) as an n x ncols column-major array."""
        n = self.S.n
        ncols = n - col0 if ncols is None else ncols
        if out is None:
            out = np.empty((n, ncols), dtype=self.dtype, order="F")
        if hasattr(out, "data_ptr"):
            check(lib().pp_star(self._h, vptr(out), out.stride(1), col0, ncols, PP_DEVICE), self._h)
            self.sync()
        else:
            if not out.flags.f_contiguous:
                raise ValueError("out must be column-major")
            check(lib().pp_star(self._h, vptr(out), n, col0, ncols, PP_HOST), self._h)
        return out


def star_cols(F, cols, out=None):
    """Columns `cols` of A* (original labels, any order) as an n x len(cols) column-major array (pp_star_cols);
    `out` may be a column-major CUDA tensor."""
    cols = np.ascontiguousarray(cols, dtype=np.int64)
    n, k = F.S.n, len(cols)
    if out is None:
        out = np.empty((n, k), dtype=F.dtype, order="F")
    if hasattr(out, "data_ptr"):
        check(lib().pp_star_cols(F._h, vptr(out), out.stride(1), i64ptr(cols), k, PP_DEVICE), F._h)
        F.sync()
    else:
        check(lib().pp_star_cols(F._h, vptr(out), out.shape[0], i64ptr(cols), k, PP_HOST), F._h)
    return out


def star_rows(F, sources, out=None):
    """Rows `sources` of A* (the closure from a set of sources; apsp_gpu(A, sources) of the reference) as a
    len(sources) x n column-major array (pp_star_rows); `out` may be a column-major CUDA tensor."""
    sources = np.ascontiguousarray(sources, dtype=np.int64)
    n, k = F.S.n, len(sources)
    if out is None:
        out = np.empty((k, n), dtype=F.dtype, order="F")
    if hasattr(out, "data_ptr"):
        check(lib().pp_star_rows(F._h, vptr(out), out.stride(1), i64ptr(sources), k, PP_DEVICE), F._h)
        F.sync()
    else:
        check(lib().pp_star_rows(F._h, vptr(out), out.shape[0], i64ptr(sources), k, PP_HOST), F._h)
    return out


class Plan:
    """A captured refactor + lmul! step of a B200SLU (see B200SLU.plan_lmul)."""

    def __init__(self, F, nzval, Bin, Bout):
        self.F, self._keep = F, (nzval, Bin, Bout)
        p = C.c_void_p()
        check(lib().pp_plan_lmul(F._h, vptr(nzval), vptr(Bin), vptr(Bout), Bin.stride(1), Bin.shape[1],
                                 C.byref(p)), F._h)
        self._p = p

    def launch(self):
        check(lib().pp_plan_launch(self._p), self.F._h)

    @property
    def launches(self):
        n = C.c_int64()
        check(lib().pp_plan_launches(self._p, C.byref(n)))
        return n.value

    def close(self):
        if getattr(self, "_p", None):
            lib().pp_plan_destroy(self._p)
            self._p = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class TransposedSLU:
    """transpose(F): the factorization of (A*)^T = (A^T)* on the same device data (the reference's
    TransposeFactorization, which lmul! / rmul! unwrap to trans = Val(:T), src/CPU/abstract_slu.jl:131-145)."""

    def __init__(self, F):
        self.parent = F

    @property
    def shape(self):
        return self.parent.shape

    def _solve(self, B, left, sync=True):
        return self.parent._solve(B, left, sync, trans=True)


def transpose(F):
    """transpose(F) for lmul_(transpose(F), B) = (A*)^T B and rmul_(B, transpose(F)) = B (A*)^T."""
    return F.parent if isinstance(F, TransposedSLU) else TransposedSLU(F)


class MultiSLU:
    """One matrix factored on several GPUs by one process (pp_multi): a handle per device joined into one group;
    factor() splits the factorization, lmul_/rmul_/star split the right-hand sides or columns by device."""

    def __init__(self, s, dtype, structure, devices, **options):
        dtype = np.dtype(dtype)
        if not sr.supported(s, dtype):
            raise TypeError("%r over %s is not supported (pp_check_semiring)" % (s, dtype))
        self.s, self.dtype, self.S, self.devices = s, dtype, structure, list(devices)
        self._dt = sr.DTYPES[dtype]
        devs = (C.c_int32 * len(self.devices))(*self.devices)
        m = C.c_void_p()
        check(lib().pp_multi_create(devs, len(self.devices), C.byref(_options(options)) if options else None,
                                    C.byref(m)))
        self._m = m
        S = structure
        check(lib().pp_multi_set_structure(m, S.n, S.nf, S.nB, i64ptr(S.Rptr), i64ptr(S.Sptr), i64ptr(S.Stgt),
                                           i64ptr(S.Bptr), i64ptr(S.Fptr), i64ptr(S.Nptr), i64ptr(S.Ntgt),
                                           i64ptr(S.perm), 0))

    def close(self):
        if getattr(self, "_m", None):
            lib().pp_multi_destroy(self._m)
            self._m = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def assemble_csc(self, colptr, rowval, nzval):
        cp = np.ascontiguousarray(colptr, dtype=np.int64)
        rv = np.ascontiguousarray(rowval, dtype=np.int64)
        nz = np.ascontiguousarray(nzval, dtype=self.dtype)
        check(lib().pp_multi_assemble(self._m, self.s.id, self._dt, i64ptr(cp), i64ptr(rv), vptr(nz), 0))
        return self

    def factor(self):
        check(lib().pp_multi_factor(self._m))
        return self

    def lmul_(self, B, trans=False):
        """B <- A* B (host n x k, column-major), the k columns split by device."""
        if not (isinstance(B, np.ndarray) and B.flags.f_contiguous and B.dtype == self.dtype):
            raise TypeError("B must be a column-major numpy array of the factor's element type")
        check(lib().pp_multi_lmul(self._m, vptr(B), B.shape[0], B.shape[1], 1 if trans else 0))
        return B

    def rmul_(self, B, trans=False):
        """B <- B A* (host k x n, column-major), the k rows split by device."""
        if not (isinstance(B, np.ndarray) and B.flags.f_contiguous and B.dtype == self.dtype):
            raise TypeError("B must be a column-major numpy array of the factor's element type")
        check(lib().pp_multi_rmul(self._m, vptr(B), B.shape[0], B.shape[0], 1 if trans else 0))
        return B

    def star(self, col0=0, ncols=None):
        """Columns col0 .. col0+ncols-1 of A* (host n x ncols), split by device."""
        n = self.S.n
        ncols = n - col0 if ncols is None else ncols
        out = np.empty((n, ncols), dtype=self.dtype, order="F")
        check(lib().pp_multi_star(self._m, vptr(out), n, col0, ncols))
        return out


def comm_id():
    """A new group id for B200SLU.join (pp_comm_id, 128 bytes): make it on one rank, send it to the others."""
    buf = C.create_string_buffer(128)
    check(lib().pp_comm_id(buf))
    return buf.raw


def mlu(s, A, *, dtype=None, structure=None, device=0, method="nd"):
    """F = mlu(s, A): symbolic analysis (host), assembly and factorization of the star on the GPU."""
    n, cp, rv, nz = _csc(A, dtype)
    dt = np.dtype(dtype) if dtype is not None else nz.dtype
    S = structure if structure is not None else ssymbolic(n, cp, rv, method)
    F = B200SLU(s, dt, S, device)
    check(lib().pp_assemble(F._h, s.id, F._dt, i64ptr(cp), i64ptr(rv), vptr(np.ascontiguousarray(nz, dt)), 0), F._h)
    return F.factor()


def lu_(F):
    """lu!(F): refactor (after assemble / set_values with new weights on the same structure)."""
    return F.factor()


def lmul_(F, B):
    """lmul!(F, B): B <- A* B, the least solution of X = A X (+) B (F may be transpose(F))."""
    return F._solve(B, True)


def rmul_(B, F):
    """rmul!(B, F): B <- B A*, the least solution of X = X A (+) B (F may be transpose(F))."""
    return F._solve(B, False)


def Matrix(F):
    """Matrix(F): the whole star A*, n x n column-major."""
    return F.star()


def mstar(s, A, **kw):
    """mstar(s, A) = Matrix(mlu(s, A))."""
    F = mlu(s, A, **kw)
    try:
        return F.star()
    finally:
        F.close()
