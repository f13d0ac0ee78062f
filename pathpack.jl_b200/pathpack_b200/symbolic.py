"""The symbolic structure a factorization needs: the fields of PATHPACK.jl's ChordalSSymbolic
(src/CPU/chordal_ssymbolic.jl:1-8) plus the permutation, as numpy arrays.

In PATHPACK.jl this comes from `ssymbolic(A; alg)` (Julia + CliqueTrees.jl).  `ssymbolic` here calls the
library's host stand-in (pp_symbolic: the reference's SCC walk, nested dissection, maximal supernodes);
`Structure.from_arrays` takes a structure computed elsewhere, e.g. by Julia, 0- or 1-based.
"""
import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._lib import check, i64ptr, lib


@dataclass
class Structure:
    """0-based: fronts' residuals Rptr, separators Sptr/Stgt, components Bptr/Fptr, coupling Nptr/Ntgt, perm."""
    n: int
    nf: int
    nB: int
    Rptr: np.ndarray
    Sptr: np.ndarray
    Stgt: np.ndarray
    Bptr: np.ndarray
    Fptr: np.ndarray
    Nptr: np.ndarray
    Ntgt: np.ndarray
    perm: np.ndarray

    @staticmethod
    def from_arrays(n, Rptr, Sptr, Stgt, Bptr, Fptr, Nptr, Ntgt, perm, base=0):
        a = lambda x: np.ascontiguousarray(np.asarray(x, dtype=np.int64) - base)
        R, B = a(Rptr), a(Bptr)
        return Structure(int(n), len(R) - 1, len(B) - 1, R, a(Sptr), a(Stgt), B, a(Fptr), a(Nptr), a(Ntgt), a(perm))

    @property
    def invp(self):
        p = np.empty(self.n, dtype=np.int64)
        p[self.perm] = np.arange(self.n, dtype=np.int64)
        return p

    @property
    def nn(self):
        return np.diff(self.Rptr)

    @property
    def na(self):
        return np.diff(self.Sptr)

    def sizes(self):
        """(|LD|, |LL|, |Nval|): the running sums of nn^2 and nn*na, and the coupling entries."""
        nn, na = self.nn, self.na
        return int((nn * nn).sum()), int((nn * na).sum()), int(self.Nptr[-1])

    def parent(self):
        """Parent front of each front (-1 for roots): the front of its first separator vertex."""
        idx = np.repeat(np.arange(self.nf), self.nn)
        p = np.full(self.nf, -1, dtype=np.int64)
        has = self.na > 0
        p[has] = idx[self.Stgt[self.Sptr[:-1][has]]]
        return p

    def pairs_factor(self):
        """(x)(+) pairs of the partial LU of every front: sum over pivots of the trailing block size squared."""
        nn, na = self.nn.astype(np.float64), self.na.astype(np.float64)
        nj = nn + na
        s = lambda m: (m - 1) * m * (2 * m - 1) / 6
        return float((s(nj) - s(na)).sum())

    def pairs_solve(self):
        """(x)(+) pairs of one right-hand side through L* and U* over every front, plus the coupling."""
        nn, na = self.nn.astype(np.float64), self.na.astype(np.float64)
        return float((nn * (nn - 1) + 2 * nn * na).sum() + self.Nptr[-1])

    def rootpath_pairs(self, sources):
        """(x)(+) pairs of the triangular solve restricted to the root paths of unit sources (positions):
        sum over sources of sum over the fronts on the path from the source's front to its root of
        nn(nn-1)/2 + nn*na."""
        nn, na = self.nn.astype(np.float64), self.na.astype(np.float64)
        cost = nn * (nn - 1) / 2 + nn * na
        par = self.parent()
        # cumulative cost from each front to its root (fronts are in postorder: parents come later)
        up = cost.copy()
        for f in range(self.nf - 1, -1, -1):
            if par[f] >= 0:
                up[f] += up[par[f]]
        idx = np.repeat(np.arange(self.nf), self.nn)
        return float(up[idx[np.asarray(sources)]].sum())


def ssymbolic(n, colptr, rowval, method="nd", leaf=64):
    """Symbolic analysis of the n x n pattern (0-based CSC, A[i, j] = arc i -> j) with the host stand-in."""
    colptr = np.ascontiguousarray(colptr, dtype=np.int64)
    rowval = np.ascontiguousarray(rowval, dtype=np.int64)
    L = lib()
    out = C.c_void_p()
    check(L.pp_symbolic(n, i64ptr(colptr), i64ptr(rowval), {"nd": 0, "natural": 1}[method], leaf, C.byref(out)))
    try:
        sz = np.zeros(5, dtype=np.int64)
        L.pp_symbolic_sizes(out, i64ptr(sz))
        n_, nf, nB, nS, nN = (int(x) for x in sz)
        R = np.zeros(nf + 1, np.int64)
        S = np.zeros(nf + 1, np.int64)
        St = np.zeros(max(nS, 1), np.int64)
        B = np.zeros(nB + 1, np.int64)
        F = np.zeros(nB + 1, np.int64)
        Np_ = np.zeros(n_ + 1, np.int64)
        Nt = np.zeros(max(nN, 1), np.int64)
        P = np.zeros(max(n_, 1), np.int64)
        L.pp_symbolic_get(out, i64ptr(R), i64ptr(S), i64ptr(St), i64ptr(B), i64ptr(F), i64ptr(Np_), i64ptr(Nt),
                          i64ptr(P))
    finally:
        L.pp_symbolic_free(out)
    return Structure(n_, nf, nB, R, S, St[:nS], B, F, Np_, Nt[:nN], P[:n_])
