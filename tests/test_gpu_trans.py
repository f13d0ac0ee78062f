"""lmul!(transpose(F), B) and rmul!(B, transpose(F)) through the C ABI (pp_lmul_t / pp_rmul_t), on the GPU.

(A*)^T B is (B^T A*)^T for the commutative (x) of every semiring here, so the oracle's rmul! of B^T gives the
expected result with the same per-element operations: bit for bit for the idempotent semirings, rtol 1e-5 /
1e-12 for PlusProd.  As an independent check the oracle also factors A^T itself (another structure), whose
lmul! is (A^T)* B = (A*)^T B, compared within the north-star tolerance.
"""
import numpy as np
import pytest

import pathpack_b200 as pp
from oracle.oracle import OracleLU
from tests.helpers import CASES, close, graph, same

pytestmark = pytest.mark.gpu

SR = {s.__class__.__name__: s for s in [pp.MinPlus(), pp.MaxPlus(), pp.MaxMin(), pp.MinMax(), pp.MaxProd(),
                                         pp.PlusProd(), pp.OrAnd()]}


def transposed_csc(n, cp, rv, nz):
    col = np.repeat(np.arange(n), np.diff(cp))
    order = np.lexsort((col, rv))  # columns of A^T are the rows of A
    I, J, W = col[order], rv[order], nz[order]
    colptr = np.zeros(n + 1, np.int64)
    np.add.at(colptr, J + 1, 1)
    return np.cumsum(colptr), I.astype(np.int64), np.ascontiguousarray(W)


@pytest.mark.parametrize("name,dtype", CASES)
@pytest.mark.parametrize("kind,k", [("sprand", 9), ("knn", 40), ("grid3d", 300)])
def test_transposed_solves(gpu, name, dtype, kind, k):
    n, cp, rv, nz = graph(kind, name, dtype, seed=4)
    S = pp.ssymbolic(n, cp, rv)
    F = pp.B200SLU(SR[name], dtype, S, device=0).assemble_csc(cp, rv, nz).factor()
    try:
        O = OracleLU(name, dtype, S).assemble(cp, rv, nz).factor()
        rng = np.random.default_rng(k)
        z, one = SR[name].zero(dtype), SR[name].one(dtype)
        B = np.full((n, k), z, dtype=dtype, order="F")
        B[rng.integers(0, n, size=k), np.arange(k)] = one
        B[rng.random(B.shape) < 0.05] = one
        Ft = pp.transpose(F)
        got_l = pp.lmul_(Ft, B.copy(order="F"))
        same(got_l, np.asfortranarray(O.rmul(np.asfortranarray(B.T)).T), name, dtype, "%s lmul!(F', B)" % kind)
        R = np.asfortranarray(B.T)
        got_r = pp.rmul_(R.copy(order="F"), Ft)
        same(got_r, np.asfortranarray(O.lmul(B).T), name, dtype, "%s rmul!(B, F')" % kind)
        # the factorization of A^T itself
        tcp, trv, tnz = transposed_csc(n, cp, rv, nz)
        St = pp.ssymbolic(n, tcp, trv)
        Ot = OracleLU(name, dtype, St).assemble(tcp, trv, tnz).factor()
        close(got_l, Ot.lmul(B), name, dtype, "%s lmul!(F', B) vs the factor of A^T" % kind)
        close(got_r, Ot.rmul(R), name, dtype, "%s rmul!(B, F') vs the factor of A^T" % kind)
        assert pp.transpose(Ft) is F
    finally:
        F.close()


def test_transposed_device_tensors(gpu):
    """Device-resident B in place, through both transposed entry points."""
    import torch

    n, cp, rv, nz = graph("grid40", "MinPlus", np.float64, seed=2)
    S = pp.ssymbolic(n, cp, rv)
    F = pp.B200SLU(pp.MinPlus(), np.float64, S, device=0).assemble_csc(cp, rv, nz).factor()
    try:
        O = OracleLU("MinPlus", np.float64, S).assemble(cp, rv, nz).factor()
        B = np.full((n, 33), np.inf, order="F")
        B[np.arange(33) * 41 % n, np.arange(33)] = 0.0
        Bd = torch.from_numpy(np.ascontiguousarray(B.T)).to("cuda:0").T  # column-major n x 33
        pp.lmul_(pp.transpose(F), Bd)
        same(Bd.cpu().numpy(), np.asfortranarray(O.rmul(np.asfortranarray(B.T)).T), "MinPlus", np.float64,
             "device lmul!(F', B)")
        R = np.asfortranarray(B.T)
        Rd = torch.from_numpy(np.ascontiguousarray(R.T)).to("cuda:0").T  # column-major 33 x n
        pp.rmul_(Rd, pp.transpose(F))
        same(Rd.cpu().numpy(), np.asfortranarray(O.lmul(B).T), "MinPlus", np.float64, "device rmul!(B, F')")
    finally:
        F.close()
