"""Amalgamation on the GPU: chains of top fronts merged into one front inside the library (the reference's GPU
path merges the same chains, ext/PATHPACKCUDAExt/chordal/amalgamate.jl).  The device plan then has fewer
fronts than the caller's structure, while the factor arrays the caller exchanges keep the caller's layout:
the factor, lmul!, rmul! and star columns equal the oracle's on the unmerged structure (bit for bit for the
idempotent semirings, whose merged fronts perform the members' operations on the same operands), and equal
the library's own results with merging switched off (pp_options.merge_width = 1).  PlusProd is never merged.
"""
import numpy as np
import pytest

import pathpack_b200 as pp
from oracle.oracle import OracleLU
from pathpack_b200 import graphs
from tests.helpers import CASES, close, same, weights

pytestmark = pytest.mark.gpu

SR = {s.__class__.__name__: s for s in [pp.MinPlus(), pp.MaxPlus(), pp.MaxMin(), pp.MinMax(), pp.MaxProd(),
                                         pp.PlusProd(), pp.OrAnd()]}


def sources(n, k, name, dtype, seed):
    rng = np.random.default_rng(seed)
    z, one = SR[name].zero(dtype), SR[name].one(dtype)
    B = np.full((n, k), z, dtype=dtype, order="F")
    B[rng.choice(n, size=k, replace=False), np.arange(k)] = one
    B[rng.random(B.shape) < 0.02] = one
    return B


def compare(got, want, name, dtype, what):
    (same if name != "PlusProd" else close)(got, want, name, dtype, what)


@pytest.mark.parametrize("name,dtype", CASES)
def test_merged_plan_matches_the_oracle(gpu, name, dtype):
    n, I, J, _ = graphs.grid2d(96, 96, seed=4)
    W = weights(name, dtype, len(I), 21)
    cp, rv, nz = graphs.csc(n, I, J, W)
    S = pp.ssymbolic(n, cp, rv)
    O = OracleLU(name, dtype, S).assemble(cp, rv, nz).factor(8)
    B = sources(n, 33, name, dtype, 1)
    R = np.asfortranarray(sources(n, 17, name, dtype, 2).T)
    res = {}
    for width in (0, 1):
        F = pp.B200SLU(SR[name], dtype, S, device=0, merge_width=width).assemble_csc(cp, rv, nz).factor()
        try:
            st = F.stats()
            assert st["nf"] == S.nf
            if width == 1 or name == "PlusProd":
                assert st["plan_fronts"] == S.nf
            else:
                assert st["plan_fronts"] < S.nf, "no chain of top fronts was merged"
            got = F.factors() + (pp.lmul_(F, B.copy(order="F")), pp.rmul_(R.copy(order="F"), F), F.star(7, 40))
        finally:
            F.close()
        want = (O.LD, O.LL, O.UD, O.UL, O.lmul(B), O.rmul(R))
        for g, w, what in zip(got, want, ("LD", "LL", "UD", "UL", "lmul!", "rmul!")):
            compare(g, w, name, dtype, "merge_width=%d %s" % (width, what))
        res[width] = got
    for a, b, what in zip(res[0], res[1], ("LD", "LL", "UD", "UL", "lmul!", "rmul!", "star")):
        compare(a, b, name, dtype, "merged vs unmerged " + what)


def test_set_values_into_a_merged_plan(gpu):
    """pp_set_values takes the caller's layout and places it into the merged blocks (padding = zero)."""
    n, I, J, W = graphs.grid2d(96, 96, 1.0, 10.0, seed=8, dtype=np.float64)
    cp, rv, nz = graphs.csc(n, I, J, W)
    S = pp.ssymbolic(n, cp, rv)
    A = OracleLU("MinPlus", np.float64, S).assemble(cp, rv, nz)
    F = pp.B200SLU(pp.MinPlus(), np.float64, S, device=0)
    try:
        F.set_values(A.LD, A.LL, A.UD, A.UL, A.Nval)
        assert F.stats()["plan_fronts"] < S.nf
        for got, want in zip(F.factors(), (A.LD, A.LL, A.UD, A.UL)):
            same(got, want, "MinPlus", np.float64, "set_values round trip")
        F.factor()
        O = A.factor()
        for got, want, what in zip(F.factors(), (O.LD, O.LL, O.UD, O.UL), ("LD", "LL", "UD", "UL")):
            same(got, want, "MinPlus", np.float64, "factor of uploaded values " + what)
        # switching to PlusProd rebuilds the plan unmerged on the same handle
        Wp = weights("PlusProd", np.float64, len(I), 3)
        cp2, rv2, nz2 = graphs.csc(n, I, J, Wp)
        G = pp.B200SLU(pp.PlusProd(), np.float64, S, device=0).assemble_csc(cp2, rv2, nz2).factor()
        try:
            assert G.stats()["plan_fronts"] == S.nf
        finally:
            G.close()
    finally:
        F.close()
