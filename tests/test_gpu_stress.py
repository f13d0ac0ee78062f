"""The device on the reference's stress families (tests/stress.py), against the oracle and Kleene, on the GPU.

Per case (seeded graph family, zero and signed-zero weights, negative arcs, one negative cycle, duplicate
arcs, self-loops, positive cycles for MaxPlus/MaxProd, coupled components) the factor, lmul!, rmul! and
Matrix(F) computed through the C ABI are compared with the oracle: bit for bit for every semiring but PlusProd
(the sign of a zero may differ where tests/stress.py:bits_equal says why), within rtol 1e-5 / 1e-12 and identical +-Inf patterns for PlusProd.  The star is
also checked against Kleene's algorithm, which shares no code with either.  Repeated runs must give the same
bits for the idempotent semirings (the reference's test/gpu/stress_large.jl:1-3).
"""
import numpy as np
import pytest

import pathpack_b200 as pp
from oracle.independent import kleene
from oracle.oracle import OracleLU
from tests import stress
from tests.test_stress_cpu import CASES, compare_closure

pytestmark = pytest.mark.gpu

SR = {s.__class__.__name__: s for s in [pp.MinPlus(), pp.MaxPlus(), pp.MaxMin(), pp.MinMax(), pp.MaxProd(),
                                         pp.PlusProd(), pp.OrAnd()]}


def check(got, want, name, dtype, what, solve=True):
    if name == "PlusProd":
        from tests.helpers import close

        close(got, want, name, dtype, what)
    else:
        stress.bits_equal(got, want, name, dtype, what, solve)


def run_case(c, k=19):
    name, dtype, n = c["name"], c["dtype"], c["n"]
    S = pp.ssymbolic(n, c["cp"], c["rv"])
    F = pp.B200SLU(SR[name], dtype, S, device=0).assemble_csc(c["cp"], c["rv"], c["nz"]).factor()
    try:
        O = OracleLU(name, dtype, S).assemble(c["cp"], c["rv"], c["nz"]).factor()
        for got, want, what in zip(F.factors(), (O.LD, O.LL, O.UD, O.UL), ("LD", "LL", "UD", "UL")):
            check(got, want, name, dtype, "%s %s" % (c["tag"], what), solve=False)
        rng = np.random.default_rng(n)
        z, one = SR[name].zero(dtype), SR[name].one(dtype)
        B = np.full((n, k), z, dtype=dtype, order="F")
        B[rng.integers(0, n, size=k), np.arange(k)] = one
        B[rng.random(B.shape) < 0.1] = one
        check(pp.lmul_(F, B.copy(order="F")), O.lmul(B), name, dtype, c["tag"] + " lmul")
        R = np.asfortranarray(B.T)
        check(pp.rmul_(R.copy(order="F"), F), O.rmul(R), name, dtype, c["tag"] + " rmul")
        C = pp.Matrix(F)
        E = np.full((n, n), z, dtype=dtype, order="F")
        np.fill_diagonal(E, one)
        check(C, O.lmul(E), name, dtype, c["tag"] + " star vs the oracle's lmul(I)")
        compare_closure(C, kleene(name, stress.dense_of(c)), name, dtype, c["tag"] + " star vs Kleene")
        return F, C
    except BaseException:
        F.close()
        raise


@pytest.mark.parametrize("name,dtype", CASES)
@pytest.mark.parametrize("seed", range(12))
def test_stress_random(gpu, name, dtype, seed):
    F, _ = run_case(stress.draw(7919 * seed + 3, name, dtype))
    F.close()


@pytest.mark.parametrize("switch", ["negative", "negcycle", "selfloops", "dups", "zeros", "asym"])
@pytest.mark.parametrize("name,dtype", [("MinPlus", np.float32), ("MinPlus", np.float64), ("MaxPlus", np.float32),
                                        ("MaxProd", np.float64), ("MaxMin", np.float32), ("MinMax", np.float64)])
def test_stress_each_switch(gpu, switch, name, dtype):
    """One switch forced on, on a graph large enough that the top of the tree runs on the tile kernels."""
    kw = {switch: True}
    if switch == "negcycle":
        kw["asym"] = False
    F, C = run_case(stress.draw(101, name, dtype, kind="er", n=250, above_one=True, **kw))
    F.close()
    if switch == "negcycle" and name == "MinPlus":
        assert np.isneginf(C).any()


@pytest.mark.parametrize("name,dtype", [("MinPlus", np.float64), ("MaxMin", np.float32), ("OrAnd", np.int32),
                                        ("MaxPlus", np.float64), ("MinMax", np.float32), ("MaxProd", np.float32)])
def test_repeat_runs_bit_identical(gpu, name, dtype):
    """Two factorizations and stars of the same input give the same bits (idempotent (+): no run-dependent
    association anywhere, the atomics included)."""
    c = stress.draw(55, name, dtype, kind="grid", n=250, dups=True, zeros=True)
    S = pp.ssymbolic(c["n"], c["cp"], c["rv"])
    outs = []
    for _ in range(2):
        F = pp.B200SLU(SR[name], dtype, S, device=0).assemble_csc(c["cp"], c["rv"], c["nz"]).factor()
        try:
            outs.append((F.factors(), pp.Matrix(F)))
        finally:
            F.close()
    (f0, c0), (f1, c1) = outs
    u = np.uint32 if np.dtype(dtype).itemsize == 4 else np.uint64
    for a, b in zip(f0 + (c0,), f1 + (c1,)):
        assert np.array_equal(np.asarray(a).view(u), np.asarray(b).view(u))


def test_int32_minplus_refuses_negative_weights(gpu):
    """Int32 MinPlus is defined on [0, INT32_MAX]; a negative weight is refused before any device work."""
    c = stress.draw(3, "MinPlus", np.int32, kind="grid", n=25)
    nz = c["nz"].copy()
    nz[0] = -1
    S = pp.ssymbolic(c["n"], c["cp"], c["rv"])
    F = pp.B200SLU(pp.MinPlus(), np.int32, S, device=0)
    try:
        with pytest.raises(pp.PPError) as e:
            F.assemble_csc(c["cp"], c["rv"], nz)
        assert e.value.code == pp._lib.PP_EUNSUPPORTED
    finally:
        F.close()
