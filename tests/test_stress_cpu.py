"""The oracle on the reference's stress families, against an independent closure, on the CPU.

Each case (tests/stress.py: Erdos-Renyi, grid, tree, path, star, dense and disconnected graphs with zero
weights, negative arcs, one negative cycle, duplicate arcs, self-loops, signed zeros, positive cycles for
MaxPlus/MaxProd and coupled components) is factored by the oracle (the C restatement of the reference CPU
solver) and its whole star is compared with Kleene's algorithm (oracle/independent.py, the reference's own
stress oracle, test/gpu/stress.jl:23-55), which shares no code with the solver.  The comparison is the
reference's: `isequal` (identical +Inf / -Inf patterns, equal values) for every semiring whose arithmetic is
exact on these weights, and a relative tolerance for PlusProd and fractional MaxProd products, whose rounding
depends on the association.
"""
import zlib

import numpy as np
import pytest

import pathpack_b200 as pp
from oracle.independent import kleene
from oracle.oracle import OracleLU
from tests import stress

CASES = [("MinPlus", np.float32), ("MinPlus", np.float64), ("MinPlus", np.int32), ("MaxPlus", np.float32),
         ("MaxPlus", np.float64), ("MaxMin", np.float32), ("MaxMin", np.float64), ("MinMax", np.float32),
         ("MinMax", np.float64), ("MaxProd", np.float32), ("MaxProd", np.float64), ("PlusProd", np.float32),
         ("PlusProd", np.float64), ("OrAnd", np.int32)]


def compare_closure(got, want, name, dtype, tag):
    if name in ("PlusProd", "MaxProd"):
        assert np.array_equal(np.isposinf(got), np.isposinf(want)), tag + ": +Inf patterns differ"
        f = np.isfinite(want)
        rtol = 1e-5 if np.dtype(dtype) == np.float32 else 1e-12
        np.testing.assert_allclose(got[f], want[f], rtol=rtol, atol=1e-30, err_msg=tag)
    else:
        stress.equal_values(got, want, tag)


@pytest.mark.parametrize("name,dtype", CASES)
@pytest.mark.parametrize("seed", range(20))
def test_oracle_star_vs_kleene(name, dtype, seed):
    c = stress.draw(1000 * seed + 7, name, dtype, nmax=100)
    S = pp.ssymbolic(c["n"], c["cp"], c["rv"])
    O = OracleLU(name, dtype, S).assemble(c["cp"], c["rv"], c["nz"]).factor()
    compare_closure(O.star(), kleene(name, stress.dense_of(c)), name, dtype, c["tag"])


@pytest.mark.parametrize("switch", ["negative", "negcycle", "selfloops", "dups", "zeros", "asym"])
@pytest.mark.parametrize("kind", stress.KINDS)
def test_oracle_each_switch(switch, kind):
    """Every family with one switch forced on (MinPlus Float64 for the negative families, where -Inf stars and
    the NaN rule appear; MaxPlus Float32 with positive cycles, where +Inf stars appear, for the others)."""
    name, dtype = ("MinPlus", np.float64) if switch in ("negative", "negcycle", "selfloops") else ("MaxPlus", np.float32)
    kw = {switch: True}
    if switch == "negcycle":
        kw["asym"] = False  # keep the arc pair that closes the cycle
    seed = zlib.crc32(("%s/%s" % (switch, kind)).encode()) % 10000
    c = stress.draw(seed, name, dtype, kind=kind, n=60, above_one=True, **kw)
    S = pp.ssymbolic(c["n"], c["cp"], c["rv"])
    O = OracleLU(name, dtype, S).assemble(c["cp"], c["rv"], c["nz"]).factor()
    got = O.star()
    compare_closure(got, kleene(name, stress.dense_of(c)), name, dtype, c["tag"])
    if switch == "negcycle" and kind not in ("pieces",):
        assert np.isneginf(got).any(), "a negative cycle gives -Inf distances"


def test_families_reach_the_edge_cases():
    """The generator produces what the cases are for: -Inf and +Inf stars, NaN-rule products (+Inf + -Inf),
    signed zeros and coupled components."""
    seen = dict(neginf=False, posinf_maxplus=False, negzero=False, coupled=False)
    for seed in range(60):
        c = stress.draw(seed, "MinPlus", np.float64, negcycle=True, kind="er", n=40)
        D = kleene("MinPlus", stress.dense_of(c))
        seen["neginf"] |= bool(np.isneginf(D).any() and np.isposinf(D).any())
        c = stress.draw(seed, "MaxPlus", np.float32, above_one=True, kind="grid", n=25)
        seen["posinf_maxplus"] |= bool(np.isposinf(kleene("MaxPlus", stress.dense_of(c))).any())
        c = stress.draw(seed, "MaxMin", np.float32, zeros=True, kind="dense", n=17)
        seen["negzero"] |= bool(np.signbit(c["nz"][c["nz"] == 0]).any())
        c = stress.draw(seed, "MinPlus", np.float32, asym=True, kind="er", n=60)
        seen["coupled"] |= pp.ssymbolic(c["n"], c["cp"], c["rv"]).nB > 1
    assert all(seen.values()), seen


def test_unsupported_pairs_are_refused():
    """A semiring / element type the backend cannot compute exactly is refused, not answered (the reference
    checks the same with check_semiring, test/gpu/stress.jl:191-200)."""
    for s, dt in [(pp.OrAnd(), np.float32), (pp.OrAnd(), np.float64), (pp.MaxPlus(), np.int32),
                  (pp.PlusProd(), np.int32), (pp.MaxMin(), np.int32)]:
        assert not pp.semiring.supported(s, dt)
        with pytest.raises(TypeError):
            pp.B200SLU(s, dt, pp.ssymbolic(2, np.array([0, 1, 2]), np.array([1, 0])))
        assert pp.lib().pp_check_semiring(s.id, pp.semiring.DTYPES[np.dtype(dt)]) == pp._lib.PP_EUNSUPPORTED
