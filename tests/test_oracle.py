"""The oracle (the C restatement of PATHPACK.jl's CPU solver, oracle/) pinned on the CPU, without a GPU.

* against the reference's own factorizations shipped with it (docs/src/public/data/{paris,bunny}-lu.bin.gz,
  MinPlus Float32 on CliqueTrees AMF structures, stored as tests/golden/*.npz by tests/golden/make_fixtures.py):
  with the reference's structure the oracle reproduces D, UL and LL bit for bit;
* against the known answers of the reference's README (README.md:75-127);
* against textbook algorithms (Floyd-Warshall test/core.jl:5-11, Kleene test/gpu/stress.jl:23-55, Dijkstra
  test/gpu/stress_large.jl:20-45) on every semiring and graph kind.
"""
import os

import numpy as np
import pytest
import scipy.sparse as sp

import pathpack_b200 as pp
from oracle import independent as ind
from oracle.oracle import OracleLU
from pathpack_b200 import graphs
from tests.helpers import CASES, EXACT, close, graph, same

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load_fixture(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    n = int(z["n"])
    cp, rv, nz = graphs.csc(n, z["I"].astype(np.int64), z["J"].astype(np.int64), z["W"])
    S = pp.Structure.from_arrays(n, z["Rptr"], z["Sptr"], z["Stgt"], z["Bptr"], z["Fptr"], z["Nptr"], z["Ntgt"],
                                 z["perm"])
    return z, n, cp, rv, nz, S


def merged_diagonal(S, LD, UD):
    """The reference fixtures' D: per front, the upper triangle and diagonal of UD, the strict lower triangle
    of LD (docs/site_factors.jl:163-171)."""
    nn = S.nn
    Dp = np.concatenate([[0], np.cumsum(nn * nn)])
    D = np.empty_like(UD)
    for f in range(S.nf):
        m = nn[f]
        blk = slice(Dp[f], Dp[f + 1])
        U = UD[blk].reshape(m, m, order="F")
        L = LD[blk].reshape(m, m, order="F")
        D[blk] = np.where(np.triu(np.ones((m, m), bool)), U, L).reshape(-1, order="F")
    return D


@pytest.mark.parametrize("fixture", ["paris", "bunny"])
def test_oracle_reproduces_reference_factor(fixture):
    z, n, cp, rv, nz, S = load_fixture(fixture)
    # the layout invariant the reference asserts (docs/site_factors.jl:147-156)
    nD, nL, nN = S.sizes()
    assert nD == len(z["D"]) and nL == len(z["UL"]) == len(z["LL"]) and nN == len(z["Nval"])
    O = OracleLU("MinPlus", np.float32, S).assemble(cp, rv, nz).factor()
    same(merged_diagonal(S, O.LD, O.UD), z["D"], "MinPlus", np.float32, fixture + " D")
    same(O.UL, z["UL"], "MinPlus", np.float32, fixture + " UL")
    same(O.LL, z["LL"], "MinPlus", np.float32, fixture + " LL")


@pytest.mark.parametrize("fixture", ["paris"])
def test_oracle_fixture_rows_are_shortest_paths(fixture):
    """rmul! rows of the reference-structured factor are Dijkstra distances (Float32 rounding)."""
    z, n, cp, rv, nz, S = load_fixture(fixture)
    O = OracleLU("MinPlus", np.float32, S).assemble(cp, rv, nz).factor()
    src = np.array([0, 17, n // 2, n - 1])
    B = np.full((len(src), n), np.inf, np.float32, order="F")
    B[np.arange(len(src)), src] = 0
    got = O.rmul(B)
    want = ind.dijkstra_rows(n, z["I"].astype(np.int64), z["J"].astype(np.int64), z["W"].astype(np.float64), src)
    assert np.array_equal(np.isinf(got), np.isinf(want))
    f = np.isfinite(want)
    np.testing.assert_allclose(got[f], want[f], rtol=1e-5)


README_A = ([1, 1, 2, 3, 4, 4], [2, 3, 4, 2, 1, 5], [3.0, 8.0, 1.0, 4.0, 2.0, 7.0])
INF = np.inf
README_MINPLUS = np.array([[0, 3, 8, 4, 11], [3, 0, 11, 1, 8], [7, 4, 0, 5, 12], [2, 5, 10, 0, 7],
                           [INF, INF, INF, INF, 0]])
README_MAXMIN = np.array([[INF, 4, 8, 1, 1], [1, INF, 1, 1, 1], [1, 4, INF, 1, 1], [2, 2, 2, INF, 7],
                          [-INF, -INF, -INF, -INF, INF]])


def readme_factor(name):
    I, J, V = (np.array(x) for x in README_A)
    A = sp.csc_matrix((V, (I - 1, J - 1)), shape=(5, 5))
    A.sort_indices()
    S = pp.ssymbolic(5, A.indptr.astype(np.int64), A.indices.astype(np.int64))
    return OracleLU(name, np.float64, S).assemble(A.indptr, A.indices, A.data).factor()


def test_readme_known_answers():
    assert np.array_equal(readme_factor("MinPlus").star(), README_MINPLUS)
    assert np.array_equal(readme_factor("MaxMin").star(), README_MAXMIN)
    F = readme_factor("MinPlus")
    b = np.full((5, 1), np.inf)
    b[4] = 0
    assert np.array_equal(F.lmul(b)[:, 0], [11, 8, 12, 7, 0])  # column 5: distances to vertex 5
    B = np.full((1, 5), np.inf)
    B[0, 0] = 0
    assert np.array_equal(F.rmul(B)[0], [0, 3, 8, 4, 11])  # row 1: distances from vertex 1


@pytest.mark.parametrize("name,dtype", CASES)
@pytest.mark.parametrize("kind", ["grid", "sprand", "knn"])
def test_oracle_star_is_the_kleene_star(name, dtype, kind):
    n, cp, rv, nz = graph(kind, name, dtype)
    if n > 500:
        pytest.skip("dense Kleene on %d vertices is slow in numpy" % n)
    S = pp.ssymbolic(n, cp, rv)
    O = OracleLU(name, dtype, S).assemble(cp, rv, nz).factor()
    I = np.repeat(np.arange(n), np.diff(cp))
    D = ind.dense(n, rv, I, nz, name, dtype)  # A[rowval, col] = weight of the arc row -> col
    K = ind.kleene(name, D)
    close(O.star(), K, name, dtype, "%s star vs Kleene" % kind)
    if name != "PlusProd":  # idempotent: Floyd-Warshall's path sums (exact where no rounding happens)
        close(O.star(), ind.floyd_warshall(name, D), name, dtype, "%s star vs Floyd-Warshall" % kind)


@pytest.mark.parametrize("kind", ["grid40", "knn", "grid3d"])
def test_oracle_lmul_is_dijkstra(kind):
    n, cp, rv, nz = graph(kind, "MinPlus", np.float64)
    S = pp.ssymbolic(n, cp, rv)
    O = OracleLU("MinPlus", np.float64, S).assemble(cp, rv, nz).factor()
    rng = np.random.default_rng(1)
    src = rng.choice(n, size=12, replace=False)
    B = np.full((n, len(src)), np.inf, order="F")
    B[src, np.arange(len(src))] = 0
    # lmul! column j: distances to src[j]; Dijkstra on the reversed graph from src[j]
    I = np.repeat(np.arange(n), np.diff(cp))
    want = ind.dijkstra_rows(n, I, rv, nz, src)  # arcs col -> row: reversed
    got = O.lmul(B)
    np.testing.assert_allclose(got.T, want, rtol=1e-12)


def test_oracle_int32_minplus_saturates():
    """Int32 MinPlus on [0, INT32_MAX]: INT32_MAX is 'no path' and absorbs in the product."""
    n, cp, rv, nz = graph("grid", "MinPlus", np.int32)
    S = pp.ssymbolic(n, cp, rv)
    O = OracleLU("MinPlus", np.int32, S).assemble(cp, rv, nz).factor()
    C = O.star()
    D = ind.dense(n, rv, np.repeat(np.arange(n), np.diff(cp)), nz, "MinPlus", np.int32)
    assert np.array_equal(C, ind.floyd_warshall("MinPlus", D))
    assert C.min() >= 0
