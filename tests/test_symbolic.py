"""The host symbolic stand-in (pp_symbolic) and the structure checks of pp_set_structure, on the CPU.

The structure must have the properties the reference's solver relies on (src/CPU/chordal_ssymbolic.jl:26-57,
src/CPU/chordal/sgetrf.jl:35-134): strongly connected components with every arc between them going from an
earlier component to a later one (sccs!, src/CPU/utils.jl:18-70), fronts in postorder whose parent is the front
of the first separator vertex, separators inside the parent's bag (running intersection), every arc inside a
component covered by a front, and the coupling N listing exactly the arcs between components (soffd,
src/CPU/chordal_ssymbolic.jl:212-269).
"""
import numpy as np
import pytest
import scipy.sparse as sp
from scipy.sparse.csgraph import connected_components

import pathpack_b200 as pp
from tests.helpers import graph

KINDS = ["grid", "grid40", "grid3d", "sprand", "knn"]


def arcs_in_positions(n, cp, rv, S):
    """(i, j) position pairs of every arc i -> j (A[i, j] stored in column j)."""
    col = np.repeat(np.arange(n), np.diff(cp))
    invp = S.invp
    return invp[rv], invp[col]


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("method", ["nd", "natural"])
def test_structure_properties(kind, method):
    n, cp, rv, _ = graph(kind, "MinPlus", np.float64)
    S = pp.ssymbolic(n, cp, rv, method)
    nn, na = S.nn, S.na
    # permutation and residual partition
    assert np.array_equal(np.sort(S.perm), np.arange(n))
    assert S.Rptr[0] == 0 and S.Rptr[-1] == n and np.all(nn >= 1)
    # components: vertex and front ranges
    assert S.Bptr[0] == 0 and S.Bptr[-1] == n and np.all(np.diff(S.Bptr) > 0)
    assert S.Fptr[0] == 0 and S.Fptr[-1] == S.nf and np.all(np.diff(S.Fptr) > 0)
    comp_of_pos = np.repeat(np.arange(S.nB), np.diff(S.Bptr))
    for b in range(S.nB):
        f0, f1 = S.Fptr[b], S.Fptr[b + 1]
        assert S.Rptr[f0] == S.Bptr[b] and S.Rptr[f1] == S.Bptr[b + 1]
    # the number of components is the number of strongly connected components
    A = sp.csc_matrix((np.ones(len(rv)), rv, cp), shape=(n, n))
    assert S.nB == connected_components(A, directed=True, connection="strong")[0]
    front_of = np.repeat(np.arange(S.nf), nn)
    par = S.parent()
    bags = []
    for f in range(S.nf):
        sep = S.Stgt[S.Sptr[f]:S.Sptr[f + 1]]
        res_end = S.Rptr[f + 1]
        assert np.all(np.diff(sep) > 0), "separator not sorted"
        if len(sep):
            assert sep[0] >= res_end, "separator before the residual"
            assert comp_of_pos[sep[-1]] == comp_of_pos[S.Rptr[f]], "separator leaves the component"
            p = front_of[sep[0]]
            assert par[f] == p and p > f, "not in postorder"
        bags.append(set(range(S.Rptr[f], res_end)) | set(sep.tolist()))
    for f in range(S.nf):
        if par[f] >= 0:
            sep = set(S.Stgt[S.Sptr[f]:S.Sptr[f + 1]].tolist())
            assert sep <= bags[par[f]], "separator outside the parent's bag"
    # every arc inside a component lies in the bag of the front of its earlier endpoint
    i, j = arcs_in_positions(n, cp, rv, S)
    inside = comp_of_pos[i] == comp_of_pos[j]
    for a, b in zip(i[inside], j[inside]):
        lo, hi = min(a, b), max(a, b)
        assert hi in bags[front_of[lo]], "arc %d-%d not covered" % (lo, hi)
    # coupling: exactly the arcs between components, from earlier to later components
    between = ~inside
    assert np.all(comp_of_pos[i[between]] < comp_of_pos[j[between]])
    want = set(zip(i[between].tolist(), j[between].tolist()))
    got = {(int(q), p) for p in range(n) for q in S.Ntgt[S.Nptr[p]:S.Nptr[p + 1]]}
    assert got == want


def test_layout_sums():
    """Dptr / Lptr are the running sums of nn^2 and nn * na (docs/site_factors.jl:147-156)."""
    n, cp, rv, _ = graph("grid3d", "MinPlus", np.float64)
    S = pp.ssymbolic(n, cp, rv)
    nD, nL, _ = S.sizes()
    assert nD == int((S.nn ** 2).sum()) and nL == int((S.nn * S.na).sum())


def test_pair_counts():
    """pairs_factor = sum_f [S2(nj) - S2(na)] with S2(m) = (m - 1) m (2m - 1) / 6: the partial LU of each front
    counted pivot by pivot, the same as the per-front formula nn^3/3-like terms of the measurement plan."""
    n, cp, rv, _ = graph("grid40", "MinPlus", np.float64)
    S = pp.ssymbolic(n, cp, rv)
    nn, na = S.nn.astype(float), S.na.astype(float)
    per_front = (nn - 1) * nn * (2 * nn - 1) / 6 + na * nn * (nn - 1) + na * na * nn
    assert abs(S.pairs_factor() - per_front.sum()) <= 1e-9 * per_front.sum()


def test_readme_graph_components():
    """The README's 5-vertex example: vertex 5 has no out-arcs, so it is its own (last) component and the
    others form one strongly connected component."""
    I = np.array([1, 1, 2, 3, 4, 4]) - 1
    J = np.array([2, 3, 4, 2, 1, 5]) - 1
    A = sp.csc_matrix((np.ones(6), (I, J)), shape=(5, 5))
    A.sort_indices()
    S = pp.ssymbolic(5, A.indptr.astype(np.int64), A.indices.astype(np.int64))
    assert S.nB == 2 and sorted(np.diff(S.Bptr).tolist()) == [1, 4]
    assert S.perm[S.Bptr[1]] == 4 or S.perm[0] == 4


@pytest.mark.parametrize("seed", range(6))
@pytest.mark.parametrize("density", [0.004, 0.012, 0.03])
def test_components_match_scipy(seed, density):
    """The components are exactly scipy's strongly connected components (same partition of the vertices),
    listed sources first: no arc goes from a later component to an earlier one."""
    rng = np.random.default_rng(seed)
    n = 300
    A = sp.random(n, n, density=density, random_state=rng, format="csc")
    A.setdiag(0)
    A.eliminate_zeros()
    A.sort_indices()
    cp, rv = A.indptr.astype(np.int64), A.indices.astype(np.int64)
    S = pp.ssymbolic(n, cp, rv)
    ncomp, lab = connected_components(A, directed=True, connection="strong")
    assert S.nB == ncomp
    comp_of_pos = np.repeat(np.arange(S.nB), np.diff(S.Bptr))
    ours = comp_of_pos[S.invp]  # component of each original vertex
    # the same partition: a bijection between the two labellings
    pairs = set(zip(ours.tolist(), lab.tolist()))
    assert len(pairs) == ncomp
    i, j = arcs_in_positions(n, cp, rv, S)
    assert np.all(comp_of_pos[i] <= comp_of_pos[j]), "an arc goes back to an earlier component"
