"""Seeded stress graphs: the families of the reference's randomized stress suite, written anew.

The reference's suite (test/gpu/stress.jl:62-140) draws a graph family (Erdos-Renyi, grid, random tree,
path, star, dense, disconnected pieces), integer-valued weights 0..100 (so that zero weights occur and sums
are exact), and switches on negative arcs (potential reweighting, which adds no negative cycle), one negative
cycle, duplicate arcs (combined with the semiring's (+), as `sparse(..., combine)` does) and self-loops.
This module adds signed zeros (+0.0 and -0.0 weights), the +Inf stars of MaxPlus and MaxProd (weights above
the semiring's one, i.e. positive cycles), and an optional asymmetric pattern so that several strongly
connected components are coupled (the reference's GPU stress uses symmetric patterns only).

TEST INFRASTRUCTURE ONLY.
"""
import numpy as np

KINDS = ("er", "grid", "tree", "path", "star", "dense", "pieces")
SIZES = (1, 2, 3, 5, 8, 17, 33, 60, 100, 160, 250)


def edges(rng, kind, n):
    """(I, J, n) of an undirected edge list of the family; grids round n down to a square."""
    I, J = [], []
    if kind == "er":
        d = rng.choice((1.5, 3.0, 6.0))
        m = int(round(d * n / 2))
        I, J = list(rng.integers(0, n, m)), list(rng.integers(0, n, m))
    elif kind == "grid":
        a = max(1, int(np.sqrt(n)))
        n = a * a
        for j in range(a):
            for i in range(a):
                v = i + j * a
                if i < a - 1:
                    I.append(v), J.append(v + 1)
                if j < a - 1:
                    I.append(v), J.append(v + a)
    elif kind == "tree":
        for v in range(1, n):
            I.append(v), J.append(int(rng.integers(0, v)))
    elif kind == "path":
        for v in range(1, n):
            I.append(v - 1), J.append(v)
    elif kind == "star":
        for v in range(1, n):
            I.append(0), J.append(v)
    elif kind == "dense":
        for i in range(n):
            for j in range(i + 1, n):
                if rng.random() < 0.5:
                    I.append(i), J.append(j)
    elif kind == "pieces":  # disconnected, with isolated vertices
        for _ in range(n):
            u = int(rng.integers(0, n))
            v = int(rng.integers(max(0, u - 5), min(n, u + 6)))
            if rng.random() < 0.6:
                I.append(u), J.append(v)
    else:
        raise ValueError(kind)
    return np.asarray(I, np.int64), np.asarray(J, np.int64), n


def combine(name, dtype, I, J, V, n):
    """CSC (colptr, rowval, nzval) of the arcs with duplicates combined by the semiring's (+)."""
    key = J * n + I
    order = np.argsort(key, kind="stable")
    key, I, J, V = key[order], I[order], J[order], V[order]
    first = np.ones(len(key), bool)
    first[1:] = key[1:] != key[:-1]
    starts = np.flatnonzero(first)
    if len(V):
        ufunc = {"MinPlus": np.minimum, "MinMax": np.minimum, "MaxPlus": np.maximum, "MaxMin": np.maximum,
                 "MaxProd": np.maximum, "PlusProd": np.add, "OrAnd": np.bitwise_or}[name]
        V = ufunc.reduceat(V, starts).astype(dtype)
    I, J = I[starts], J[starts]
    colptr = np.zeros(n + 1, np.int64)
    np.add.at(colptr, J + 1, 1)
    return np.cumsum(colptr), I.astype(np.int64), np.ascontiguousarray(V, dtype=dtype)


def draw(seed, name, dtype, kind=None, n=None, negative=None, negcycle=None, selfloops=None, dups=None,
         zeros=None, asym=None, above_one=None, nmax=250):
    """One stress case: a dict with n, colptr, rowval, nzval and a tag naming the switches."""
    rng = np.random.default_rng(seed)
    dtype = np.dtype(dtype)
    kind = kind or KINDS[int(rng.integers(len(KINDS)))]
    if n is None:
        sizes = [s for s in SIZES if s <= nmax]
        n = int(sizes[int(rng.integers(len(sizes)))])
    flip = lambda p, v: bool(rng.random() < p) if v is None else bool(v)
    negative, negcycle = flip(0.25, negative), flip(0.1, negcycle)
    selfloops, dups, zeros, asym = flip(0.2, selfloops), flip(0.2, dups), flip(0.3, zeros), flip(0.3, asym)
    above_one = flip(0.5, above_one)
    is_int = dtype == np.int32
    if name != "MinPlus" or is_int:
        negative = negcycle = False  # -Inf is not representable in Int32; other semirings have no "negative"
    I, J, n = edges(rng, kind, n)
    keep = I != J
    I, J = I[keep], J[keep]
    m = len(I)

    def w(k):
        if name == "OrAnd":
            return rng.integers(0, 2 ** 31 - 1, size=k, dtype=np.int64).astype(np.int32)
        if name == "PlusProd":
            return (rng.random(k) / (4 * max(1, n))).astype(dtype)
        v = rng.integers(0, 101, size=k).astype(dtype)
        if name == "MaxPlus" and not above_one:
            v = -v  # no positive cycle: finite longest paths
        if name in ("MaxProd",) and not above_one:
            v = (v / 100).astype(dtype)  # in [0, 1]: finite stars
        return v

    if asym and m:
        # drop one direction of a third of the edges: the pattern loses symmetry and splits into coupled SCCs
        back = rng.random(m) >= 1 / 3
        II, JJ = np.concatenate([I, J[back]]), np.concatenate([J, I[back]])
    else:
        II, JJ = np.concatenate([I, J]), np.concatenate([J, I])
    if name == "PlusProd" and not asym:
        V0 = w(m)
        VV = np.concatenate([V0, V0])  # symmetric, so that I - A is a nonsingular M-matrix
    else:
        VV = w(len(II))
    if negative:  # potential reweighting: w + phi[i] - phi[j] adds no negative cycle
        phi = rng.integers(0, 201, size=n).astype(dtype)
        VV = (VV + phi[II] - phi[JJ]).astype(dtype)
    if negcycle and m:  # one arc whose pair has negative total weight
        e = int(rng.integers(m))
        II, JJ, VV = np.append(II, I[e]), np.append(JJ, J[e]), np.append(VV, dtype.type(-150))
    if dups and len(II):
        for _ in range(max(1, m // 5)):
            e = int(rng.integers(len(II)))
            II, JJ, VV = np.append(II, II[e]), np.append(JJ, JJ[e]), np.append(VV, w(1))
    if selfloops:
        loops = rng.integers(0, n, size=max(1, n // 10))
        lw = np.full(len(loops), -3, dtype) if (name == "MinPlus" and negcycle) else w(len(loops))
        II, JJ, VV = np.concatenate([II, loops]), np.concatenate([JJ, loops]), np.concatenate([VV, lw])
    if zeros and dtype != np.int32 and name != "PlusProd" and len(VV):
        z = rng.random(len(VV))
        VV = VV.copy()
        VV[z < 0.1] = dtype.type(0.0)
        VV[(z >= 0.1) & (z < 0.2)] = dtype.type(-0.0)
    cp, rv, nz = combine(name, dtype, II.astype(np.int64), JJ.astype(np.int64), VV.astype(dtype), n)
    tag = "%s %s %s n=%d neg=%d negcyc=%d loops=%d dups=%d zeros=%d asym=%d above1=%d" % (
        name, dtype, kind, n, negative, negcycle, selfloops, dups, zeros, asym, above_one)
    return dict(n=n, cp=cp, rv=rv, nz=nz, tag=tag, name=name, dtype=dtype)


def dense_of(case):
    """The n x n matrix of the case's arcs (szero elsewhere), for the independent oracles."""
    from oracle.independent import semiring_ops

    n, cp, rv, nz = case["n"], case["cp"], case["rv"], case["nz"]
    zero = semiring_ops(case["name"], case["dtype"])[2]
    D = np.full((n, n), zero, dtype=case["dtype"])
    col = np.repeat(np.arange(n), np.diff(cp))
    D[rv, col] = nz
    return D


def equal_values(a, b, what=""):
    """Exact equality of two results as values: the same +Inf and -Inf masks, no NaN, equal elsewhere (a zero
    equals a zero of either sign)."""
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape, what
    assert not np.isnan(a).any() and not np.isnan(b).any(), what + ": NaN in a result"
    assert np.array_equal(np.isposinf(a), np.isposinf(b)), what + ": +Inf patterns differ"
    assert np.array_equal(np.isneginf(a), np.isneginf(b)), what + ": -Inf patterns differ"
    bad = a != b
    if bad.any():
        i = np.flatnonzero(bad)[:5]
        raise AssertionError("%s: %d entries differ, e.g. %s vs %s" % (what, bad.sum(), a.ravel()[i], b.ravel()[i]))


def bits_equal(a, b, name, dtype, what="", solve=False):
    """Bit-exact, except for the sign of a zero, which the order in which equal values meet in (+) decides.
    (1) Float32 min/max on the device are the hardware min/max (the reference's GPU kernels use the same,
    llvm.minnum), which order -0.0 below +0.0, where the reference CPU's select ifelse(x < y, x, y) returns its
    second operand on a tie.  (2) The solves' separator scatters (lmul!, rmul!, the star) combine the
    contributions of several fronts with atomics in whatever order they arrive (the reference's GPU scatters,
    atomic_splus!, have the same freedom).  (3) Merged fronts (amalgamation, as the reference's GPU path does)
    combine the children's update matrices and the entries of A in one front instead of member by member.
    `solve` is kept for the callers; every float comparison allows a zero of either sign."""
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape, what
    u = np.uint32 if a.itemsize == 4 else np.uint64
    bad = a.view(u) != b.view(u)
    if np.dtype(dtype).kind == "f":
        bad &= ~((a == 0) & (b == 0))
    if bad.any():
        i = np.flatnonzero(bad)[:5]
        raise AssertionError("%s: %d of %d entries differ, e.g. at %s: %s vs %s" % (
            what, bad.sum(), bad.size, i, a.ravel()[i], b.ravel()[i]))
