"""Independent checks of the star that share no code with the solver (no symbolic phase, no factorization).

TEST INFRASTRUCTURE ONLY.  Restated from the reference's own test oracles:
  - floyd_warshall: test/core.jl:5-11, the closure I (+) A (+) A^2 (+) ... by Floyd-Warshall in a semiring
    given by (plus, times, zero, one);
  - kleene: test/gpu/stress.jl:23-55, Kleene's algorithm with the star of the pivot (handles negative
    cycles and non-idempotent PlusProd);
  - dijkstra: test/gpu/stress_large.jl:20-45, heap Dijkstra for MinPlus with non-negative weights (scipy).
Dense matrices, vectorised with numpy over one pivot at a time.
"""
import numpy as np

INF = np.inf


def semiring_ops(name, dtype):
    """(plus, times, zero, one, star) as numpy ufunc-style callables for the named semiring."""
    dtype = np.dtype(dtype)
    i32 = dtype == np.int32
    imax = np.iinfo(np.int32).max
    if name == "MinPlus":
        if i32:
            times = lambda a, b: np.minimum(a.astype(np.int64) + b, imax).astype(np.int32)
            return np.minimum, times, np.int32(imax), np.int32(0), lambda a: np.where(a >= 0, 0, np.iinfo(np.int32).min)
        def times(a, b):
            with np.errstate(invalid="ignore"):
                c = np.add(a, b)
            return np.where(np.isnan(c), INF, c).astype(dtype)
        return np.fmin, times, dtype.type(INF), dtype.type(0), lambda a: np.where(a >= 0, 0.0, -INF).astype(dtype)
    if name == "MaxPlus":
        def times(a, b):
            with np.errstate(invalid="ignore"):
                c = np.add(a, b)
            return np.where(np.isnan(c), -INF, c).astype(dtype)
        return np.fmax, times, dtype.type(-INF), dtype.type(0), lambda a: np.where(0 >= a, 0.0, INF).astype(dtype)
    if name == "MaxMin":
        return np.fmax, np.fmin, dtype.type(-INF), dtype.type(INF), lambda a: np.full_like(a, INF)
    if name == "MinMax":
        return np.fmin, np.fmax, dtype.type(INF), dtype.type(-INF), lambda a: np.full_like(a, -INF)
    if name == "MaxProd":
        def times(a, b):
            with np.errstate(invalid="ignore"):
                c = np.multiply(a, b)
            return np.where(np.isnan(c), 0.0, c).astype(dtype)
        return np.fmax, times, dtype.type(0), dtype.type(1), lambda a: np.where(1 >= a, 1.0, INF).astype(dtype)
    if name == "PlusProd":
        def star(a):
            with np.errstate(divide="ignore"):
                return np.where(a < 1, 1.0 / (1.0 - a), INF).astype(dtype)
        return np.add, np.multiply, dtype.type(0), dtype.type(1), star
    if name == "OrAnd":
        return np.bitwise_or, np.bitwise_and, np.int32(0), np.int32(imax), lambda a: np.full_like(a, imax)
    raise ValueError(name)


def dense(n, I, J, V, name, dtype):
    """The n x n dense matrix of arcs I -> J with weights V, duplicates combined with (+)."""
    plus, _, zero, _, _ = semiring_ops(name, dtype)
    D = np.full((n, n), zero, dtype=dtype)
    for i, j, v in zip(I, J, V):
        D[i, j] = plus(D[i, j], v)
    return D


def floyd_warshall(name, D):
    """test/core.jl:5-11: D[i, i] = one, then D[i, j] (+)= D[i, k] (x) D[k, j] for every pivot k
    (for idempotent semirings without negative cycles)."""
    plus, times, zero, one, _ = semiring_ops(name, D.dtype)
    D = D.copy()
    n = D.shape[0]
    for i in range(n):
        D[i, i] = one
    for k in range(n):
        D = plus(D, times(D[:, k:k + 1], D[k:k + 1, :]))
    return D


def kleene(name, D):
    """test/gpu/stress.jl:23-55: Kleene's algorithm, out of place at each pivot, then I (+) D."""
    plus, times, zero, one, star = semiring_ops(name, D.dtype)
    D = D.copy()
    n = D.shape[0]
    for k in range(n):
        t = star(np.asarray([D[k, k]]))[0]
        tkj = times(np.asarray(t, dtype=D.dtype), D[k, :])
        D = plus(D, times(D[:, k:k + 1], tkj[None, :]))
    for i in range(n):
        D[i, i] = plus(D[i, i], one)
    return D


def dijkstra_rows(n, I, J, V, sources):
    """Shortest-path rows from the sources (MinPlus, non-negative weights), float64, via scipy."""
    import scipy.sparse as sp
    from scipy.sparse.csgraph import dijkstra

    W = {}
    for i, j, v in zip(I, J, V):
        W[(i, j)] = min(W.get((i, j), np.inf), float(v))
    keys = list(W)
    A = sp.csr_matrix(([W[k] for k in keys], ([k[0] for k in keys], [k[1] for k in keys])), shape=(n, n))
    # explicit zero weights must survive: scipy treats stored zeros as arcs only in csgraph 'directed' mode
    return dijkstra(A, directed=True, indices=np.asarray(sources))
