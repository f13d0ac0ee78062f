"""Seeded synthetic graphs with the shapes of the benchmark configurations (and of the reference's test
graphs, test/gpu/graphs.jl:3-25, test/core.jl:13-20).  Arcs are (I, J, W): weight W[e] on the arc
I[e] -> J[e], i.e. A[I[e], J[e]] = W[e]; no self-loops unless stated; duplicates never generated.
"""
import numpy as np


def grid2d(nx, ny, lo=1.0, hi=10.0, seed=0, dtype=np.float64):
    """4-connected nx x ny grid digraph: each undirected edge gives two arcs with independent weights
    uniform in [lo, hi)."""
    rng = np.random.default_rng(seed)
    v = np.arange(nx * ny).reshape(ny, nx)
    h = np.stack([v[:, :-1].ravel(), v[:, 1:].ravel()], 1)
    w = np.stack([v[:-1, :].ravel(), v[1:, :].ravel()], 1)
    E = np.concatenate([h, w])
    I = np.concatenate([E[:, 0], E[:, 1]])
    J = np.concatenate([E[:, 1], E[:, 0]])
    W = rng.uniform(lo, hi, size=len(I)).astype(dtype)
    return nx * ny, I.astype(np.int64), J.astype(np.int64), W


def grid3d(nx, ny, nz, seed=0, dtype=np.float32):
    """7-point nx x ny x nz grid digraph, capacities uniform in (0, 1] independent per direction."""
    rng = np.random.default_rng(seed)
    v = np.arange(nx * ny * nz).reshape(nz, ny, nx)
    pairs = [np.stack([v[:, :, :-1].ravel(), v[:, :, 1:].ravel()], 1),
             np.stack([v[:, :-1, :].ravel(), v[:, 1:, :].ravel()], 1),
             np.stack([v[:-1, :, :].ravel(), v[1:, :, :].ravel()], 1)]
    E = np.concatenate(pairs)
    I = np.concatenate([E[:, 0], E[:, 1]])
    J = np.concatenate([E[:, 1], E[:, 0]])
    W = (1.0 - rng.uniform(0.0, 1.0, size=len(I))).astype(dtype)  # (0, 1]
    return nx * ny * nz, I.astype(np.int64), J.astype(np.int64), W


def knn_directed(npts, k=6, seed=0, dtype=np.float32):
    """Directed k-nearest-neighbour graph of npts points uniform in the unit square: arcs p -> each of its k
    nearest neighbours, weight = Euclidean length x an independent factor uniform in [1, 1.2)."""
    from scipy.spatial import cKDTree

    rng = np.random.default_rng(seed)
    P = rng.uniform(0.0, 1.0, size=(npts, 2))
    d, nb = cKDTree(P).query(P, k=k + 1)
    I = np.repeat(np.arange(npts), k)
    J = nb[:, 1:].ravel()
    W = (d[:, 1:].ravel() * rng.uniform(1.0, 1.2, size=npts * k)).astype(dtype)
    return npts, I.astype(np.int64), J.astype(np.int64), W


def sprand(n, p, lo=1.0, hi=100.0, seed=0, dtype=np.float64, loops=False):
    """Random digraph: each arc i -> j present with probability p, weights uniform in [lo, hi]."""
    rng = np.random.default_rng(seed)
    M = rng.random((n, n)) < p
    if not loops:
        np.fill_diagonal(M, False)
    I, J = np.nonzero(M)
    W = rng.uniform(lo, hi, size=len(I)).astype(dtype)
    return n, I.astype(np.int64), J.astype(np.int64), W


def csc(n, I, J, W):
    """(colptr, rowval, nzval) of A with A[I, J] = W (no duplicates), rows sorted within columns."""
    order = np.lexsort((I, J))
    I, J, W = I[order], J[order], W[order]
    colptr = np.zeros(n + 1, dtype=np.int64)
    np.add.at(colptr, J + 1, 1)
    return np.cumsum(colptr), I.astype(np.int64), np.ascontiguousarray(W)


def unit_columns(n, k, seed=0, dtype=np.float64, zero=np.inf, one=0.0):
    """n x k column-major matrix of szero with sone at k distinct seeded vertices, one per column
    (config 2's right-hand sides); returns (B, sources)."""
    rng = np.random.default_rng(seed)
    src = rng.choice(n, size=k, replace=False)
    B = np.full((n, k), zero, dtype=dtype, order="F")
    B[src, np.arange(k)] = one
    return B, src
