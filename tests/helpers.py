"""Shared helpers of the tests: seeded graphs with weights valid for each semiring, and comparisons."""
import numpy as np

from pathpack_b200 import graphs

SEMIRINGS = ["MinPlus", "MaxPlus", "MaxMin", "MinMax", "MaxProd", "PlusProd", "OrAnd"]
CASES = [(s, np.float32) for s in SEMIRINGS[:6]] + [(s, np.float64) for s in SEMIRINGS[:6]] + \
    [("MinPlus", np.int32), ("OrAnd", np.int32)]
EXACT = {"MinPlus", "MaxPlus", "MaxMin", "MinMax", "MaxProd", "OrAnd"}  # idempotent (+): same dataflow, same bits


def weights(name, dtype, m, seed, maxdeg=8):
    """m weights valid for the semiring: MaxPlus weights are negative (no positive cycle), PlusProd weights
    keep the spectral radius below 1, OrAnd weights are bit masks."""
    rng = np.random.default_rng(seed)
    dtype = np.dtype(dtype)
    if name == "OrAnd":
        return rng.integers(0, 2 ** 31 - 1, size=m, dtype=np.int64).astype(np.int32)
    if dtype == np.int32:
        return rng.integers(1, 1001, size=m).astype(np.int32)
    if name == "MinPlus":
        return rng.uniform(1.0, 10.0, size=m).astype(dtype)
    if name == "MaxPlus":
        return (-rng.uniform(1.0, 10.0, size=m)).astype(dtype)
    if name in ("MaxMin", "MinMax", "MaxProd"):
        return (1.0 - rng.uniform(0.0, 1.0, size=m)).astype(dtype)
    if name == "PlusProd":
        return rng.uniform(0.0, 0.9 / maxdeg, size=m).astype(dtype)
    raise ValueError(name)


def graph(kind, name, dtype, seed=0):
    """(n, colptr, rowval, nzval) of a test graph with weights for the semiring."""
    if kind == "grid":
        n, I, J, _ = graphs.grid2d(12, 10, seed=seed)
    elif kind == "grid40":
        n, I, J, _ = graphs.grid2d(40, 40, seed=seed)
    elif kind == "grid3d":
        n, I, J, _ = graphs.grid3d(8, 8, 8, seed=seed)
    elif kind == "grid3d14":
        n, I, J, _ = graphs.grid3d(14, 14, 14, seed=seed)
    elif kind == "sprand":
        n, I, J, _ = graphs.sprand(80, 0.03, seed=seed)
    elif kind == "knn":
        n, I, J, _ = graphs.knn_directed(400, 6, seed=seed)
    else:
        raise ValueError(kind)
    W = weights(name, dtype, len(I), seed + 17)
    return (n,) + graphs.csc(n, I, J, W)


def same(a, b, name, dtype, what=""):
    """Bit-exact for idempotent semirings, rtol 1e-5 (Float32) / 1e-12 (Float64) for PlusProd; the
    +-Inf patterns must agree everywhere."""
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape, what
    if name in EXACT:
        bad = a.view(np.uint32 if a.itemsize == 4 else np.uint64) != b.view(np.uint32 if b.itemsize == 4 else np.uint64)
        if np.any(bad):
            i = np.flatnonzero(bad)[:5]
            raise AssertionError("%s: %d of %d entries differ, e.g. at %s: %s vs %s" % (
                what, bad.sum(), bad.size, i, a.ravel()[i], b.ravel()[i]))
        return
    rtol = 1e-5 if np.dtype(dtype) == np.float32 else 1e-12
    assert np.array_equal(np.isinf(a), np.isinf(b)), what + ": Inf patterns differ"
    f = np.isfinite(b)
    np.testing.assert_allclose(a[f], b[f], rtol=rtol, atol=tiny_floor(dtype), err_msg=what)


def tiny_floor(dtype):
    """Absolute floor of the PlusProd comparisons: 100 x the smallest normal number.  Below the normal range
    (walk sums of 1e-38 in Float32) a value has fewer significant bits than the relative tolerance assumes,
    and the order of the additions decides its last ones."""
    return 100 * float(np.finfo(dtype).tiny) if np.dtype(dtype).kind == "f" else 0


def close(a, b, name, dtype, what=""):
    """Within the north-star tolerance: exact for MaxMin/MinMax/OrAnd and Int32, rtol 1e-5 / 1e-12 for the
    floating semirings, identical +-Inf patterns."""
    a, b = np.asarray(a), np.asarray(b)
    if name in ("MaxMin", "MinMax", "OrAnd") or np.dtype(dtype) == np.int32:
        return same(a, b, "MinPlus" if np.dtype(dtype) == np.int32 else name, dtype, what)
    rtol = 1e-5 if np.dtype(dtype) == np.float32 else 1e-12
    assert np.array_equal(np.isposinf(a), np.isposinf(b)), what + ": +Inf patterns differ"
    assert np.array_equal(np.isneginf(a), np.isneginf(b)), what + ": -Inf patterns differ"
    f = np.isfinite(b)
    np.testing.assert_allclose(a[f], b[f], rtol=rtol, atol=tiny_floor(dtype) if name == "PlusProd" else 0,
                               err_msg=what)
