"""Parity of the B200 library (through the C ABI) with the oracle, on the GPU.

Every case runs the same seeded inputs through libpathpack_b200.so and through the oracle (the CPU
restatement of the reference solver) and compares: bit-exact for the idempotent semirings (the device
kernels keep the reference's per-element dataflow), rtol 1e-5 / 1e-12 for PlusProd and for the star of the
floating tropical semirings (whose dense triangular star the reference associates differently).
"""
import numpy as np
import pytest

import pathpack_b200 as pp
from oracle.oracle import OracleLU
from oracle import oracle as orc
from pathpack_b200 import graphs
from tests.helpers import CASES, EXACT, close, graph, same, weights

pytestmark = pytest.mark.gpu

SR = {s.__class__.__name__: s for s in [pp.MinPlus(), pp.MaxPlus(), pp.MaxMin(), pp.MinMax(), pp.MaxProd(),
                                         pp.PlusProd(), pp.OrAnd()]}


def torch_dt(dtype):
    import torch

    return {np.dtype(np.float32): torch.float32, np.dtype(np.float64): torch.float64,
            np.dtype(np.int32): torch.int32}[np.dtype(dtype)]


@pytest.mark.parametrize("name,dtype", CASES)
@pytest.mark.parametrize("mnk", [(1, 1, 1), (7, 5, 3), (33, 65, 17), (130, 129, 40), (257, 200, 129), (2, 4, 6),
                                 (192, 66, 96), (64, 130, 258)])
def test_gemm(gpu, name, dtype, mnk):
    """C (+)= A (x) B against the oracle.  For PlusProd Float64 the sizes with even leading dimensions (m and k
    even) run the TMA-staged tensor-core kernel, with partial tiles in m, n and k; the others the
    register-staged one."""
    import torch

    m, n, k = mnk
    rng = np.random.default_rng(m * 1000 + n * 10 + k)
    A = np.asfortranarray(weights(name, dtype, m * k, 1).reshape(m, k))
    B = np.asfortranarray(weights(name, dtype, k * n, 2).reshape(k, n))
    C = np.asfortranarray(weights(name, dtype, m * n, 3).reshape(m, n))
    if name != "OrAnd" and np.dtype(dtype) != np.int32:  # some "no path" entries
        A[rng.random(A.shape) < 0.2] = SR[name].zero(dtype)
    want = orc.gemm(name, C.copy(order="F"), A, B)
    td = torch_dt(dtype)
    At = torch.from_numpy(A.T.copy()).to("cuda").T  # column-major views
    Bt = torch.from_numpy(B.T.copy()).to("cuda").T
    Ct = torch.from_numpy(C.T.copy()).to("cuda").T
    L = pp.lib()
    pp._lib.check(L.pp_gemm(SR[name].id, pp.semiring.DTYPES[np.dtype(dtype)], m, n, k, Ct.data_ptr(), m,
                            At.data_ptr(), m, Bt.data_ptr(), k, None))
    torch.cuda.synchronize()
    got = Ct.cpu().numpy()
    assert Ct.dtype == td
    same(got, want, name, dtype, "gemm %s" % (mnk,))


@pytest.mark.parametrize("name,dtype", [("MinPlus", np.int32), ("MinPlus", np.float32), ("MaxMin", np.float64),
                                        ("PlusProd", np.float64), ("OrAnd", np.int32)])
@pytest.mark.parametrize("n", [1, 5, 64, 65, 128])
def test_getrf_batched(gpu, name, dtype, n):
    import torch

    count = 7
    A = weights(name, dtype, count * n * n, n).reshape(count, n, n)
    if name == "MinPlus":
        for b in range(count):
            np.fill_diagonal(A[b], 0)
    want = orc.getrf_batched(name, A.copy())
    At = torch.from_numpy(A.copy()).to("cuda")
    pp._lib.check(pp.lib().pp_getrf_batched(SR[name].id, pp.semiring.DTYPES[np.dtype(dtype)], n, count,
                                            At.data_ptr(), None))
    torch.cuda.synchronize()
    same(At.cpu().numpy(), want, name, dtype, "getrf n=%d" % n)


def factor_both(kind, name, dtype, seed=0):
    n, cp, rv, nz = graph(kind, name, dtype, seed)
    S = pp.ssymbolic(n, cp, rv)
    F = pp.B200SLU(SR[name], dtype, S, device=0).assemble_csc(cp, rv, nz).factor()
    O = OracleLU(name, dtype, S).assemble(cp, rv, nz).factor()
    return n, S, F, O


@pytest.mark.parametrize("name,dtype", CASES)
@pytest.mark.parametrize("kind", ["grid", "sprand", "knn", "grid3d"])
def test_factor_and_solves(gpu, name, dtype, kind):
    n, S, F, O = factor_both(kind, name, dtype)
    try:
        for got, want, what in zip(F.factors(), (O.LD, O.LL, O.UD, O.UL), ("LD", "LL", "UD", "UL")):
            same(got, want, name, dtype, "%s %s" % (kind, what))
        rng = np.random.default_rng(5)
        z, one = SR[name].zero(dtype), SR[name].one(dtype)
        k = 37
        B = np.full((n, k), z, dtype=dtype, order="F")
        src = rng.choice(n, size=k, replace=False)
        B[src, np.arange(k)] = one
        B[rng.random(B.shape) < 0.05] = one
        same(pp.lmul_(F, B.copy(order="F")), O.lmul(B), name, dtype, "%s lmul" % kind)
        R = np.asfortranarray(B.T)
        same(pp.rmul_(R.copy(order="F"), F), O.rmul(R), name, dtype, "%s rmul" % kind)
        C = pp.Matrix(F)
        close(C, O.star(), name, dtype, "%s star" % kind)
        # the star through lmul's dataflow is the oracle's lmul of the identity, bit for bit
        E = np.full((n, n), z, dtype=dtype, order="F")
        np.fill_diagonal(E, one)
        same(C, O.lmul(E), name, dtype, "%s star vs lmul(I)" % kind)
    finally:
        F.close()


@pytest.mark.parametrize("name,dtype", [("MinPlus", np.float64), ("MaxMin", np.float32), ("PlusProd", np.float64),
                                        ("MinPlus", np.float32)])
def test_large_fronts(gpu, name, dtype):
    """Fronts larger than the shared-memory kernel takes go through the blocked path (panel + GEMM)."""
    n, S, F, O = factor_both("grid3d14", name, dtype)
    try:
        assert (S.nn + S.na).max() > {4: 202, 8: 143}[np.dtype(dtype).itemsize], "no large front"
        for got, want, what in zip(F.factors(), (O.LD, O.LL, O.UD, O.UL), ("LD", "LL", "UD", "UL")):
            same(got, want, name, dtype, "grid3d14 %s" % what)
        B = np.asfortranarray(weights(name, dtype, n * 40, 9).reshape(n, 40))
        same(pp.lmul_(F, B.copy(order="F")), O.lmul(B), name, dtype, "grid3d14 lmul")
    finally:
        F.close()


@pytest.mark.parametrize("fixture", ["paris", "bunny"])
def test_reference_structures(gpu, fixture):
    """The reference's own AMF structures and factors (docs/src/public/data/*-lu.bin.gz): the device
    factorization of MinPlus Float32 reproduces PATHPACK.jl's factor bit for bit."""
    import os

    z = np.load(os.path.join(os.path.dirname(__file__), "golden", fixture + ".npz"))
    n = int(z["n"])
    from pathpack_b200 import graphs

    cp, rv, nz = graphs.csc(n, z["I"].astype(np.int64), z["J"].astype(np.int64), z["W"])
    S = pp.Structure.from_arrays(n, z["Rptr"], z["Sptr"], z["Stgt"], z["Bptr"], z["Fptr"], z["Nptr"], z["Ntgt"],
                                 z["perm"])
    F = pp.B200SLU(pp.MinPlus(), np.float32, S).assemble_csc(cp, rv, nz).factor()
    try:
        LD, LL, UD, UL = F.factors()
        nn = S.nn
        Dp = np.concatenate([[0], np.cumsum(nn * nn)])
        D = np.empty_like(UD)
        for f in range(S.nf):
            m = nn[f]
            blk = slice(Dp[f], Dp[f + 1])
            U = UD[blk].reshape(m, m, order="F")
            L = LD[blk].reshape(m, m, order="F")
            D[blk] = np.where(np.triu(np.ones((m, m), bool)), U, L).reshape(-1, order="F")
        same(D, z["D"], "MinPlus", np.float32, fixture + " D")
        same(UL, z["UL"], "MinPlus", np.float32, fixture + " UL")
        same(LL, z["LL"], "MinPlus", np.float32, fixture + " LL")
        O = OracleLU("MinPlus", np.float32, S).assemble(cp, rv, nz).factor()
        B = np.full((n, 16), np.inf, np.float32, order="F")
        B[np.arange(16) * 97 % n, np.arange(16)] = 0
        same(pp.lmul_(F, B.copy(order="F")), O.lmul(B), "MinPlus", np.float32, fixture + " lmul")
        R = np.asfortranarray(B.T)
        same(pp.rmul_(R.copy(order="F"), F), O.rmul(R), "MinPlus", np.float32, fixture + " rmul")
    finally:
        F.close()


@pytest.mark.parametrize("name,dtype", [("MinPlus", np.float64), ("MaxMin", np.float32)])
def test_star_panels(gpu, name, dtype):
    """The column panels of pathpack_b200.panels (one per rank of a multi-GPU star) put together are the whole
    star, bit for bit."""
    from pathpack_b200.panels import star_panel

    n, S, F, O = factor_both("sprand", name, dtype)
    try:
        full = pp.Matrix(F)
        for world in (2, 3, 8):
            parts = [star_panel(F, r, world) for r in range(world)]
            C = np.concatenate([c for _, c in parts], axis=1)
            assert [c0 for c0, _ in parts] == sorted(c0 for c0, _ in parts)
            same(C, full, name, dtype, "star from %d panels" % world)
    finally:
        F.close()


@pytest.mark.parametrize("name,dtype", [("MinPlus", np.float64), ("MaxMin", np.float32), ("PlusProd", np.float64),
                                        ("OrAnd", np.int32)])
@pytest.mark.parametrize("kind", ["grid3d", "knn"])
def test_star_device_output(gpu, name, dtype, kind):
    """Matrix(F) into device memory (its columns taken in elimination order and written to their own columns)
    equals the star into host memory (columns in label order), for whole and partial column ranges."""
    import torch

    n, S, F, O = factor_both(kind, name, dtype)
    try:
        for col0, ncols in [(0, n), (7, n - 20), (n // 3, 33), (5, 32), (n - 1, 1)]:
            host = F.star(col0, ncols)
            dev = torch.empty((ncols, n), dtype=torch_dt(dtype), device="cuda:0").t()
            F.star(col0, ncols, out=dev)
            same(dev.cpu().numpy(), host, name, dtype, "%s device star [%d, +%d)" % (kind, col0, ncols))
    finally:
        F.close()


@pytest.mark.parametrize("name,dtype", [("MinPlus", np.float64), ("MaxMin", np.float32), ("PlusProd", np.float64),
                                        ("OrAnd", np.int32), ("MaxPlus", np.float32)])
@pytest.mark.parametrize("k", [300, 513, 1100])
def test_wide_solves(gpu, name, dtype, k):
    """lmul! and rmul! with more than 256 right-hand sides (the top fronts' 128-column tasks) against the oracle."""
    n, S, F, O = factor_both("grid3d", name, dtype)
    try:
        rng = np.random.default_rng(k)
        z, one = SR[name].zero(dtype), SR[name].one(dtype)
        B = np.full((n, k), z, dtype=dtype, order="F")
        B[rng.integers(0, n, size=k), np.arange(k)] = one
        B[rng.random(B.shape) < 0.02] = one
        same(pp.lmul_(F, B.copy(order="F")), O.lmul(B), name, dtype, "wide lmul k=%d" % k)
        R = np.asfortranarray(B.T)
        same(pp.rmul_(R.copy(order="F"), F), O.rmul(R), name, dtype, "wide rmul k=%d" % k)
    finally:
        F.close()


def test_star_into_pageable_and_pinned_host_memory(gpu):
    """Matrix(F) into host memory: a pageable array goes through the library's page-locked ring (host threads copy
    each panel out while the GPU computes the next; four panels here, so the ring's three slots are reused) and a
    page-locked array takes the device-to-host copies directly; both equal the star computed into device memory."""
    import torch

    n, I, J, W = graphs.grid2d(100, 100, 1.0, 10.0, seed=21, dtype=np.float64)
    cp, rv, nz = graphs.csc(n, I, J, W)
    S = pp.ssymbolic(n, cp, rv)
    F = pp.B200SLU(pp.MinPlus(), np.float64, S, device=0).assemble_csc(cp, rv, nz).factor()
    try:
        pageable = F.star()
        pinned = torch.empty((n, n), dtype=torch.float64).pin_memory()
        F.star(out=pinned.numpy().T)  # the transpose of a row-major n x n array is column-major
        dev = torch.empty((n, n), dtype=torch.float64, device="cuda:0").t()
        F.star(out=dev)
        want = dev.cpu().numpy()
        assert np.array_equal(pageable.view(np.uint64), want.view(np.uint64))
        assert np.array_equal(pinned.numpy().T.view(np.uint64), want.view(np.uint64))
        part = F.star(5000, 4001)  # a column range that does not start a panel
        assert np.array_equal(part.view(np.uint64), want[:, 5000:9001].view(np.uint64))
    finally:
        F.close()


@pytest.mark.parametrize("name,dtype", [("MinPlus", np.float64), ("MaxMin", np.float32), ("OrAnd", np.int32),
                                        ("PlusProd", np.float64), ("MinPlus", np.int32)])
def test_star_columns_and_rows_of_a_source_set(gpu, name, dtype):
    """pp_star_cols / pp_star_rows: the star towards / from a set of vertices (unsorted, with a repeat), into
    host memory (pageable: the page-locked ring) and device memory; columns against lmul! of unit columns, rows
    against rmul! of unit rows, both the oracle's (rows: the apsp_gpu(A, sources) of the reference)."""
    import torch

    n, I, J, _ = graphs.grid2d(60, 50, seed=7)
    W = weights(name, dtype, len(I), 8)
    cp, rv, nz = graphs.csc(n, I, J, W)
    S = pp.ssymbolic(n, cp, rv)
    F = pp.B200SLU(SR[name], dtype, S, device=0).assemble_csc(cp, rv, nz).factor()
    O = OracleLU(name, dtype, S).assemble(cp, rv, nz).factor()
    try:
        rng = np.random.default_rng(3)
        src = rng.choice(n, 700, replace=False)
        src = np.concatenate([src, src[:1]])  # a repeated vertex
        z, one = SR[name].zero(dtype), SR[name].one(dtype)
        E = np.full((n, len(src)), z, dtype=dtype, order="F")
        E[src, np.arange(len(src))] = one
        want_c = O.lmul(E)
        want_r = O.rmul(np.asfortranarray(E.T))
        same(pp.star_cols(F, src), want_c, name, dtype, "star columns (host)")
        same(pp.star_rows(F, src), want_r, name, dtype, "star rows (host)")
        td = torch_dt(dtype)
        Dc = torch.empty((len(src), n), dtype=td, device="cuda:0").t()
        same(pp.star_cols(F, src, out=Dc).cpu().numpy(), want_c, name, dtype, "star columns (device)")
        Dr = torch.empty((n, len(src)), dtype=td, device="cuda:0").t()
        same(pp.star_rows(F, src, out=Dr).cpu().numpy(), want_r, name, dtype, "star rows (device)")
    finally:
        F.close()
