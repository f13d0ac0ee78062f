"""BASELINE.json's configurations at their full sizes on the GPU, checked through properties that do not need
the oracle to run at that size: shortest and widest path columns against independent Dijkstra searches, the
batched getrf and the 8192^3 GEMMs against the oracle and exact recomputation on sampled entries.  (Config 2 is
bench.py's workload; its device result is compared with the oracle there and in test_gpu_parity.)"""
import heapq

import numpy as np
import pytest

import pathpack_b200 as pp
from oracle import independent as ind
from oracle import oracle as orc
from pathpack_b200 import graphs
from pathpack_b200._lib import check

pytestmark = pytest.mark.gpu


def factor(s, dtype, n, I, J, W):
    cp, rv, nz = graphs.csc(n, I, J, W)
    S = pp.ssymbolic(n, cp, rv)
    return pp.B200SLU(s, dtype, S).assemble_csc(cp, rv, nz).factor()


def widest_to(n, I, J, W, target):
    """Max-min capacity of the widest path from every vertex to `target` (Dijkstra on the reversed graph)."""
    radj = [[] for _ in range(n)]
    for i, j, w in zip(I.tolist(), J.tolist(), W.tolist()):
        radj[j].append((i, w))
    best = np.full(n, -np.inf)
    best[target] = np.inf
    heap = [(-np.inf, target)]
    done = np.zeros(n, bool)
    while heap:
        negc, v = heapq.heappop(heap)
        if done[v]:
            continue
        done[v] = True
        c = -negc
        for u, w in radj[v]:
            cu = min(c, w)
            if cu > best[u]:
                best[u] = cu
                heapq.heappush(heap, (-cu, u))
    return best


def test_config1_mstar_minplus_grid64(gpu):
    """mstar(MinPlus(), A) Float64 on the 64x64 grid digraph (4,096 vertices, 16,128 arcs): the whole star
    against Dijkstra on sampled rows."""
    n, I, J, W = graphs.grid2d(64, 64, 1.0, 10.0, seed=11, dtype=np.float64)
    F = factor(pp.MinPlus(), np.float64, n, I, J, W)
    try:
        C = F.star()
        assert C.shape == (n, n)
        src = np.random.default_rng(1).choice(n, 64, replace=False)
        want = ind.dijkstra_rows(n, I, J, W, src)  # distances from the sources
        np.testing.assert_allclose(C[src], want, rtol=1e-12)
        assert np.all(np.isfinite(C)) and np.all(np.diag(C) == 0)
    finally:
        F.close()


def test_config3_widest_paths_grid40(gpu):
    """mlu(MaxMin(), A) Float32 on the 40x40x40 7-point grid digraph (64,000 vertices, 374,400 arcs): columns
    of the star (a column panel, as Matrix(F) computes them) equal the widest-path capacities bit for bit."""
    n, I, J, W = graphs.grid3d(40, 40, 40, seed=12, dtype=np.float32)
    F = factor(pp.MaxMin(), np.float32, n, I, J, W)
    try:
        targets = np.random.default_rng(2).choice(n, 3, replace=False)
        for t in targets:
            col = F.star(int(t), 1)[:, 0]
            want = widest_to(n, I, J, W.astype(np.float64), int(t)).astype(np.float32)
            assert np.array_equal(col, want), "column %d: %d entries differ" % (t, (col != want).sum())
        # a 1024-column panel runs the blocked path (the widths of the real Matrix(F) panels)
        P = F.star(5000, 1024)
        assert P.shape == (n, 1024) and np.all(P[5000 + np.arange(1024), np.arange(1024)] == np.inf)
    finally:
        F.close()


def test_config4_knn_star_columns(gpu):
    """mstar(MinPlus(), A) Float32 on the directed 6-NN graph of 32,768 points (weights |p - q| x U[1, 1.2)),
    with its strongly connected components coupled: star columns against Dijkstra (Float32 rounding)."""
    n, I, J, W = graphs.knn_directed(32768, 6, seed=13, dtype=np.float32)
    F = factor(pp.MinPlus(), np.float32, n, I, J, W)
    try:
        assert F.S.nB > 1
        cols = np.random.default_rng(3).choice(n, 32, replace=False)
        C = np.concatenate([F.star(int(c), 1) for c in cols], axis=1)
        want = ind.dijkstra_rows(n, J, I, W.astype(np.float64), cols).T  # distances to the columns
        assert np.array_equal(np.isinf(C), np.isinf(want))
        f = np.isfinite(want)
        np.testing.assert_allclose(C[f], want[f], rtol=1e-5)
        # the whole star into device memory (two wide panels in elimination order): the same columns, bit for bit
        import torch

        D = torch.empty((n, n), dtype=torch.float32, device="cuda:0").t()
        F.star(out=D)
        got = D[:, torch.from_numpy(cols).cuda()].cpu().numpy()
        assert np.array_equal(got.view(np.uint32), C.view(np.uint32))
        del D
    finally:
        F.close()


def test_config5a_batched_getrf_int32(gpu):
    """4,096 dense 128x128 MinPlus Int32 blocks (entries U{1..1000}, diagonal 0, 40% of the off-diagonal
    entries INT32_MAX): all factored on the device, the first 512 compared with the oracle bit for bit."""
    import torch

    rng = np.random.default_rng(14)
    count, n = 4096, 128
    A = rng.integers(1, 1001, size=(count, n, n)).astype(np.int32)
    A[rng.random(A.shape) < 0.4] = np.iinfo(np.int32).max
    A[:, np.arange(n), np.arange(n)] = 0
    Ad = torch.from_numpy(A).cuda()
    check(pp.lib().pp_getrf_batched(0, 2, n, count, Ad.data_ptr(), None))
    torch.cuda.synchronize()
    got = Ad.cpu().numpy()
    want = orc.getrf_batched("MinPlus", np.ascontiguousarray(A[:512]), nthreads=8)
    assert np.array_equal(got[:512], want)


@pytest.mark.parametrize("name,dtype,sr,dt", [("MinPlus", np.int32, 0, 2), ("MinPlus", np.float32, 0, 0),
                                              ("PlusProd", np.float64, 5, 1)])
def test_config5b_gemm_8192(gpu, name, dtype, sr, dt):
    """C <- C (+) A (x) B at 8192^3: 64 sampled entries recomputed exactly (min over k of a + b in the element
    type), PlusProd Float64 (entries U[0, 1/8192)) within 1e-12."""
    import torch

    N = 8192
    g = torch.Generator(device="cuda").manual_seed(15)
    if dtype == np.int32:
        A = torch.randint(1, 1001, (N, N), dtype=torch.int32, device="cuda", generator=g)
        B = torch.randint(1, 1001, (N, N), dtype=torch.int32, device="cuda", generator=g)
        C = torch.full((N, N), 2 ** 31 - 1, dtype=torch.int32, device="cuda")
    elif dtype == np.float32:
        A = torch.rand((N, N), dtype=torch.float32, device="cuda", generator=g)
        B = torch.rand((N, N), dtype=torch.float32, device="cuda", generator=g)
        C = torch.full((N, N), float("inf"), dtype=torch.float32, device="cuda")
    else:
        A = torch.rand((N, N), dtype=torch.float64, device="cuda", generator=g) / N
        B = torch.rand((N, N), dtype=torch.float64, device="cuda", generator=g) / N
        C = torch.zeros((N, N), dtype=torch.float64, device="cuda")
    # column-major: the (i, j) entry of a torch tensor T stored as T.t() is T[j, i]
    check(pp.lib().pp_gemm(sr, dt, N, N, N, C.data_ptr(), N, A.data_ptr(), N, B.data_ptr(), N, None))
    torch.cuda.synchronize()
    rng = np.random.default_rng(16)
    ii, jj = rng.integers(0, N, 64), rng.integers(0, N, 64)
    Ah = A.cpu().numpy()  # Ah[k, i] = A(i, k)
    Bh = B.cpu().numpy()  # Bh[j, k] = B(k, j)
    Ch = C.cpu().numpy()  # Ch[j, i] = C(i, j)
    for i, j in zip(ii, jj):
        a, b = Ah[:, i], Bh[j, :]
        if name == "MinPlus":
            want = (a.astype(np.int64) + b).min() if dtype == np.int32 else (a + b).min()
            assert Ch[j, i] == want
        else:
            want = float(np.dot(a, b))
            assert abs(Ch[j, i] - want) <= 1e-12 * want
