"""BASELINE.json's configurations at their full sizes on the GPU, against the oracle run on the same inputs.

  config 1  the whole 4,096^2 star (Matrix(F)) against the oracle's lmul!(I), bit for bit;
  config 2  the factor, lmul! of the 256 unit columns and rmul! of 256 unit rows, bit for bit;
  config 3  the MaxMin factor (12 G pairs) bit for bit; the whole 64,000^2 star computed into device memory
            (16.4 GB: the wide-panel path) and 2,048 of its columns, drawn from every part of the elimination
            order and of the label range, against the oracle's lmul!(I[:, cols]) bit for bit; a second star of
            the same factor gives the same bits (repeat-run identity at full size);
  config 4  the star of the coupled kNN graph (26 strongly connected components) into device memory and
            1,024 of its columns against the oracle bit for bit.
MinPlus and MaxMin are idempotent, so the device's dataflow gives the reference's bits.
"""
import os

import numpy as np
import pytest

import pathpack_b200 as pp
from oracle.oracle import OracleLU
from pathpack_b200 import graphs
from tests.helpers import same

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 1


def build(s, dtype, n, I, J, W):
    cp, rv, nz = graphs.csc(n, I, J, W)
    S = pp.ssymbolic(n, cp, rv)
    F = pp.B200SLU(s, dtype, S).assemble_csc(cp, rv, nz).factor()
    O = OracleLU(type(s).__name__, dtype, S).assemble(cp, rv, nz).factor(THREADS)
    return F, O, S


def unit_columns(n, cols, name, dtype):
    s = {"MinPlus": pp.MinPlus(), "MaxMin": pp.MaxMin()}[name]
    E = np.full((n, len(cols)), s.zero(dtype), dtype=dtype, order="F")
    E[np.asarray(cols), np.arange(len(cols))] = s.one(dtype)
    return E


def spread_columns(S, m, seed):
    """m distinct labels: half drawn uniformly from the labels, half from the elimination order (every part of
    the tree: leaves of all subtrees and the top separators)."""
    rng = np.random.default_rng(seed)
    a = rng.choice(S.n, m // 2, replace=False)
    pos = np.linspace(0, S.n - 1, m - m // 2).astype(np.int64)
    b = S.perm[pos]
    cols = np.unique(np.concatenate([a, b]))
    extra = np.setdiff1d(np.arange(S.n), cols)
    return np.sort(np.concatenate([cols, rng.choice(extra, m - len(cols), replace=False)]))


def test_config1_whole_star_vs_oracle(gpu):
    n, I, J, W = graphs.grid2d(64, 64, 1.0, 10.0, seed=11, dtype=np.float64)
    F, O, S = build(pp.MinPlus(), np.float64, n, I, J, W)
    try:
        same(F.star(), O.lmul(unit_columns(n, np.arange(n), "MinPlus", np.float64), THREADS), "MinPlus",
             np.float64, "config 1 star")
    finally:
        F.close()


def test_config2_factor_lmul_rmul_vs_oracle(gpu):
    n, I, J, W = graphs.grid2d(256, 256, 1.0, 10.0, seed=1000, dtype=np.float64)
    F, O, S = build(pp.MinPlus(), np.float64, n, I, J, W)
    try:
        for got, want, what in zip(F.factors(), (O.LD, O.LL, O.UD, O.UL), ("LD", "LL", "UD", "UL")):
            same(got, want, "MinPlus", np.float64, "config 2 " + what)
        B, _ = graphs.unit_columns(n, 256, seed=2000, dtype=np.float64)
        same(pp.lmul_(F, B.copy(order="F")), O.lmul(B, THREADS), "MinPlus", np.float64, "config 2 lmul!")
        R, _ = graphs.unit_columns(n, 256, seed=2001, dtype=np.float64)
        R = np.asfortranarray(R.T)
        same(pp.rmul_(R.copy(order="F"), F), O.rmul(R, THREADS), "MinPlus", np.float64, "config 2 rmul!")
    finally:
        F.close()


def test_config3_factor_and_star_columns_vs_oracle(gpu):
    import torch

    n, I, J, W = graphs.grid3d(40, 40, 40, seed=12, dtype=np.float32)
    F, O, S = build(pp.MaxMin(), np.float32, n, I, J, W)
    try:
        for got, want, what in zip(F.factors(), (O.LD, O.LL, O.UD, O.UL), ("LD", "LL", "UD", "UL")):
            same(got, want, "MaxMin", np.float32, "config 3 " + what)
        cols = spread_columns(S, 2048, 31)
        D = torch.empty((n, n), dtype=torch.float32, device="cuda:0").t()  # column-major n x n
        F.star(out=D)
        idx = torch.from_numpy(cols).cuda()
        got = D[:, idx].cpu().numpy()
        want = O.lmul(unit_columns(n, cols, "MaxMin", np.float32), THREADS)
        same(got, want, "MaxMin", np.float32, "config 3 star columns")
        # the same star again into a second buffer: identical bits everywhere (compared on the device)
        D2 = torch.empty_like(D.t()).t()
        F.star(out=D2)
        assert torch.equal(D.view(torch.int32), D2.view(torch.int32))
        del D, D2
    finally:
        F.close()


def test_config4_star_columns_vs_oracle(gpu):
    import torch

    n, I, J, W = graphs.knn_directed(32768, 6, seed=13, dtype=np.float32)
    F, O, S = build(pp.MinPlus(), np.float32, n, I, J, W)
    try:
        assert S.nB > 1
        for got, want, what in zip(F.factors(), (O.LD, O.LL, O.UD, O.UL), ("LD", "LL", "UD", "UL")):
            same(got, want, "MinPlus", np.float32, "config 4 " + what)
        cols = spread_columns(S, 1024, 41)
        D = torch.empty((n, n), dtype=torch.float32, device="cuda:0").t()
        F.star(out=D)
        got = D[:, torch.from_numpy(cols).cuda()].cpu().numpy()
        del D
        want = O.lmul(unit_columns(n, cols, "MinPlus", np.float32), THREADS)
        same(got, want, "MinPlus", np.float32, "config 4 star columns")
    finally:
        F.close()


def test_star_wide_device_panel(gpu):
    """Matrix(F) into device memory in one panel wider than 16,384 columns (the star takes panels of up to 32,768
    columns): 256 columns spread over the panel, bit for bit against the oracle's lmul! of their unit columns."""
    import torch

    n, I, J, W = graphs.grid2d(141, 141, 1.0, 10.0, seed=77, dtype=np.float32)
    cp, rv, nz = graphs.csc(n, I, J, W)
    S = pp.ssymbolic(n, cp, rv)
    F = pp.B200SLU(pp.MinPlus(), np.float32, S, device=0).assemble_csc(cp, rv, nz).factor()
    try:
        assert n > 16384
        out = torch.empty((n, n), dtype=torch.float32, device="cuda:0").t()  # column-major n x n
        F.star(0, n, out=out)
        cols = np.sort(np.random.default_rng(5).choice(n, 256, replace=False))
        O = OracleLU("MinPlus", np.float32, S).assemble(cp, rv, nz).factor()
        E = np.full((n, len(cols)), np.inf, dtype=np.float32, order="F")
        E[cols, np.arange(len(cols))] = 0.0
        want = O.lmul(E)
        got = out[:, torch.from_numpy(cols).cuda()].cpu().numpy()
        same(got, want, "MinPlus", np.float32, "star columns of a 19,881-column device panel")
    finally:
        F.close()
