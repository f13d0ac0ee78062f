"""pp_lmul_static, the lmul! entry point that allocates nothing, against pp_lmul on the GPU.

The library's static per-device scratch replaces the handle's right-hand-side workspace and sweep counters;
the kernels are the same, so two calls in a row must each give pp_lmul's result (bit for bit for the
idempotent semirings, within rtol 1e-12 for PlusProd Float64, whose separator scatter adds in a run-dependent
order), and must leave the device's free memory unchanged.  Collected last so that it also runs after every
other test in one process.
"""
import numpy as np
import pytest

import pathpack_b200 as pp
from pathpack_b200 import _lib
from tests.helpers import graph, same

pytestmark = pytest.mark.gpu

SR = {s.__class__.__name__: s for s in [pp.MinPlus(), pp.MaxPlus(), pp.MaxMin(), pp.MinMax(), pp.MaxProd(),
                                         pp.PlusProd(), pp.OrAnd()]}
SCRATCH = 32 << 20  # PP_STATIC_SCRATCH_BYTES


def torch_dt(dtype):
    import torch

    return {np.dtype(np.float32): torch.float32, np.dtype(np.float64): torch.float64,
            np.dtype(np.int32): torch.int32}[np.dtype(dtype)]


def factored(kind, name, dtype):
    n, cp, rv, nz = graph(kind, name, dtype, seed=3)
    S = pp.ssymbolic(n, cp, rv)
    return n, pp.B200SLU(SR[name], dtype, S, device=0).assemble_csc(cp, rv, nz).factor()


def sources(n, k, name, dtype, seed=11):
    rng = np.random.default_rng(seed)
    z, one = SR[name].zero(dtype), SR[name].one(dtype)
    B = np.full((n, k), z, dtype=dtype, order="F")
    B[rng.choice(n, size=k, replace=k > n), np.arange(k)] = one
    B[rng.random(B.shape) < 0.05] = one
    return B


def on_device(B):
    import torch

    t = torch.empty((B.shape[1], B.shape[0]), dtype=torch_dt(B.dtype), device="cuda:0").t()
    t.copy_(torch.from_numpy(np.ascontiguousarray(B.T)).t())
    return t


@pytest.mark.parametrize("kind,name,dtype,k", [("grid40", "MinPlus", np.float64, 64),
                                               ("grid3d", "PlusProd", np.float64, 37),
                                               ("knn", "MinPlus", np.int32, 96),
                                               ("sprand", "OrAnd", np.int32, 33),
                                               ("grid", "MaxMin", np.float32, 120)])
def test_static_matches_lmul(gpu, kind, name, dtype, k):
    import torch

    n, F = factored(kind, name, dtype)
    try:
        B = sources(n, k, name, dtype)
        want = on_device(B)
        F._solve(want, True)  # pp_lmul, device-resident
        want = want.cpu().numpy()
        first, second = on_device(B), on_device(B)
        F.lmul_static(first)  # the first call also does the per-device setup
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info(0)[0]
        F.lmul_static(second)
        torch.cuda.synchronize()
        free1 = torch.cuda.mem_get_info(0)[0]
        assert free1 == free0, "pp_lmul_static changed the free device memory: %d -> %d" % (free0, free1)
        same(first.cpu().numpy(), want, name, dtype, "%s first static call" % kind)
        same(second.cpu().numpy(), want, name, dtype, "%s second static call" % kind)
        # and again after pp_lmul has used the handle's own workspace in between
        third = on_device(B)
        F._solve(on_device(B), True)
        F.lmul_static(third)
        same(third.cpu().numpy(), want, name, dtype, "%s static call after pp_lmul" % kind)
    finally:
        F.close()


def test_static_rejects_what_does_not_fit(gpu):
    n, F = factored("grid40", "MinPlus", np.float64)
    try:
        k = SCRATCH // (8 * n) + 8  # the right-hand sides alone exceed the static scratch
        B = on_device(sources(n, k, "MinPlus", np.float64))
        before = B.clone()
        with pytest.raises(pp.PPError) as e:
            F.lmul_static(B)
        assert e.value.code == _lib.PP_EINVAL and "static scratch" in str(e.value)
        assert bool((B == before).all()), "a rejected call changed B"
        # a host pointer is rejected before any device work
        H = np.asfortranarray(sources(n, 4, "MinPlus", np.float64))
        rc = _lib.lib().pp_lmul_static(F._h, _lib.vptr(H), n, 4)
        assert rc == _lib.PP_EINVAL
        # the handle still works through both entry points
        small = on_device(sources(n, 8, "MinPlus", np.float64))
        ref = small.clone()
        F.lmul_static(small)
        F._solve(ref, True)
        same(small.cpu().numpy(), ref.cpu().numpy(), "MinPlus", np.float64, "after rejections")
    finally:
        F.close()


def test_static_needs_a_factorization(gpu):
    rc = _lib.lib().pp_lmul_static(None, None, 1, 1)
    assert rc == _lib.PP_EINVAL
