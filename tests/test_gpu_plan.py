"""Plan reuse on the GPU: refactorization with new weights on the same pattern, through the C ABI.

  - pp_update_values (host and device weights) then pp_factor, against the oracle run on the new weights;
  - pp_set_values with the oracle's factor arrays, then lmul!/rmul!, against the oracle's solves;
  - pp_plan_lmul / pp_plan_launch: the step (re-assembly, factorization, lmul!) captured once as a CUDA graph
    and replayed with new weights written into its device buffer, against the oracle for each set of weights.
Bit for bit for the idempotent semirings, rtol 1e-5 / 1e-12 for PlusProd.
"""
import numpy as np
import pytest

import pathpack_b200 as pp
from oracle.oracle import OracleLU
from tests.helpers import close, graph, same, weights

pytestmark = pytest.mark.gpu

SR = {s.__class__.__name__: s for s in [pp.MinPlus(), pp.MaxPlus(), pp.MaxMin(), pp.MinMax(), pp.MaxProd(),
                                         pp.PlusProd(), pp.OrAnd()]}
CASES = [("MinPlus", np.float64), ("MinPlus", np.float32), ("MaxMin", np.float32), ("PlusProd", np.float64),
         ("OrAnd", np.int32), ("MinPlus", np.int32), ("MaxPlus", np.float64)]


def torch_dt(dtype):
    import torch

    return {np.dtype(np.float32): torch.float32, np.dtype(np.float64): torch.float64,
            np.dtype(np.int32): torch.int32}[np.dtype(dtype)]


def sources(n, k, name, dtype, seed):
    rng = np.random.default_rng(seed)
    z, one = SR[name].zero(dtype), SR[name].one(dtype)
    B = np.full((n, k), z, dtype=dtype, order="F")
    B[rng.choice(n, size=k, replace=False), np.arange(k)] = one
    B[rng.random(B.shape) < 0.03] = one
    return B


def dev_colmajor(B):
    import torch

    return torch.from_numpy(np.ascontiguousarray(B.T)).to("cuda:0").T


@pytest.mark.parametrize("name,dtype", CASES)
@pytest.mark.parametrize("kind", ["grid40", "knn"])
def test_refactor_with_new_weights(gpu, name, dtype, kind):
    import torch

    n, cp, rv, nz = graph(kind, name, dtype, seed=1)
    S = pp.ssymbolic(n, cp, rv)
    F = pp.B200SLU(SR[name], dtype, S, device=0).assemble_csc(cp, rv, nz).factor()
    try:
        for it, where in enumerate(["host", "device", "host"]):
            nz2 = weights(name, dtype, len(nz), 100 + it)  # new weights, same pattern
            F.update_values(nz2 if where == "host" else torch.from_numpy(nz2).to("cuda:0")).factor()
            O = OracleLU(name, dtype, S).assemble(cp, rv, nz2).factor()
            for got, want, what in zip(F.factors(), (O.LD, O.LL, O.UD, O.UL), ("LD", "LL", "UD", "UL")):
                same(got, want, name, dtype, "%s refactor %d (%s) %s" % (kind, it, where, what))
            B = sources(n, 21, name, dtype, it)
            same(pp.lmul_(F, B.copy(order="F")), O.lmul(B), name, dtype, "%s refactor %d lmul" % (kind, it))
    finally:
        F.close()


@pytest.mark.parametrize("name,dtype", CASES)
def test_set_values_from_the_oracle(gpu, name, dtype):
    """Factor arrays assembled on the host (the reference keeps copyto! on the host; here the oracle's
    assembly) uploaded with pp_set_values, then pp_factor: the factor and the solves are the oracle's."""
    n, cp, rv, nz = graph("knn", name, dtype, seed=2)
    S = pp.ssymbolic(n, cp, rv)
    A = OracleLU(name, dtype, S).assemble(cp, rv, nz)  # assembled, not factored
    F = pp.B200SLU(SR[name], dtype, S, device=0)
    try:
        F.set_values(A.LD, A.LL, A.UD, A.UL, A.Nval)
        for got, want in zip(F.factors(), (A.LD, A.LL, A.UD, A.UL)):
            same(got, want, name, dtype, "set_values round trip")
        F.factor()
        O = A.factor()
        for got, want, what in zip(F.factors(), (O.LD, O.LL, O.UD, O.UL), ("LD", "LL", "UD", "UL")):
            same(got, want, name, dtype, "factor of uploaded values " + what)
        B = sources(n, 17, name, dtype, 4)
        same(pp.lmul_(F, B.copy(order="F")), O.lmul(B), name, dtype, "lmul after set_values")
        R = np.asfortranarray(B.T)
        same(pp.rmul_(R.copy(order="F"), F), O.rmul(R), name, dtype, "rmul after set_values")
    finally:
        F.close()


@pytest.mark.parametrize("name,dtype", CASES)
@pytest.mark.parametrize("inplace", [False, True])
def test_plan_replay(gpu, name, dtype, inplace):
    import torch

    n, cp, rv, nz = graph("grid40", name, dtype, seed=3)
    S = pp.ssymbolic(n, cp, rv)
    F = pp.B200SLU(SR[name], dtype, S, device=0).assemble_csc(cp, rv, nz)
    try:
        k = 40
        B = sources(n, k, name, dtype, 9)
        nz_d = torch.from_numpy(nz.copy()).to("cuda:0")
        Bin = dev_colmajor(B)
        Bout = Bin if inplace else torch.empty_like(Bin.T).T
        plan = F.plan_lmul(nz_d, Bin, Bout)
        assert plan.launches > 10
        stream = torch.cuda.ExternalStream(F.stream(), device=0)
        try:
            for it in range(3):
                nz2 = weights(name, dtype, len(nz), 200 + it)
                with torch.cuda.stream(stream):
                    nz_d.copy_(torch.from_numpy(nz2).to("cuda:0"))
                    if inplace:
                        Bin.copy_(dev_colmajor(B))
                plan.launch()
                F.sync()
                O = OracleLU(name, dtype, S).assemble(cp, rv, nz2).factor()
                same(Bout.cpu().numpy(), O.lmul(B), name, dtype, "plan step %d" % it)
                for got, want, what in zip(F.factors(), (O.LD, O.LL, O.UD, O.UL), ("LD", "LL", "UD", "UL")):
                    same(got, want, name, dtype, "plan step %d %s" % (it, what))
            # the handle's ordinary calls still work after replays
            R = np.asfortranarray(sources(n, 7, name, dtype, 5).T)
            same(pp.rmul_(R.copy(order="F"), F), O.rmul(R), name, dtype, "rmul after the plan")
        finally:
            plan.close()
    finally:
        F.close()


def test_plan_rejects_host_memory(gpu):
    import torch

    n, cp, rv, nz = graph("grid", "MinPlus", np.float64, seed=3)
    S = pp.ssymbolic(n, cp, rv)
    F = pp.B200SLU(pp.MinPlus(), np.float64, S, device=0).assemble_csc(cp, rv, nz)
    try:
        import ctypes as C

        B = torch.full((4, n), np.inf, dtype=torch.float64).T  # host tensor
        with pytest.raises(TypeError):  # the Python layer refuses it first
            F.plan_lmul(torch.from_numpy(nz).to("cuda:0"), B)
        # and the C ABI itself, given the host pointer
        nz_d = torch.from_numpy(nz).to("cuda:0")
        p = C.c_void_p()
        L = pp.lib()
        r = L.pp_plan_lmul(F._h, C.c_void_p(nz_d.data_ptr()), C.c_void_p(B.data_ptr()), C.c_void_p(B.data_ptr()),
                           n, 4, C.byref(p))
        assert r == pp._lib.PP_EINVAL and not p.value
        assert b"memory of the handle's device" in L.pp_last_error(F._h)
    finally:
        F.close()
