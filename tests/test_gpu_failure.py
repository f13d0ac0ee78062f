"""Failure paths of the library on the GPU, provoked without faulting anything.

  - A bounded device wait that runs out: the handle's wait timeout (pp_options.wait_timeout_us) set to 1 us,
    so that the persistent kernels' waits on other blocks (every factorization and solve of a tree this size
    has waits of tens of microseconds) give up.  The kernels return early, the next call that waits for the
    stream reports PP_ETIMEOUT, and with the default timeout back the same handle factors and solves exactly
    as the oracle does.
  - Device memory running out: pp_options.fail_alloc_after makes the k-th device allocation of the handle fail
    as if the device were out of memory (a host-side fake of cudaMalloc's answer).  For every k the call that
    meets it returns PP_ENOMEM, the handle then completes the whole sequence once the hook is off, with the
    oracle's results, and device memory does not grow over the cycles.
"""
import numpy as np
import pytest

import pathpack_b200 as pp
from oracle.oracle import OracleLU
from pathpack_b200 import graphs
from pathpack_b200._lib import PP_ENOMEM, PP_ETIMEOUT
from tests.helpers import same

pytestmark = pytest.mark.gpu


def grid(a=128, seed=5):
    n, I, J, W = graphs.grid2d(a, a, 1.0, 10.0, seed=seed, dtype=np.float64)
    cp, rv, nz = graphs.csc(n, I, J, W)
    return n, cp, rv, nz, pp.ssymbolic(n, cp, rv)


def test_wait_timeout_reports_and_recovers(gpu):
    import torch

    n, cp, rv, nz, S = grid()
    O = OracleLU("MinPlus", np.float64, S).assemble(cp, rv, nz).factor()
    B, _ = graphs.unit_columns(n, 64, seed=3)
    F = pp.B200SLU(pp.MinPlus(), np.float64, S, device=0, wait_timeout_us=1)
    try:
        assert F.options()["wait_timeout_us"] == 1
        F.assemble_csc(cp, rv, nz)
        with pytest.raises(pp.PPError) as e:
            F.factor()  # enqueues, then waits: the expired wait is reported here
        assert e.value.code == PP_ETIMEOUT
        # a solve whose waits run out, on device memory: reported by the next wait for the stream
        F.set_options(wait_timeout_us=0)
        F.factor()
        F.set_options(wait_timeout_us=1)
        Bd = torch.from_numpy(np.ascontiguousarray(B.T)).to("cuda:0").T
        with pytest.raises(pp.PPError) as e:
            pp.lmul_(F, Bd)
        assert e.value.code == PP_ETIMEOUT
        # the default bound again: the same handle gives the oracle's factor and solves
        F.set_options(wait_timeout_us=0)
        assert F.options()["wait_timeout_us"] == 0
        F.update_values(nz).factor()
        for got, want, what in zip(F.factors(), (O.LD, O.LL, O.UD, O.UL), ("LD", "LL", "UD", "UL")):
            same(got, want, "MinPlus", np.float64, "after a timeout: " + what)
        same(pp.lmul_(F, B.copy(order="F")), O.lmul(B), "MinPlus", np.float64, "lmul! after a timeout")
    finally:
        F.close()


def run_sequence(F, cp, rv, nz, B, R):
    F.assemble_csc(cp, rv, nz).factor()
    X = pp.lmul_(F, B.copy(order="F"))
    Y = pp.rmul_(R.copy(order="F"), F)
    C = F.star(100, 300)
    return X, Y, C


def test_out_of_memory_at_every_allocation(gpu):
    import torch

    n, cp, rv, nz, S = grid(48, seed=6)
    O = OracleLU("MinPlus", np.float64, S).assemble(cp, rv, nz).factor()
    B, _ = graphs.unit_columns(n, 40, seed=4)
    R = np.asfortranarray(graphs.unit_columns(n, 24, seed=5)[0].T)
    E = np.full((n, 300), np.inf)
    E[np.arange(100, 400), np.arange(300)] = 0.0
    want = (O.lmul(B), O.rmul(R), O.lmul(E))
    names = ("lmul!", "rmul!", "star columns")
    # a first full run loads every kernel the sequence uses, so that later memory readings compare like with like
    F = pp.B200SLU(pp.MinPlus(), np.float64, S, device=0)
    run_sequence(F, cp, rv, nz, B, R)
    F.close()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(0)[0]
    failures = 0
    for k in range(200):
        try:
            F = pp.B200SLU(pp.MinPlus(), np.float64, S, device=0, fail_alloc_after=k)
        except pp.PPError as e:  # the structure upload met the failing allocation
            assert e.code == PP_ENOMEM, e
            failures += 1
            continue
        try:
            try:
                got = run_sequence(F, cp, rv, nz, B, R)
                hit = False
            except pp.PPError as e:
                assert e.code == PP_ENOMEM, "allocation %d: %s" % (k, e)
                hit = True
                failures += 1
                F.set_options(fail_alloc_after=-1)
                got = run_sequence(F, cp, rv, nz, B, R)  # the same handle finishes the sequence
            for g, w, what in zip(got, want, names):
                same(g, w, "MinPlus", np.float64, "allocation %d: %s" % (k, what))
        finally:
            F.close()
        if not hit:
            break  # the whole sequence needs fewer than k + 1 allocations
    else:
        raise AssertionError("the sequence still failed after 200 allocations")
    assert failures == k, (failures, k)
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info(0)[0]
    assert free1 >= free0 - (64 << 20), "device memory grew by %d bytes over %d cycles" % (free0 - free1, k)
