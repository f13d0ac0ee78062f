"""The split factorization on two GPUs (pp_comm_init): each rank factors its part of the bottom of the tree,
NCCL broadcasts give every rank the other parts, and every rank factors the top.  Each rank's whole factor must
equal the oracle's (bit for bit for the idempotent semirings), and each rank's column panel of lmul! / the star
the oracle's columns.  Cases: the config-2 grid in Float64 MinPlus, the coupled kNN graph (several strongly
connected components) in Float32 MinPlus, a 3D grid in Float32 MaxMin (merged top fronts), and a
refactorization with new weights.  Runs only where two GPUs are visible (gpurun --gpus 2); NVLS is off.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _case(name):
    from pathpack_b200 import graphs

    if name == "grid":
        return "MinPlus", np.float64, graphs.grid2d(128, 128, 1.0, 10.0, seed=31, dtype=np.float64)
    if name == "knn":
        return "MinPlus", np.float32, graphs.knn_directed(6000, 6, seed=32, dtype=np.float32)
    return "MaxMin", np.float32, graphs.grid3d(20, 20, 20, seed=33, dtype=np.float32)


def _worker(rank, world, port, case, errq):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        import pathpack_b200 as pp
        from oracle.oracle import OracleLU
        from pathpack_b200 import graphs
        from pathpack_b200.panels import column_panels, join_group
        from tests.helpers import same, weights

        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
        name, dtype, (n, I, J, W) = _case(case)
        cp, rv, nz = graphs.csc(n, I, J, W)
        S = pp.ssymbolic(n, cp, rv)
        s = getattr(pp, name)()
        F = pp.B200SLU(s, dtype, S, device=rank)
        try:
            join_group(F)
            F.assemble_csc(cp, rv, nz).factor()
            O = OracleLU(name, dtype, S).assemble(cp, rv, nz).factor(4)
            for got, want, what in zip(F.factors(), (O.LD, O.LL, O.UD, O.UL), ("LD", "LL", "UD", "UL")):
                same(got, want, name, dtype, "rank %d %s %s" % (rank, case, what))
            B, _ = graphs.unit_columns(n, 64, seed=5, dtype=dtype, zero=s.zero(dtype), one=s.one(dtype))
            c0, kw = column_panels(64, world)[rank]
            want = O.lmul(B)[:, c0:c0 + kw]
            X = pp.lmul_(F, np.array(B[:, c0:c0 + kw], order="F"))  # a copy: lmul! works in place
            same(X, want, name, dtype, "rank %d %s lmul! panel" % (rank, case))
            col0, ncols = column_panels(n, world)[rank]
            ncols = min(ncols, 96)
            E = np.full((n, ncols), s.zero(dtype), dtype=dtype, order="F")
            E[np.arange(col0, col0 + ncols), np.arange(ncols)] = s.one(dtype)
            same(F.star(col0, ncols), O.lmul(E), name, dtype, "rank %d %s star panel" % (rank, case))
            if case == "grid":  # refactorization with new weights, twice (the collective runs every time)
                for it in range(2):
                    nz2 = weights(name, dtype, len(nz), 70 + it)
                    F.update_values(nz2).factor()
                    O2 = OracleLU(name, dtype, S).assemble(cp, rv, nz2).factor(4)
                    for got, want, what in zip(F.factors(), (O2.LD, O2.LL, O2.UD, O2.UL), ("LD", "LL", "UD", "UL")):
                        same(got, want, name, dtype, "rank %d refactor %d %s" % (rank, it, what))
            dist.barrier()
        finally:
            F.close()
            dist.destroy_process_group()
    except BaseException as e:  # noqa: BLE001
        errq.put("rank %d: %r" % (rank, e))
        raise


@pytest.mark.parametrize("case", ["grid", "knn", "grid3d"])
def test_split_factorization_two_gpus(gpu, case):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, case, errq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    for p in procs:
        if p.is_alive():
            p.kill()
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs and all(p.exitcode == 0 for p in procs), errs


def test_multi_device_handle(gpu):
    """pp_multi (one process driving the GPUs it is given, one host thread per device): factor, lmul!, rmul!
    (and their transposes) and star columns split by device, against the oracle.  On one GPU it is a group of
    one; with two it runs the split factorization."""
    import torch

    import pathpack_b200 as pp
    from oracle.oracle import OracleLU
    from pathpack_b200 import graphs
    from tests.helpers import same

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    devices = list(range(min(2, torch.cuda.device_count())))
    n, I, J, W = graphs.grid2d(96, 96, 1.0, 10.0, seed=41, dtype=np.float64)
    cp, rv, nz = graphs.csc(n, I, J, W)
    S = pp.ssymbolic(n, cp, rv)
    O = OracleLU("MinPlus", np.float64, S).assemble(cp, rv, nz).factor()
    M = pp.MultiSLU(pp.MinPlus(), np.float64, S, devices)
    try:
        M.assemble_csc(cp, rv, nz).factor()
        B, _ = graphs.unit_columns(n, 37, seed=2)
        same(M.lmul_(B.copy(order="F")), O.lmul(B), "MinPlus", np.float64, "multi lmul!")
        R = np.asfortranarray(graphs.unit_columns(n, 23, seed=3)[0].T)
        same(M.rmul_(R.copy(order="F")), O.rmul(R), "MinPlus", np.float64, "multi rmul!")
        E = np.full((n, 300), np.inf, order="F")
        E[np.arange(1000, 1300), np.arange(300)] = 0.0
        same(M.star(1000, 300), O.lmul(E), "MinPlus", np.float64, "multi star columns")
        # the transposed factor: lmul!(transpose(F), B) = (rmul!(B^T, F))^T
        Bt = M.lmul_(B.copy(order="F"), trans=True)
        same(Bt, np.asfortranarray(O.rmul(np.asfortranarray(B.T)).T), "MinPlus", np.float64, "multi lmul! transposed")
    finally:
        M.close()
