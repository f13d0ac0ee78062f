"""The multi-rank host logic on the CPU: column panels of one star shared by ranks and gathered over gloo
(world size 2 and 3), with the oracle standing in for each rank's GPU panel computation."""
import os
import socket

import numpy as np
import pytest

from pathpack_b200.panels import column_panels


def test_column_panels_partition():
    for n in (1, 7, 64, 4096, 65536):
        for world in (1, 2, 3, 4, 8):
            p = column_panels(n, world)
            assert len(p) == world and p[0][0] == 0
            assert sum(w for _, w in p) == n
            assert all(p[r][0] + p[r][1] == p[r + 1][0] for r in range(world - 1))
            ws = [w for _, w in p]
            assert max(ws) - min(ws) <= 1
    with pytest.raises(ValueError):
        column_panels(5, 0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, name, dtype_str):
    import datetime

    import torch.distributed as dist

    import pathpack_b200 as pp
    from oracle.oracle import OracleLU
    from pathpack_b200.panels import gather_columns
    from tests.helpers import close, graph, same

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        dtype = np.dtype(dtype_str)
        n, cp, rv, nz = graph("sprand", name, dtype)
        S = pp.ssymbolic(n, cp, rv)
        O = OracleLU(name, dtype, S).assemble(cp, rv, nz).factor()
        col0, w = column_panels(n, world)[rank]
        # this rank's columns of A* in original labels: lmul! of the unit columns col0 .. col0 + w - 1
        s = pp.MinPlus() if name == "MinPlus" else pp.MaxMin()
        E = np.full((n, w), s.zero(dtype), dtype=dtype, order="F")
        E[np.arange(col0, col0 + w), np.arange(w)] = s.one(dtype)
        panel = O.lmul(E)
        full = gather_columns(panel, col0, n, dst=0)
        if rank == 0:
            I = np.full((n, n), s.zero(dtype), dtype=dtype, order="F")
            np.fill_diagonal(I, s.one(dtype))
            assert full.shape == (n, n)
            same(full, O.lmul(I), name, dtype, "gathered star panels")  # bit for bit: same dataflow
            close(full, O.star(), name, dtype, "gathered star panels vs the oracle's star")
        else:
            assert full is None
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("name,dtype", [("MinPlus", "float64"), ("MaxMin", "float32")])
def test_star_panels_gathered_over_gloo(world, name, dtype):
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(world, _free_port(), name, dtype), nprocs=world, join=True)


def _id_worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    from pathpack_b200.panels import share_comm_id

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        q.put((rank, share_comm_id()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_group_id_reaches_every_rank_over_gloo(world):
    """The id of the split factorization's NCCL group (pp_comm_id, made on rank 0) reaches every rank intact."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.start_processes(_id_worker, args=(world, _free_port(), q), nprocs=world, join=True, start_method="spawn")
    got = dict(q.get() for _ in range(world))
    assert sorted(got) == list(range(world))
    assert all(len(v) == 128 and v == got[0] for v in got.values())
    assert any(got[0])
