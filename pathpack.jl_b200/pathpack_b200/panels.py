"""Several GPUs: the split factorization's group, and the column panels of a star or a multi-right-hand-side
solve.

join_group makes every rank's factor (its own handle on its own GPU) a member of one NCCL group
(pp_comm_init): the factorization is then split across the ranks and every rank ends with the whole factor.
Each rank then computes a contiguous block of columns of A* (pp_star with col0 / ncols) or of A* B; the panels
are independent, so no collective runs on the solve's data path.  The only other exchange is the optional
gather of the panels to one rank (host memory; `torch.distributed.gather` over gloo, or over NCCL with device
tensors).  This is the reference's row-block split of the multi-GPU APSP (ext/PATHPACKCUDAExt/
multigpu.jl:254-258) in column form, which is lmul!'s natural layout.
"""
import numpy as np


def share_comm_id(group=None):
    """A group id made on rank 0 (pp_comm_id) and sent to every rank with torch.distributed (any backend)."""
    import torch.distributed as dist

    obj = [None]
    if dist.get_rank(group) == 0:
        from .api import comm_id

        obj[0] = comm_id()
    dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]


def join_group(F, group=None):
    """Join F (a B200SLU on this rank's GPU) to the NCCL group of all ranks of `group` (pp_comm_init)."""
    import torch.distributed as dist

    world, rank = dist.get_world_size(group), dist.get_rank(group)
    return F.join(share_comm_id(group) if world > 1 else None, world, rank)


def column_panels(n, world):
    """[(col0, ncols)] for ranks 0 .. world-1: contiguous, sizes differing by at most one, in rank order."""
    if world < 1:
        raise ValueError("world must be positive")
    base, extra = divmod(int(n), int(world))
    out, c = [], 0
    for r in range(world):
        w = base + (1 if r < extra else 0)
        out.append((c, w))
        c += w
    return out


def star_panel(F, rank, world, out=None):
    """(col0, C): this rank's columns of A* in original labels, computed on the rank's own GPU (pp_star)."""
    col0, ncols = column_panels(F.S.n, world)[rank]
    return col0, F.star(col0, ncols, out=out)


def lmul_panel(F, B, rank, world):
    """(col0, X): this rank's columns of A* B (B is n x k, host or device, column-major); X = A* B[:, panel]
    solved on the rank's GPU (pp_lmul).  The other columns are untouched."""
    col0, w = column_panels(B.shape[1], world)[rank]
    X = B[:, col0:col0 + w]
    if not hasattr(X, "data_ptr"):
        X = np.asfortranarray(X)
    from .api import lmul_

    return col0, lmul_(F, X)


def gather_columns(panel, col0, n_cols, dst=0, group=None):
    """Gather every rank's column panel (n x w, numpy or torch) into an n x n_cols array on rank `dst` (None
    elsewhere), with torch.distributed (gloo for host tensors, NCCL for device tensors).  Panels may differ in
    width by the balanced split of `column_panels`; they are padded to the widest for the collective."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    spans = column_panels(n_cols, world)
    if spans[rank][0] != col0 or spans[rank][1] != panel.shape[1]:
        raise ValueError("panel (%d, %d) is not rank %d's span %s" % (col0, panel.shape[1], rank, spans[rank]))
    t = panel if isinstance(panel, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(panel))
    n, wmax = t.shape[0], max(w for _, w in spans)
    # (width, n) row-major is the column-major n x width panel
    send = torch.zeros((wmax, n), dtype=t.dtype, device=t.device)
    send[:t.shape[1]] = t.t()
    bufs = [torch.empty_like(send) for _ in range(world)] if rank == dst else None
    dist.gather(send, bufs, dst=dst, group=group)
    if rank != dst:
        return None
    full = torch.empty((n_cols, n), dtype=t.dtype, device=t.device)
    for r, (c0, w) in enumerate(spans):
        full[c0:c0 + w] = bufs[r][:w]
    out = full.t()
    return out.cpu().numpy() if not isinstance(panel, torch.Tensor) else out
