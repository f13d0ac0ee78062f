"""pathpack_b200 — the host side of the B200 backend for PATHPACK.jl's numeric hot path.

The numeric work is in libpathpack_b200.so (hand-written sm_100a CUDA behind the C ABI of
include/pathpack_b200.h); this package mirrors the reference's user API (mlu, mstar, lu!, lmul!, rmul!,
Matrix) and its semirings on top of it.  Import it with pathpack.jl_b200/ on sys.path.
"""
from .semiring import MinPlus, MaxPlus, MaxMin, MinMax, MaxProd, PlusProd, OrAnd, supported  # noqa: F401
from .symbolic import Structure, ssymbolic  # noqa: F401
from .api import B200SLU, MultiSLU, TransposedSLU, comm_id, mlu, mstar, lu_, lmul_, rmul_, Matrix, star_cols, star_rows, transpose  # noqa: F401
from ._lib import PPError, lib  # noqa: F401
