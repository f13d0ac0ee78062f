"""The semirings of PATHPACK.jl (src/CPU/semiring/*.jl) as descriptors of the C ABI.

Each class names a semiring the way the reference does (`MinPlus()`, `MaxMin()`, ...) and carries its
identifier, its zero and one per element type, and which element types the B200 library takes
(check_semiring, ext/PATHPACKCUDAExt/runtime/config.jl:359-377, is pp_check_semiring).
"""
import numpy as np

PP_F32, PP_F64, PP_I32 = 0, 1, 2
DTYPES = {np.dtype(np.float32): PP_F32, np.dtype(np.float64): PP_F64, np.dtype(np.int32): PP_I32}
I32MAX = np.iinfo(np.int32).max


class AbstractSemiring:
    id = -1
    integral = False

    def zero(self, dtype):
        raise NotImplementedError

    def one(self, dtype):
        raise NotImplementedError

    def __repr__(self):
        return type(self).__name__ + "()"

    def __eq__(self, other):
        return type(self) is type(other)

    def __hash__(self):
        return hash(type(self).__name__)


class MinPlus(AbstractSemiring):
    """([-inf, inf], min, +): shortest paths.  zero inf, one 0.  Int32: weights in [0, typemax], saturating."""
    id = 0

    def zero(self, dtype):
        return np.dtype(dtype).type(I32MAX if np.dtype(dtype) == np.int32 else np.inf)

    def one(self, dtype):
        return np.dtype(dtype).type(0)


class MaxPlus(AbstractSemiring):
    """([-inf, inf], max, +): longest paths.  zero -inf, one 0."""
    id = 1

    def zero(self, dtype):
        return np.dtype(dtype).type(-np.inf)

    def one(self, dtype):
        return np.dtype(dtype).type(0)


class MaxMin(AbstractSemiring):
    """([-inf, inf], max, min): widest paths.  zero -inf, one inf."""
    id = 2
    integral = True

    def zero(self, dtype):
        return np.dtype(dtype).type(-np.inf)

    def one(self, dtype):
        return np.dtype(dtype).type(np.inf)


class MinMax(AbstractSemiring):
    """([-inf, inf], min, max): bottleneck paths.  zero inf, one -inf."""
    id = 3
    integral = True

    def zero(self, dtype):
        return np.dtype(dtype).type(np.inf)

    def one(self, dtype):
        return np.dtype(dtype).type(-np.inf)


class MaxProd(AbstractSemiring):
    """([0, inf], max, *): most reliable paths.  zero 0, one 1."""
    id = 4

    def zero(self, dtype):
        return np.dtype(dtype).type(0)

    def one(self, dtype):
        return np.dtype(dtype).type(1)


class PlusProd(AbstractSemiring):
    """([0, inf], +, *): walk sums, (I - A)^-1.  zero 0, one 1."""
    id = 5

    def zero(self, dtype):
        return np.dtype(dtype).type(0)

    def one(self, dtype):
        return np.dtype(dtype).type(1)


class OrAnd(AbstractSemiring):
    """(2^n, |, &) on Int32 bit sets: labels carried by some path.  zero 0, one typemax(Int32)."""
    id = 6
    integral = True

    def zero(self, dtype):
        return np.int32(0)

    def one(self, dtype):
        return np.int32(I32MAX)


ALL = [MinPlus(), MaxPlus(), MaxMin(), MinMax(), MaxProd(), PlusProd(), OrAnd()]
BY_ID = {s.id: s for s in ALL}


def supported(s, dtype):
    """Whether the B200 library takes the semiring over the element type (as pp_check_semiring)."""
    d = DTYPES.get(np.dtype(dtype))
    if d is None:
        return False
    if isinstance(s, OrAnd):
        return d == PP_I32
    if d == PP_I32:
        return isinstance(s, MinPlus)
    return True
