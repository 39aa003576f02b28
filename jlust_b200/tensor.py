"""USTensor: the buffers-plus-format container of JLUST (src/tensor.jl:29-43).

Buffers are torch tensors (device memory on a CUDA device for every op of
the backend).  Level numbering of positions()/coordinates() is 1-based, as in
the reference (src/tensor.jl:91-107): a CSR matrix keeps its row pointer in
positions(u, 2) and its column indices in coordinates(u, 2).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from .errors import IncompatibleExtents, InvalidLevelAccess, UnsupportedIndexType
from .formats import Formats, TensorFormat


class OneBased:
    offset = 1

    def __eq__(self, o):
        return isinstance(o, OneBased)

    def __hash__(self):
        return 1

    def __repr__(self):
        return "OneBased()"


class ZeroBased:
    offset = 0

    def __eq__(self, o):
        return isinstance(o, ZeroBased)

    def __hash__(self):
        return 0

    def __repr__(self):
        return "ZeroBased()"


def _origin(o):
    if isinstance(o, (OneBased, ZeroBased)):
        return o
    if o in (0, 1):
        return OneBased() if o == 1 else ZeroBased()
    raise ValueError(f"index origin must be OneBased(), ZeroBased(), 0 or 1, got {o!r}")


@dataclass
class USTensor:
    extents: tuple
    format: TensorFormat
    pos: tuple              # per level: tensor or None
    crd: tuple              # per level: tensor or None
    val: torch.Tensor
    origin: object = field(default_factory=OneBased)
    owner: object = None    # keeps a wrapped source alive (src/tensor.jl:42)

    @property
    def shape(self):
        return self.extents

    @property
    def dtype(self):
        return self.val.dtype

    @property
    def device(self):
        return self.val.device

    def __repr__(self):
        return (f"USTensor({self.format.name}, extents={self.extents}, nnz={nnz(self)}, "
                f"dtype={self.val.dtype}, origin={self.origin}, device={self.val.device})")


def positions(u: USTensor, level: int) -> torch.Tensor:
    if not 1 <= level <= len(u.pos):
        raise InvalidLevelAccess(f"level {level} out of range")
    p = u.pos[level - 1]
    if p is None:
        raise InvalidLevelAccess(f"level {level} has no position buffer")
    return p


def coordinates(u: USTensor, level: int) -> torch.Tensor:
    if not 1 <= level <= len(u.crd):
        raise InvalidLevelAccess(f"level {level} out of range")
    c = u.crd[level - 1]
    if c is None:
        raise InvalidLevelAccess(f"level {level} has no coordinate buffer")
    return c


def has_positions(u, level):
    return 1 <= level <= len(u.pos) and u.pos[level - 1] is not None


def has_coordinates(u, level):
    return 1 <= level <= len(u.crd) and u.crd[level - 1] is not None


def nonzeros(u: USTensor) -> torch.Tensor:
    return u.val


def nnz(u: USTensor) -> int:
    """Stored values (src/tensor.jl:111); for BSR this counts tile entries."""
    return int(u.val.numel())


def format(u: USTensor) -> TensorFormat:  # noqa: A001 - mirrors JLUST's name
    return u.format


def extents(u: USTensor) -> tuple:
    return u.extents


def index_origin(u: USTensor):
    return u.origin


def _idx(t: torch.Tensor, what: str) -> torch.Tensor:
    if t.dtype != torch.int32:
        raise UnsupportedIndexType(f"{what}: index buffers must be Int32 (got {t.dtype})")
    if t.dim() != 1 or not t.is_contiguous():
        raise IncompatibleExtents(f"{what}: index buffers must be contiguous vectors")
    return t


def csr_tensor(rowptr, colind, nzval, dims, origin=None) -> USTensor:
    """CSR from buffers (src/interop.jl:57-67); buffers are not copied."""
    origin = _origin(OneBased() if origin is None else origin)
    m, n = dims
    _idx(rowptr, "csr_tensor rowptr")
    _idx(colind, "csr_tensor colind")
    if rowptr.numel() != m + 1:
        raise IncompatibleExtents(f"csr_tensor: rowptr has {rowptr.numel()} entries, need {m + 1}")
    if colind.numel() != nzval.numel():
        raise IncompatibleExtents("csr_tensor: colind and nzval lengths differ")
    return USTensor((int(m), int(n)), Formats.CSR, (None, rowptr), (None, colind), nzval, origin)


def shifted_diag_tensor(dtype, n_rows, n_cols, shift=0, val=1.0, device="cpu") -> USTensor:
    """A structural shifted scaled identity (src/interop.jl:155-181): row r
    has one entry, `val` at column r + shift, with no position, coordinate or
    value buffers (the value lives in the format)."""
    from .formats import Formats
    return USTensor((int(n_rows), int(n_cols)), Formats.ShiftedDiag(shift, val), (None, None),
                    (None, None), torch.empty(0, dtype=dtype, device=device), OneBased())


def coo_tensor(rows, cols, nzval, dims, origin=None) -> USTensor:
    """COO from buffers (src/interop.jl:248-260)."""
    origin = _origin(OneBased() if origin is None else origin)
    _idx(rows, "coo_tensor rows")
    _idx(cols, "coo_tensor cols")
    if not rows.numel() == cols.numel() == nzval.numel():
        raise IncompatibleExtents("coo_tensor: rows, cols and nzval lengths differ")
    return USTensor((int(dims[0]), int(dims[1])), Formats.COO, (None, None), (rows, cols), nzval,
                    origin)


def bsr_tensor(browptr, bcolind, bval, dims, blocksize, origin=None) -> USTensor:
    """BSRRight((b1, b2)) from buffers: block row pointer at level 2, block
    columns at level 2, values as nnzb row-major b1 x b2 tiles (the layout of
    ust(::CuSparseMatrixBSR), ext/CUDAExt/CUDAExt.jl:144-156)."""
    origin = _origin(OneBased() if origin is None else origin)
    b1, b2 = blocksize
    m, n = dims
    _idx(browptr, "bsr_tensor browptr")
    _idx(bcolind, "bsr_tensor bcolind")
    mb = -(-m // b1)
    if browptr.numel() != mb + 1:
        raise IncompatibleExtents(f"bsr_tensor: browptr has {browptr.numel()} entries, need {mb + 1}")
    if bval.numel() != bcolind.numel() * b1 * b2:
        raise IncompatibleExtents("bsr_tensor: bval must hold nnzb * b1 * b2 values")
    return USTensor((int(m), int(n)), Formats.BSRRight((b1, b2)), (None, browptr, None, None),
                    (None, bcolind, None, None), bval, origin)


def dense_layout(t: torch.Tensor):
    """(order, leading dimension) of a 1-D or 2-D strided tensor, or None when
    neither row- nor column-major."""
    if t.dim() == 1:
        return (0, max(t.numel(), 1)) if t.stride(0) == 1 or t.numel() <= 1 else None
    if t.dim() != 2:
        return None
    r, c = t.shape
    s0, s1 = t.stride()
    if (s1 == 1 or c <= 1) and s0 >= max(c, 1):
        return (0, s0 if r > 1 else max(c, 1))
    if (s0 == 1 or r <= 1) and s1 >= max(r, 1):
        return (1, s1 if c > 1 else max(r, 1))
    return None


def ust(a) -> USTensor:
    """Zero-copy dense USTensor of a torch tensor (src/interop.jl:36-46).
    A transposed view keeps its memory and is read column-major."""
    if isinstance(a, USTensor):
        return a
    if not isinstance(a, torch.Tensor):
        raise TypeError("ust: expected a torch.Tensor")
    nd = a.dim()
    return USTensor(tuple(a.shape), Formats.DensedRight(nd), (None,) * nd, (None,) * nd, a,
                    OneBased(), owner=a)
