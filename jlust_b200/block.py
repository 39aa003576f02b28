"""BlockSparseMatrix: a matrix of sparse blocks (src/block_sparse.jl:27-77)
and its products, y = A x and Y = A X.

Two paths, as in the reference:

* per block (src/block_sparse.jl:266-302): every stored block multiplies its
  slice of x into its slice of y through the backend's SpMV / SpMM (the first
  block of a block row with beta = 0, the rest with beta = 1; BlockSpMM zeroes
  Y and adds every block).  Any block format the backend supports.
* compiled (ext/CUDAExt/ops/block_mul.jl:36-288): when every stored block is
  CSR, the blocks are assembled once into one CSR of the whole matrix (on the
  host, at the first product; block (i, j)'s entries of row r land at the
  slots reserved for that row, columns shifted by the block column's offset),
  with a slot map per block.  y = A x is then that CSR's SpMV, captured in a
  CUDA graph per (y, x) buffer pair and replayed on later calls; inside a
  capture the caller started, the SpMV is launched directly instead.
  `update_block_values` copies new values into a block and, through the slot
  map, into the assembled CSR in place, so captured graphs see them.

The reference treats constant-value selector blocks through a separate patch
kernel; here such blocks are assembled like any other CSR block (this library
has no ShiftedDiag format).
"""
from __future__ import annotations

import numpy as np
import torch

from .errors import IncompatibleExtents, UnsupportedFormat
from .tensor import USTensor, coordinates, csr_tensor, nonzeros, positions, ust


class BlockSparseMatrix:
    """`BlockSparseMatrix(blocks)`: blocks is a list of block rows, each a list
    of USTensor or None; every block row and block column needs at least one
    stored block, blocks in one block row (column) share their row (column)
    count, and all blocks share one value type (src/block_sparse.jl:34-73)."""

    def __init__(self, blocks):
        blocks = [list(r) for r in blocks]
        nb_r = len(blocks)
        nb_c = len(blocks[0]) if nb_r else 0
        if nb_r == 0 or nb_c == 0 or any(len(r) != nb_c for r in blocks):
            raise ValueError("BlockSparseMatrix: blocks must be a non-empty rectangular grid")
        row_sizes, col_sizes, ref = [0] * nb_r, [0] * nb_c, None
        for i in range(nb_r):
            for j in range(nb_c):
                b = blocks[i][j]
                if b is None:
                    continue
                if not isinstance(b, USTensor):
                    raise ValueError(f"BlockSparseMatrix: block ({i + 1},{j + 1}) must be a "
                                     f"USTensor or None, got {type(b).__name__}")
                rs, cs = b.extents
                if row_sizes[i] == 0:
                    row_sizes[i] = rs
                elif row_sizes[i] != rs:
                    raise ValueError(f"BlockSparseMatrix: block row {i + 1} has inconsistent "
                                     f"sizes ({row_sizes[i]} vs {rs} at col {j + 1})")
                if col_sizes[j] == 0:
                    col_sizes[j] = cs
                elif col_sizes[j] != cs:
                    raise ValueError(f"BlockSparseMatrix: block col {j + 1} has inconsistent "
                                     f"sizes ({col_sizes[j]} vs {cs} at row {i + 1})")
                t = nonzeros(b).dtype
                if ref is None:
                    ref = t
                elif ref != t:
                    raise ValueError(f"BlockSparseMatrix: mixed element types ({ref} vs {t} "
                                     f"at block ({i + 1},{j + 1}))")
        if ref is None:
            raise ValueError("BlockSparseMatrix: all blocks are nothing")
        empty_r = [i + 1 for i, s in enumerate(row_sizes) if s == 0]
        empty_c = [j + 1 for j, s in enumerate(col_sizes) if s == 0]
        if empty_r:
            raise ValueError(f"BlockSparseMatrix: block row(s) {empty_r} are entirely nothing")
        if empty_c:
            raise ValueError(f"BlockSparseMatrix: block col(s) {empty_c} are entirely nothing")
        self.blocks = blocks
        self.row_sizes, self.col_sizes = row_sizes, col_sizes
        self.row_off = np.concatenate([[0], np.cumsum(row_sizes)]).astype(np.int64)
        self.col_off = np.concatenate([[0], np.cumsum(col_sizes)]).astype(np.int64)
        self.dtype = ref
        self._compiled = None

    @property
    def shape(self):
        return int(self.row_off[-1]), int(self.col_off[-1])

    def stored(self):
        for i, r in enumerate(self.blocks):
            for j, b in enumerate(r):
                if b is not None:
                    yield i, j, b

    def compilable(self) -> bool:
        return all(b.format.family == "CSR" for _, _, b in self.stored())


class _Compiled:
    """The assembled CSR, the per-block slot maps and the captured graphs."""

    def __init__(self, A: BlockSparseMatrix):
        m, n = A.shape
        dev = nonzeros(next(A.stored())[2]).device
        row_nnz = np.zeros(m, np.int64)
        host = {}
        for i, j, b in A.stored():
            base = b.origin.offset
            rp = positions(b, 2).cpu().numpy().astype(np.int64) - base
            ci = coordinates(b, 2).cpu().numpy().astype(np.int64) - base
            host[(i, j)] = (rp, ci)
            r0 = A.row_off[i]
            row_nnz[r0:r0 + A.row_sizes[i]] += np.diff(rp)
        rowptr = np.zeros(m + 1, np.int64)
        np.cumsum(row_nnz, out=rowptr[1:])
        if rowptr[-1] > np.iinfo(np.int32).max - 1:
            raise IncompatibleExtents("BlockSparseMatrix: assembled nnz exceeds Int32 positions")
        colind = np.zeros(int(rowptr[-1]), np.int32)
        cursor = rowptr[:-1].copy()
        maps = {}
        # blocks in (block row, block column) order, so a row's entries follow
        # its blocks left to right, each block's in its own storage order
        for (i, j), (rp, ci) in sorted(host.items()):
            r0, c0 = A.row_off[i], A.col_off[j]
            lens = np.diff(rp)
            rows = np.repeat(np.arange(A.row_sizes[i]), lens)
            within = np.arange(ci.shape[0]) - np.repeat(rp[:-1], lens)
            slots = cursor[r0 + rows] + within
            colind[slots] = (ci + c0).astype(np.int32)
            cursor[r0:r0 + A.row_sizes[i]] += lens
            maps[(i, j)] = torch.from_numpy(slots).to(dev)
        self.maps = maps
        self.val = torch.empty(int(rowptr[-1]), dtype=A.dtype, device=dev)
        for (i, j), slots in maps.items():
            self.val[slots] = nonzeros(A.blocks[i][j])
        self.csr = csr_tensor(torch.from_numpy(rowptr.astype(np.int32)).to(dev),
                              torch.from_numpy(colind).to(dev), self.val, (m, n), origin=0)
        self.graphs = {}

    def spmv(self, x, y):
        from .backend import spmv
        spmv(self.csr, x, y)

    def run(self, x, y):
        if torch.cuda.is_current_stream_capturing():
            self.spmv(x, y)          # a capture the caller started records the launch
            return
        key = (y.data_ptr(), x.data_ptr())
        g = self.graphs.get(key)
        if g is None:
            self.spmv(x, y)          # first use outside the graph, then capture
            torch.cuda.current_stream(y.device).synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.spmv(x, y)
            self.graphs[key] = g
        g.replay()


def _vec(t, what):
    t = ust(t).val
    if t.dim() != 1:
        raise IncompatibleExtents(f"BlockSpMV: {what} must be a vector")
    return t


def block_spmv(A: BlockSparseMatrix, x, y, backend=None):
    """y = A x (mul!(y, A, x), src/block_sparse.jl:266-282 and
    ext/CUDAExt/ops/block_mul.jl:231-306)."""
    from .backend import B200Backend, backend_execute
    from .ops import SpMVOp
    x, y = _vec(x, "x"), _vec(y, "y")
    m, n = A.shape
    if x.numel() != n or y.numel() != m:
        raise IncompatibleExtents(f"BlockSpMV: A is {m}x{n}, x has {x.numel()}, y has {y.numel()}")
    if A.compilable() and (backend is None or isinstance(backend, B200Backend)):
        if A._compiled is None:
            A._compiled = _Compiled(A)
        A._compiled.run(x, y)
        return y
    be = backend if backend is not None else B200Backend()
    for i, row in enumerate(A.blocks):
        ys = y[A.row_off[i]:A.row_off[i + 1]]
        first = True
        for j, b in enumerate(row):
            if b is None:
                continue
            xs = x[A.col_off[j]:A.col_off[j + 1]]
            op = SpMVOp(b.format, ust(xs).format, ust(ys).format)
            backend_execute(be, op, b, xs, ys, beta=0.0 if first else 1.0)
            first = False
    return y


def block_spmm(A: BlockSparseMatrix, X, Y, backend=None):
    """Y = A X (src/block_sparse.jl:284-302): Y zeroed, then every stored
    block adds its product into its slice of Y."""
    from .backend import B200Backend, backend_execute
    from .ops import SpMMOp
    X, Y = ust(X).val, ust(Y).val
    m, n = A.shape
    if X.dim() != 2 or Y.dim() != 2 or X.shape[0] != n or Y.shape[0] != m or X.shape[1] != Y.shape[1]:
        raise IncompatibleExtents(f"BlockSpMM: A is {m}x{n}, X {tuple(X.shape)}, Y {tuple(Y.shape)}")
    be = backend if backend is not None else B200Backend()
    Y.zero_()
    for i, j, b in A.stored():
        Xs = X[A.col_off[j]:A.col_off[j + 1]]
        Ys = Y[A.row_off[i]:A.row_off[i + 1]]
        op = SpMMOp(b.format, ust(Xs).format, ust(Ys).format)
        backend_execute(be, op, b, Xs, Ys, beta=1.0)
    return Y


def update_block_values(A: BlockSparseMatrix, i: int, j: int, new_val: torch.Tensor):
    """Replace block (i, j)'s values (1-based block indices, as
    update_block_values!, ext/CUDAExt/ops/block_mul.jl:310-346): in place in
    the block, and in the assembled CSR through its slot map, so graphs
    captured earlier use the new values."""
    b = A.blocks[i - 1][j - 1]
    if b is None:
        raise UnsupportedFormat(f"update_block_values: block ({i},{j}) is not a USTensor")
    v = nonzeros(b)
    if new_val.numel() != v.numel():
        raise IncompatibleExtents(f"update_block_values: new values length {new_val.numel()} "
                                  f"!= nnz {v.numel()}")
    v.copy_(new_val)
    c = A._compiled
    if c is not None and (i - 1, j - 1) in c.maps:
        c.val[c.maps[(i - 1, j - 1)]] = v
    return A


def mul(y, A: BlockSparseMatrix, x, backend=None):
    """mul!(y, A, x) / mul!(Y, A, X) for a BlockSparseMatrix."""
    if ust(x).val.dim() == 1:
        return block_spmv(A, x, y, backend)
    return block_spmm(A, x, y, backend)
