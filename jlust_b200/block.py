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

ShiftedDiag blocks and CSR blocks that are a constant times the identity
become selector patches (ext/CUDAExt/ops/block_mul.jl:89-229): they are kept
out of the assembled CSR and added by the patched SpMV kernel.
"""
from __future__ import annotations

import numpy as np
import torch

from .errors import IncompatibleExtents, UnsupportedFormat, UnsupportedValueType
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
        return all(b.format.family in ("CSR", "ShiftedDiag") for _, _, b in self.stored())


def _host_csr(b: USTensor):
    base = b.origin.offset
    rp = positions(b, 2).cpu().numpy().astype(np.int64) - base
    ci = coordinates(b, 2).cpu().numpy().astype(np.int64) - base
    return rp, ci


class _Graphed:
    """Replays self.spmv(x, y) from a CUDA graph captured per (y, x) buffer
    pair; inside a capture the caller started, launches it directly."""

    def run(self, x, y):
        if torch.cuda.is_current_stream_capturing():
            self.spmv(x, y)          # a capture the caller started records the launch
            return
        # a graph bakes in the buffers' addresses, element type and strides
        key = (y.data_ptr(), x.data_ptr(), x.dtype, y.dtype, x.stride(), y.stride())
        g = self.graphs.get(key)
        if g is None:
            self.spmv(x, y)          # first use outside the graph, then capture
            torch.cuda.current_stream(y.device).synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.spmv(x, y)
            self.graphs[key] = g
        g.replay()


class _Assembled(_Graphed):
    """One CSR of m x n assembled from parts (key, row offset, column offset,
    CSR block) in order: each part's rows append their entries, in storage
    order, to the rows at its row offset, columns shifted by its column offset
    (the order of ext/CUDAExt/ops/block_mul.jl:128-229).  Keeps a slot map per
    keyed part and the CUDA graphs of its SpMV per (y, x) buffer pair."""

    def __init__(self, m, n, parts, dtype, dev=None, patches=()):
        dev = nonzeros(parts[0][3]).device if dev is None else dev
        row_nnz = np.zeros(m, np.int64)
        host = []
        for key, r0, c0, b in parts:
            rp, ci = _host_csr(b)
            host.append((key, r0, c0, b, rp, ci))
            row_nnz[r0:r0 + rp.shape[0] - 1] += np.diff(rp)
        rowptr = np.zeros(m + 1, np.int64)
        np.cumsum(row_nnz, out=rowptr[1:])
        if rowptr[-1] > np.iinfo(np.int32).max - 1:
            raise IncompatibleExtents("assembled nnz exceeds Int32 positions")
        colind = np.zeros(int(rowptr[-1]), np.int32)
        cursor = rowptr[:-1].copy()
        self.val = torch.empty(int(rowptr[-1]), dtype=dtype, device=dev)
        self.maps = {}
        for key, r0, c0, b, rp, ci in host:
            nr = rp.shape[0] - 1
            lens = np.diff(rp)
            rows = np.repeat(np.arange(nr), lens)
            within = np.arange(ci.shape[0]) - np.repeat(rp[:-1], lens)
            slots_np = cursor[r0 + rows] + within
            colind[slots_np] = (ci + c0).astype(np.int32)
            cursor[r0:r0 + nr] += lens
            slots = torch.from_numpy(slots_np).to(dev)
            self.val[slots] = nonzeros(b)
            if key is not None:
                self.maps[key] = slots
        self.csr = csr_tensor(torch.from_numpy(rowptr.astype(np.int32)).to(dev),
                              torch.from_numpy(colind).to(dev), self.val, (m, n), origin=0)
        # selector patches (first row, last row, column of the first row, value)
        self.patches = list(patches)
        if self.patches:
            pr = np.array([[p[0], p[1]] for p in self.patches], np.int64).reshape(-1)
            self.p_rows = torch.from_numpy(pr).to(dev)
            self.p_cols = torch.from_numpy(np.array([p[2] for p in self.patches], np.int64)).to(dev)
            self.p_vals = torch.from_numpy(np.array([p[3] for p in self.patches], np.float64)).to(dev)
        self.graphs = {}

    def spmv(self, x, y):
        if not self.patches:
            from .backend import spmv
            spmv(self.csr, x, y)
            return
        import ctypes as C

        from . import _lib
        from .backend import _DTYPE, _same_device, _stream
        m, n = self.csr.extents
        dev = _same_device(self.val, x, y)

        def p(t):
            return C.c_void_p(t.data_ptr())
        _lib.call("jlb_csr_patched_spmv", _stream(dev), _DTYPE[self.val.dtype], 0, m, n,
                  self.val.numel(), p(positions(self.csr, 2)), p(coordinates(self.csr, 2)),
                  p(self.val), len(self.patches), p(self.p_rows), p(self.p_cols), p(self.p_vals),
                  p(x), p(y), 1.0, 0.0)


def _bsm_parts(A: "BlockSparseMatrix", r0=0, c0=0, key=True):
    return [((i, j) if key else None, r0 + int(A.row_off[i]), c0 + int(A.col_off[j]), b)
            for i, j, b in sorted(A.stored(), key=lambda t: (t[0], t[1]))]


def _selector_value(b: USTensor):
    """(True, v) when CSR block b is v times the identity on its rows: one
    entry per row, at the row's own column, all equal (ext/CUDAExt/ops/
    block_mul.jl:89-115); else (False, 0)."""
    if b.format.family != "CSR":
        return False, 0.0
    m = b.extents[0]
    rp, ci = _host_csr(b)
    if rp.shape[0] != m + 1 or rp[-1] - rp[0] != m or np.any(np.diff(rp) != 1):
        return False, 0.0
    if np.any(ci[rp[:-1]] != np.arange(m)):
        return False, 0.0
    v = nonzeros(b).cpu().numpy()
    if v.size == 0 or np.any(v != v[0]):
        return False, 0.0
    return True, float(v[0])


def _Compiled(A: "BlockSparseMatrix") -> _Assembled:
    """The reference's compile of a BlockSparseMatrix (block_mul.jl:128-229):
    ShiftedDiag blocks and CSR blocks that are constant multiples of the
    identity become selector patches, the other CSR blocks one CSR."""
    m, n = A.shape
    parts, patches = [], []
    for i, j, b in sorted(A.stored(), key=lambda t: (t[0], t[1])):
        r0, c0, rows = int(A.row_off[i]), int(A.col_off[j]), A.row_sizes[i]
        if b.format.family == "ShiftedDiag":
            shift, v = b.format.diag
            if shift < 0 or rows - 1 + shift >= A.col_sizes[j]:
                raise IncompatibleExtents(f"BlockSparseMatrix: ShiftedDiag block ({i + 1},{j + 1}) "
                                          f"with shift {shift} reaches outside its columns")
            patches.append((r0, r0 + rows - 1, c0 + shift, v))
            continue
        sel, v = _selector_value(b)
        if sel:
            patches.append((r0, r0 + rows - 1, c0, v))
        else:
            parts.append(((i, j), r0, c0, b))
    # the CSR blocks' device; a matrix of patches only takes its first block's
    dev = nonzeros(parts[0][3] if parts else next(A.stored())[2]).device
    return _Assembled(m, n, parts, A.dtype, dev, patches)


def _vec(t, what, dtype, op="BlockSpMV"):
    """x or y of a block product: a contiguous vector of the matrix's value
    type (the kernels read and write dtype-sized elements at unit stride)."""
    t = ust(t).val
    if t.dim() != 1 or (t.numel() > 1 and t.stride(0) != 1):
        raise IncompatibleExtents(f"{op}: {what} must be a contiguous vector")
    if t.dtype != dtype:
        raise UnsupportedValueType(f"{op}: {what} has value type {t.dtype}, the matrix {dtype}")
    return t


def block_spmv(A: BlockSparseMatrix, x, y, backend=None):
    """y = A x (mul!(y, A, x), src/block_sparse.jl:266-282 and
    ext/CUDAExt/ops/block_mul.jl:231-306)."""
    from .backend import B200Backend, backend_execute
    from .ops import SpMVOp
    x, y = _vec(x, "x", A.dtype), _vec(y, "y", A.dtype)
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
    if c is not None:
        if (i - 1, j - 1) in c.maps:
            c.val[c.maps[(i - 1, j - 1)]] = v
        else:
            A._compiled = None       # a block compiled into a patch: rebuild next time
    return A


def mul(y, A, x, backend=None):
    """mul!(y, A, x) / mul!(Y, A, X) for a BlockSparseMatrix, mul!(y, M, x)
    for a BlockBandedMatrix."""
    if isinstance(A, BlockBandedMatrix):
        return bbm_spmv(A, x, y)
    if ust(x).val.dim() == 1:
        return block_spmv(A, x, y, backend)
    return block_spmm(A, x, y, backend)


class BlockBandedMatrix:
    """`BlockBandedMatrix(diags, off_diags, T, bw, n_diag_rows, n_off_rows,
    n_cols)` (src/block_banded.jl): T periods of n_cols columns each; `diags`
    is one diagonal block (a CSR USTensor or an all-CSR BlockSparseMatrix of
    n_diag_rows x n_cols) shared by every period, or a list of T of them;
    `off_diags[k-1]` couples period t with period t+k for k = 1..bw, as one
    (neg, pos) pair of n_off_rows[k-1] x n_cols CSR blocks shared by every
    transition or a list of T-k pairs.  Rows run period by period: period t's
    n_diag_rows diagonal rows, then for each k <= min(bw, T-t) its coupling
    rows, which compute neg x_t + pos x_{t+k} (block_banded.jl:79-122).

    The reference's bw = 1 form `BlockBandedMatrix(diag, neg_off, pos_off, T,
    n_diag_rows, n_off_rows, n_cols)` (src/block_banded.jl:56-62: one shared
    coupling pair, n_off_rows an Int) is accepted too: it is recognised, as
    Julia's dispatch does, by a coupling block in the second position."""

    def __init__(self, diags, off_diags, T, bw, n_diag_rows, n_off_rows, n_cols):
        if isinstance(off_diags, USTensor):
            # (diag, neg_off, pos_off, T, n_diag_rows, n_off_rows, n_cols)
            neg, pos, T, n_diag_rows, n_off, n_cols = off_diags, T, bw, n_diag_rows, n_off_rows, n_cols
            if not isinstance(pos, USTensor) or not isinstance(n_off, (int, np.integer)):
                raise ValueError("BlockBandedMatrix(diag, neg_off, pos_off, T, n_diag_rows, "
                                 "n_off_rows, n_cols): neg_off and pos_off must be USTensors "
                                 "and n_off_rows an Int")
            off_diags, bw, n_off_rows = [(neg, pos)], 1, [int(n_off)]
        if T < 1 or bw < 0 or len(off_diags) != bw or len(n_off_rows) != bw:
            raise ValueError("BlockBandedMatrix: need T >= 1 and bw levels of (neg, pos) blocks "
                             "and row counts")
        self.diags = diags if isinstance(diags, (list, tuple)) else [diags] * T
        if len(self.diags) != T:
            raise ValueError(f"BlockBandedMatrix: {len(self.diags)} diagonal blocks for T = {T}")
        self.off = []
        for k in range(1, bw + 1):
            lv = off_diags[k - 1]
            pairs = [lv] * (T - k) if isinstance(lv, tuple) else list(lv)
            if len(pairs) != T - k:
                raise ValueError(f"BlockBandedMatrix: level {k} needs {T - k} (neg, pos) pairs")
            self.off.append(pairs)
        self.T, self.bw, self.n_cols = T, bw, n_cols
        self.n_diag_rows, self.n_off_rows = n_diag_rows, list(n_off_rows)
        for t, d in enumerate(self.diags):
            if tuple(d.shape if isinstance(d, BlockSparseMatrix) else d.extents) != (n_diag_rows, n_cols):
                raise ValueError(f"BlockBandedMatrix: diagonal block of period {t + 1} is not "
                                 f"{n_diag_rows}x{n_cols}")
        # a coupling block may be narrower than a period: its columns are the
        # first ones of the period's x slice, as the reference's fused
        # periodic kernel indexes them (block_periodic.jl:114-163)
        for k, pairs in enumerate(self.off, start=1):
            for neg, pos in pairs:
                for b in (neg, pos):
                    rows, cols = b.extents
                    if rows != self.n_off_rows[k - 1] or cols > n_cols:
                        raise ValueError(f"BlockBandedMatrix: level-{k} blocks must have "
                                         f"{self.n_off_rows[k - 1]} rows and at most {n_cols} "
                                         f"columns (got {rows}x{cols})")
        # first row of each period (block_banded.jl _bbm_diag_starts)
        cum = np.concatenate([[0], np.cumsum(self.n_off_rows)]).astype(np.int64)
        starts = [0]
        for t in range(1, T):
            starts.append(starts[-1] + n_diag_rows + int(cum[min(bw, T - t)]))
        self.starts, self.cum_off = starts, cum
        # one value type for every block (Base.eltype(M) is the diagonal's,
        # src/block_banded.jl:72-75; the fused products read all blocks as it)
        ts = {_values_dtype(d) for d in self.diags}
        ts |= {nonzeros(b).dtype for pairs in self.off for pr in pairs for b in pr
               if b.format.family != "ShiftedDiag"}
        if len(ts) != 1:
            raise ValueError(f"BlockBandedMatrix: mixed element types {sorted(map(str, ts))}")
        self.dtype = ts.pop()
        self._compiled = None

    @property
    def shape(self):
        rows = self.T * self.n_diag_rows + sum((self.T - k) * self.n_off_rows[k - 1]
                                               for k in range(1, self.bw + 1))
        return rows, self.T * self.n_cols

    def parts(self):
        parts = []
        for t in range(self.T):
            r0, c0 = self.starts[t], t * self.n_cols
            d = self.diags[t]
            if isinstance(d, BlockSparseMatrix):
                if not d.compilable():
                    raise UnsupportedFormat("BlockBandedMatrix: diagonal blocks must be CSR or ShiftedDiag")
                parts += _bsm_parts(d, r0, c0, key=False)
            else:
                parts.append((None, r0, c0, d))
            for k in range(1, min(self.bw, self.T - 1 - t) + 1):
                neg, pos = self.off[k - 1][t]
                rk = r0 + self.n_diag_rows + int(self.cum_off[k - 1])
                parts.append((None, rk, c0, neg))
                parts.append((None, rk, (t + k) * self.n_cols, pos))
        for _, _, _, b in parts:
            if b.format.family not in ("CSR", "ShiftedDiag"):
                raise UnsupportedFormat("BlockBandedMatrix: blocks must be CSR or ShiftedDiag")
        return parts


def _values_dtype(d):
    return d.dtype if isinstance(d, BlockSparseMatrix) else nonzeros(d).dtype


def _split_patches(parts):
    """Parts (key, row offset, column offset, block) split into CSR parts and
    selector patches, one per ShiftedDiag block (first row, last row, column
    of the first row, value)."""
    csr, patches = [], []
    for key, r0, c0, b in parts:
        if b.format.family != "ShiftedDiag":
            csr.append((key, r0, c0, b))
            continue
        (rows, cols), (shift, v) = b.extents, b.format.diag
        if shift < 0 or rows - 1 + shift >= cols:
            raise IncompatibleExtents(f"ShiftedDiag block with shift {shift} reaches outside "
                                      f"its {cols} columns")
        patches.append((r0, r0 + rows - 1, c0 + shift, v))
    return csr, patches


def bbm_spmv(M: BlockBandedMatrix, x, y):
    """y = M x (execute(BBMSpMVOp, M, x, y), src/block_banded.jl:79-122): the
    periodic kernel when one diagonal block and one coupling pair are shared
    (bw = 1), otherwise one assembled CSR; either replayed from a CUDA graph
    per buffer pair."""
    x, y = _vec(x, "x", M.dtype, "BBMSpMV"), _vec(y, "y", M.dtype, "BBMSpMV")
    m, n = M.shape
    if x.numel() != n or y.numel() != m:
        raise IncompatibleExtents(f"BBMSpMV: M is {m}x{n}, x has {x.numel()}, y has {y.numel()}")
    if M._compiled is None:
        if _Periodic.eligible(M):
            M._compiled = _Periodic(M)
        else:
            parts, patches = _split_patches(M.parts())
            first = parts[0][3] if parts else M.parts()[0][3]
            M._compiled = _Assembled(m, n, parts, nonzeros(first).dtype, nonzeros(first).device,
                                     patches)
    M._compiled.run(x, y)
    return y


class _Periodic(_Graphed):
    """A periodic BlockBandedMatrix (one shared diagonal block, bw = 1, one
    shared coupling pair) through jlb_bbm_periodic_spmv: the shared blocks are
    stored once, not T times (JLUST's fused periodic path,
    ext/CUDAExt/ops/block_mul.jl:584-680).  A BlockSparseMatrix diagonal is
    compiled once, its selector blocks kept as patches; a coupling block may
    be CSR or ShiftedDiag."""

    def __init__(self, M: "BlockBandedMatrix"):
        d = M.diags[0]
        self.patches = []
        if isinstance(d, BlockSparseMatrix):
            self.diag_asm = _Compiled(d)          # the diagonal assembled once
            self.patches = self.diag_asm.patches
            d = self.diag_asm.csr
        neg, pos = M.off[0][0]
        for b in (neg, pos):
            if b.format.family == "ShiftedDiag":
                shift, _ = b.format.diag
                if shift < 0 or M.n_off_rows[0] - 1 + shift >= b.extents[1]:
                    raise IncompatibleExtents(f"BlockBandedMatrix: ShiftedDiag coupling block "
                                              f"with shift {shift} reaches outside its columns")
        self.blocks = (d, neg, pos)
        self.M = M
        self.graphs = {}

    @staticmethod
    def eligible(M: "BlockBandedMatrix") -> bool:
        if M.bw != 1 or M.T < 2 or any(d is not M.diags[0] for d in M.diags):
            return False
        if any(p is not M.off[0][0] for p in M.off[0]):
            return False
        d = M.diags[0]
        if isinstance(d, BlockSparseMatrix):
            if not d.compilable():
                return False
            base = 0
        else:
            if d.format.family != "CSR":
                return False
            base = d.origin.offset
        neg, pos = M.off[0][0]
        return all(b.format.family == "ShiftedDiag"
                   or (b.format.family == "CSR" and b.origin.offset == base) for b in (neg, pos))

    def spmv(self, x, y):
        import ctypes as C

        from . import _lib
        from .backend import _DTYPE, _same_device, _stream
        d, neg, pos = self.blocks
        M = self.M
        val = nonzeros(d)
        dev = _same_device(val, x, y)

        def p(t):
            return C.c_void_p(t.data_ptr()) if t is not None else C.c_void_p(0)

        def blk(b):
            if b.format.family == "ShiftedDiag":
                shift, v = b.format.diag
                return [None, None, None, shift, v]
            _same_device(nonzeros(b), val)
            return [p(positions(b, 2)), p(coordinates(b, 2)), p(nonzeros(b)), 0, 0.0]
        a = getattr(self, "diag_asm", None)
        pr, pc, pv = (a.p_rows, a.p_cols, a.p_vals) if self.patches else (None, None, None)
        _lib.call("jlb_bbm_periodic_spmv", _stream(dev), _DTYPE[val.dtype], d.origin.offset, M.T,
                  M.n_diag_rows, M.n_off_rows[0], M.n_cols,
                  p(positions(d, 2)), p(coordinates(d, 2)), p(val),
                  len(self.patches), p(pr), p(pc), p(pv),
                  *blk(neg), *blk(pos), p(x), p(y), 1.0, 0.0)
