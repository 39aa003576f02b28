"""numpy front end of the C restatement in oracle.c.

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() and by
bench.py's CPU-baseline leg, always as the checker or as the timed CPU
baseline, never by the product package.  See oracle.c for the reference
semantics (file:line in the JLUST project) that each routine follows.

Dense operands are numpy 2-D arrays in either C order (row-major) or Fortran
order (column-major); their layout is passed to C as (order, leading dim).
bf16 arrays are numpy uint16 arrays holding the bf16 bit patterns.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "liboracle.so")

F32, F64, BF16 = 0, 1, 2

_lib = None


def build() -> str:
    """Compile oracle.c with oracle/Makefile (idempotent) and return the .so path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(
                os.path.join(_HERE, "oracle.c")):
            build()
        _lib = C.CDLL(_SO)
        _declare(_lib)
    return _lib


_p = C.c_void_p
_i64 = C.c_int64
_i = C.c_int
_d = C.c_double


def _declare(L):
    L.or_max_threads.restype = _i
    L.or_set_threads.argtypes = [_i]
    for n in ("or_csr_spmv_f64", "or_csr_spmv_f32"):
        getattr(L, n).argtypes = [_i64, _p, _p, _p, _p, _p, _d, _d, _i]
    L.or_csr_spmv_ref64.argtypes = [_i, _i64, _p, _p, _p, _p, _p, _p, _p, _d, _d, _i]
    for n in ("or_dcsr_spmv_f64", "or_dcsr_spmv_f32"):
        getattr(L, n).argtypes = [_i64, _p, _p, _p, _p, _p, _p, _d, _d, _i]
    for n in ("or_entry_spmv_f64", "or_entry_spmv_f32"):
        getattr(L, n).argtypes = [_i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _d, _d, _i]
    for n in ("or_bbm_periodic_spmv_f64", "or_bbm_periodic_spmv_f32"):
        getattr(L, n).argtypes = ([_i64, _i64, _i64, _i64, _p, _p, _p, _i64, _p, _p, _p]
                                  + [_p, _p, _p, _i64, _d] * 2 + [_p, _p, _d, _d, _i])
    for n in ("or_spgemm_f64", "or_spgemm_f32"):
        getattr(L, n).argtypes = [_i64, _p, _p, _p, _p, _p, _p, _d, _i, _p, _p, _p]
        getattr(L, n).restype = _i64
    for n in ("or_csr_spmm_f32", "or_csr_spmm_f64"):
        getattr(L, n).argtypes = [_i64, _i64, _p, _p, _p, _p, _i64, _i, _p, _i64, _i, _d, _d, _i]
    L.or_csr_spmm_ref64_f32.argtypes = [_i64, _i64, _p, _p, _p, _p, _i64, _i, _p, _i64, _i,
                                        _p, _p, _d, _d, _i]
    for n in ("or_sddmm_f32", "or_sddmm_f64"):
        getattr(L, n).argtypes = [_i64, _i64, _p, _p, _p, _i64, _i, _p, _i64, _i, _p, _p,
                                  _i, _d, _d, _i]
    L.or_sddmm_ref64_f32.argtypes = [_i64, _i64, _p, _p, _p, _i64, _i, _p, _i64, _i, _p, _p,
                                     _p, _p, _i, _d, _d, _i]
    L.or_bsr_spmm_bf16.argtypes = [_i64, _i64, _i, _i, _p, _p, _p, _p, _i64, _p, _i64,
                                   _d, _d, _i]
    L.or_bsr_spmm_ref64_bf16.argtypes = [_i64, _i64, _i, _i, _p, _p, _p, _p, _i64, _p, _i64,
                                         _p, _p, _d, _d, _i]
    L.or_exclusive_scan_i32.argtypes = [_i64, _p, _p, _i]
    L.or_exclusive_scan_i32.restype = _i64
    L.or_csr_to_bsr.argtypes = [_i64, _i64, _i, _i, _p, _p, _p, _i, _i, _p, _p, _p]
    L.or_csr_to_bsr.restype = _i64
    L.or_coo_to_bsr.argtypes = [_i64, _i64, _i64, _i, _i, _p, _p, _p, _i, _i, _p, _p, _p]
    L.or_coo_to_bsr.restype = _i64


def _ptr(a):
    return None if a is None else a.ctypes.data


def _c(a, dtype=None):
    a = np.asarray(a)
    if dtype is not None and a.dtype != dtype:
        a = a.astype(dtype)
    return np.ascontiguousarray(a)


def _layout(a):
    """(order, ld) of a 2-D numpy array: order 0 row-major, 1 column-major."""
    if a.flags.c_contiguous:
        return 0, (a.shape[1] if a.shape[1] > 0 else 1)
    if a.flags.f_contiguous:
        return 1, (a.shape[0] if a.shape[0] > 0 else 1)
    raise ValueError("dense operand must be C- or Fortran-contiguous")


def dtype_code(dt) -> int:
    dt = np.dtype(dt)
    if dt == np.float64:
        return F64
    if dt == np.float32:
        return F32
    if dt == np.uint16:
        return BF16
    raise TypeError(f"oracle: unsupported value type {dt}")


def set_threads(n: int) -> None:
    lib().or_set_threads(int(n))


def max_threads() -> int:
    return int(lib().or_max_threads())


# ---------------------------------------------------------------- SpMV -------
def spmv(rowptr, colind, val, x, y=None, alpha=1.0, beta=0.0, base=0):
    """y = alpha*A*x + beta*y in the reference's row order and value type."""
    rowptr, colind = _c(rowptr, np.int32), _c(colind, np.int32)
    val = _c(val)
    x = _c(x, val.dtype)
    m = rowptr.shape[0] - 1
    y = np.zeros(m, val.dtype) if y is None else _c(y, val.dtype).copy()
    fn = {np.dtype(np.float64): lib().or_csr_spmv_f64,
          np.dtype(np.float32): lib().or_csr_spmv_f32}[val.dtype]
    fn(m, _ptr(rowptr), _ptr(colind), _ptr(val), _ptr(x), _ptr(y), alpha, beta, base)
    return y


def dcsr_spmv(m, fibptr, row_ids, colind, val, x, y=None, alpha=1.0, beta=0.0, base=0):
    """DCSR y = alpha*A*x + beta*y on the stored rows only (JLUST's DCSR walk,
    ext/KernelAbstractionsExt/ops/_walker.jl:323-342); other rows keep y."""
    fibptr, row_ids, colind = (_c(a, np.int32) for a in (fibptr, row_ids, colind))
    val = _c(val)
    x = _c(x, val.dtype)
    y = np.zeros(m, val.dtype) if y is None else _c(y, val.dtype).copy()
    fn = {np.dtype(np.float64): lib().or_dcsr_spmv_f64,
          np.dtype(np.float32): lib().or_dcsr_spmv_f32}[val.dtype]
    fn(row_ids.shape[0], _ptr(fibptr), _ptr(row_ids), _ptr(colind), _ptr(val), _ptr(x), _ptr(y),
       alpha, beta, base)
    return y


def entry_spmv(m, n, rows, val, x, cols=None, colptr=None, y=None, alpha=1.0, beta=0.0, base=0):
    """COO (rows, cols) or CSC (colptr, rows) SpMV as JLUST's COO / scatter
    paths (ops/spmv.jl:386-420): y scaled by beta, then each entry adds
    (alpha*v)*x[col] to its row, here in storage order."""
    rows = _c(rows, np.int32)
    val = _c(val)
    x = _c(x, val.dtype)
    cols = None if cols is None else _c(cols, np.int32)
    colptr = None if colptr is None else _c(colptr, np.int32)
    y = np.zeros(m, val.dtype) if y is None else _c(y, val.dtype).copy()
    fn = {np.dtype(np.float64): lib().or_entry_spmv_f64,
          np.dtype(np.float32): lib().or_entry_spmv_f32}[val.dtype]
    fn(m, n, val.shape[0], _ptr(rows), _ptr(cols), _ptr(colptr), _ptr(val), _ptr(x), _ptr(y),
       alpha, beta, base)
    return y


def entry_spmv_ref64(m, rows, cols, val, x, y=None, alpha=1.0, beta=0.0, base=0):
    """fp64 y and the bound |alpha|*sum|v*x| + |beta*y| per row, from the
    (row, col) list of the entries (COO, or CSC with cols expanded)."""
    r = np.asarray(rows, np.int64) - base
    c = np.asarray(cols, np.int64) - base
    t = np.asarray(val, np.float64) * np.asarray(x, np.float64)[c]
    acc = np.zeros(m)
    mag = np.zeros(m)
    np.add.at(acc, r, t)
    np.add.at(mag, r, np.abs(t))
    yo = np.zeros(m) if y is None or beta == 0 else np.asarray(y, np.float64)
    return alpha * acc + beta * yo, abs(alpha) * mag + np.abs(beta * yo)


def spmv_ref64(rowptr, colind, val, x, y=None, alpha=1.0, beta=0.0, base=0):
    """fp64 y and the per-row bound |alpha|*sum|v*x| + |beta*y|."""
    rowptr, colind = _c(rowptr, np.int32), _c(colind, np.int32)
    val = _c(val)
    x = _c(x, val.dtype)
    m = rowptr.shape[0] - 1
    yin = None if y is None else _c(y, val.dtype)
    out = np.empty(m, np.float64)
    bound = np.empty(m, np.float64)
    lib().or_csr_spmv_ref64(dtype_code(val.dtype), m, _ptr(rowptr), _ptr(colind), _ptr(val),
                            _ptr(x), _ptr(yin), _ptr(out), _ptr(bound), alpha, beta, base)
    return out, bound


# ---------------------------------------------------------------- SpMM -------
def spmm(rowptr, colind, val, B, C=None, alpha=1.0, beta=0.0, base=0, c_order=0):
    """C = alpha*A*B + beta*C (Tiled per-(row,col) order).  B keeps its layout;
    C is returned in `c_order` (0 row-major, 1 column-major) unless given."""
    rowptr, colind = _c(rowptr, np.int32), _c(colind, np.int32)
    val = _c(val)
    B = np.asarray(B)
    assert B.dtype == val.dtype
    m, k = rowptr.shape[0] - 1, B.shape[1]
    if C is None:
        C = np.zeros((m, k), val.dtype, order="C" if c_order == 0 else "F")
    else:
        C = C.copy(order="K")
    bo, ldb = _layout(B)
    co, ldc = _layout(C)
    fn = {np.dtype(np.float32): lib().or_csr_spmm_f32,
          np.dtype(np.float64): lib().or_csr_spmm_f64}[val.dtype]
    fn(m, k, _ptr(rowptr), _ptr(colind), _ptr(val), _ptr(B), ldb, bo, _ptr(C), ldc, co,
       alpha, beta, base)
    return C


def spmm_ref64(rowptr, colind, val, B, C=None, alpha=1.0, beta=0.0, base=0):
    """fp64 C (row-major) and bound, fp32 inputs."""
    rowptr, colind = _c(rowptr, np.int32), _c(colind, np.int32)
    val = _c(val, np.float32)
    B = np.asarray(B)
    m, k = rowptr.shape[0] - 1, B.shape[1]
    bo, ldb = _layout(B)
    if C is not None:
        co, ldc = _layout(C)
    else:
        co, ldc = 0, max(k, 1)
    out = np.empty((m, k), np.float64)
    bound = np.empty((m, k), np.float64)
    lib().or_csr_spmm_ref64_f32(m, k, _ptr(rowptr), _ptr(colind), _ptr(val), _ptr(B), ldb, bo,
                                _ptr(C), ldc, co, _ptr(out), _ptr(bound), alpha, beta, base)
    return out, bound


# ---------------------------------------------------------------- SDDMM ------
def sddmm(rowptr, colind, A, B_kn, out, S=None, mode=0, alpha=1.0, beta=0.0, base=0):
    """Sampled product over the CSR pattern.  A is m x K, B_kn is the logical
    K x n operand (a row-major n x K array enters as its transpose view).
    mode 0: out = alpha*dot + beta*out;  mode 1: out = (alpha*dot)*S + beta*out."""
    rowptr, colind = _c(rowptr, np.int32), _c(colind, np.int32)
    A, B_kn = np.asarray(A), np.asarray(B_kn)
    out = _c(out, A.dtype).copy()
    S = None if S is None else _c(S, A.dtype)
    m, K = rowptr.shape[0] - 1, A.shape[1]
    ao, lda = _layout(A)
    bo, ldb = _layout(B_kn)
    fn = {np.dtype(np.float32): lib().or_sddmm_f32,
          np.dtype(np.float64): lib().or_sddmm_f64}[A.dtype]
    fn(m, K, _ptr(rowptr), _ptr(colind), _ptr(A), lda, ao, _ptr(B_kn), ldb, bo, _ptr(S),
       _ptr(out), mode, alpha, beta, base)
    return out


def sddmm_ref64(rowptr, colind, A, B_kn, out_in=None, S=None, mode=0, alpha=1.0, beta=0.0,
                base=0):
    rowptr, colind = _c(rowptr, np.int32), _c(colind, np.int32)
    A, B_kn = np.asarray(A), np.asarray(B_kn)
    m, K = rowptr.shape[0] - 1, A.shape[1]
    nnz = colind.shape[0]
    ao, lda = _layout(A)
    bo, ldb = _layout(B_kn)
    S = None if S is None else _c(S, np.float32)
    out_in = None if out_in is None else _c(out_in, np.float32)
    out = np.empty(nnz, np.float64)
    bound = np.empty(nnz, np.float64)
    lib().or_sddmm_ref64_f32(m, K, _ptr(rowptr), _ptr(colind), _ptr(A), lda, ao, _ptr(B_kn),
                             ldb, bo, _ptr(S), _ptr(out_in), _ptr(out), _ptr(bound), mode,
                             alpha, beta, base)
    return out, bound


# ---------------------------------------------------------------- BSR SpMM ---
def bsr_spmm(browptr, bcolind, bval_u16, X_u16, b1=64, b2=64, Y=None, alpha=1.0, beta=0.0,
             base=0):
    """fp32 Y = alpha*A*X + beta*Y for a BSRRight matrix with bf16 values/X."""
    browptr, bcolind = _c(browptr, np.int32), _c(bcolind, np.int32)
    bval = _c(bval_u16, np.uint16)
    X = _c(X_u16, np.uint16)
    mb, N = browptr.shape[0] - 1, X.shape[1]
    Y = np.zeros((mb * b1, N), np.float32) if Y is None else _c(Y, np.float32).copy()
    lib().or_bsr_spmm_bf16(mb, N, b1, b2, _ptr(browptr), _ptr(bcolind), _ptr(bval), _ptr(X),
                           N, _ptr(Y), N, alpha, beta, base)
    return Y


def bsr_spmm_ref64(browptr, bcolind, bval_u16, X_u16, b1=64, b2=64, Y=None, alpha=1.0,
                   beta=0.0, base=0):
    browptr, bcolind = _c(browptr, np.int32), _c(bcolind, np.int32)
    bval = _c(bval_u16, np.uint16)
    X = _c(X_u16, np.uint16)
    mb, N = browptr.shape[0] - 1, X.shape[1]
    Yin = None if Y is None else _c(Y, np.float32)
    out = np.empty((mb * b1, N), np.float64)
    bound = np.empty((mb * b1, N), np.float64)
    lib().or_bsr_spmm_ref64_bf16(mb, N, b1, b2, _ptr(browptr), _ptr(bcolind), _ptr(bval),
                                 _ptr(X), N, _ptr(Yin), N, _ptr(out), _ptr(bound), alpha, beta,
                                 base)
    return out, bound


# ---------------------------------------------------------------- scans ------
def exclusive_scan(counts, base=0):
    counts = _c(counts, np.int32)
    out = np.empty(counts.shape[0] + 1, np.int32)
    tot = lib().or_exclusive_scan_i32(counts.shape[0], _ptr(counts), _ptr(out), base)
    if tot < 0:
        raise OverflowError("exclusive_scan: running total exceeds int32")
    return out


# ---------------------------------------------------------------- conversion -
def _bsr_alloc(mb, nnzb, b1, b2, dt):
    return (np.empty(mb + 1, np.int32), np.empty(max(nnzb, 0), np.int32),
            np.empty(max(nnzb, 0) * b1 * b2, dt))


def csr_to_bsr(m, n, rowptr, colind, val, b1, b2, base=0):
    """(browptr, bcolind, bval) of BSRRight((b1,b2)) with ceil(m/b1) block rows."""
    rowptr, colind, val = _c(rowptr, np.int32), _c(colind, np.int32), _c(val)
    dt = dtype_code(val.dtype)
    nnzb = lib().or_csr_to_bsr(m, n, b1, b2, _ptr(rowptr), _ptr(colind), _ptr(val), dt, base,
                               None, None, None)
    mb = (m + b1 - 1) // b1
    bp, bc, bv = _bsr_alloc(mb, nnzb, b1, b2, val.dtype)
    lib().or_csr_to_bsr(m, n, b1, b2, _ptr(rowptr), _ptr(colind), _ptr(val), dt, base,
                        _ptr(bp), _ptr(bc), _ptr(bv))
    return bp, bc, bv


def coo_to_bsr(m, n, rows, cols, val, b1, b2, base=0):
    rows, cols, val = _c(rows, np.int32), _c(cols, np.int32), _c(val)
    dt = dtype_code(val.dtype)
    nnz = rows.shape[0]
    nnzb = lib().or_coo_to_bsr(m, n, nnz, b1, b2, _ptr(rows), _ptr(cols), _ptr(val), dt, base,
                               None, None, None)
    mb = (m + b1 - 1) // b1
    bp, bc, bv = _bsr_alloc(mb, nnzb, b1, b2, val.dtype)
    lib().or_coo_to_bsr(m, n, nnz, b1, b2, _ptr(rows), _ptr(cols), _ptr(val), dt, base,
                        _ptr(bp), _ptr(bc), _ptr(bv))
    return bp, bc, bv


def spgemm(m, n, a_rp, a_ci, a_v, b_rp, b_ci, b_v, alpha=1.0, base=0):
    """C = alpha*A*B as CSR (rowptr, colind, val) with the input's origin, in
    the order of JLUST's scatter-sort-reduce SpGEMM (ext/KernelAbstractionsExt/
    ops/spgemm.jl:40-80, 330-400): row i's products in A-entry then B-entry
    order, scaled by alpha unless it is 1, sorted stably by column, each run
    summed from zero left to right in the value type."""
    a_rp, a_ci, b_rp, b_ci = (_c(x, np.int32) for x in (a_rp, a_ci, b_rp, b_ci))
    a_v = _c(a_v)
    b_v = _c(b_v, a_v.dtype)
    fn = {np.dtype(np.float64): lib().or_spgemm_f64, np.dtype(np.float32): lib().or_spgemm_f32}[a_v.dtype]
    args = [m, _ptr(a_rp), _ptr(a_ci), _ptr(a_v), _ptr(b_rp), _ptr(b_ci), _ptr(b_v), alpha, base]
    nnz = fn(*args, None, None, None)
    rp = np.empty(m + 1, np.int32)
    ci = np.empty(max(nnz, 1), np.int32)
    v = np.empty(max(nnz, 1), a_v.dtype)
    fn(*args, _ptr(rp), _ptr(ci), _ptr(v))
    return rp, ci[:nnz], v[:nnz]


def compose_compressed(n_outer, n_inner, outer, inner, val, base=0, sort=True):
    """The reference's convert_format for a 2-D target whose first level is
    dense over `outer` and whose second is compressed (unique) over `inner`
    (src/convert.jl:302-388), given the source's entries as coordinate pairs in
    storage order: explicit zeros dropped (:316; bf16 given as uint16 bits);
    with `sort`, the entries stably lexsorted by (outer, inner) (:343-355,
    419-424: the level order changes), else kept in storage order, where the
    outer coordinate must not decrease (the dense level's assertion, :246,
    raised here as ValueError); then each run of equal (outer, inner) keeps its
    first value (:222-238).  Returns (ptr, inner, val) with the input's origin."""
    outer = np.asarray(outer, np.int64) - base
    inner = np.asarray(inner, np.int64) - base
    val = np.asarray(val)
    nz = (val & 0x7FFF) != 0 if val.dtype == np.uint16 else val != 0
    o, i, v = outer[nz], inner[nz], val[nz]
    if o.size and (o.min() < 0 or o.max() >= n_outer or i.min() < 0 or i.max() >= n_inner):
        raise ValueError("coordinate outside the extents")
    if sort:
        order = np.lexsort((i, o))
        o, i, v = o[order], i[order], v[order]
    elif np.any(np.diff(o) < 0):
        raise ValueError("outer coordinates decrease in an ordered source")
    keep = np.ones(o.shape[0], bool)
    keep[1:] = (o[1:] != o[:-1]) | (i[1:] != i[:-1])
    o, i, v = o[keep], i[keep], v[keep]
    ptr = np.zeros(n_outer + 1, np.int64)
    np.cumsum(np.bincount(o, minlength=n_outer), out=ptr[1:])
    return (ptr + base).astype(np.int32), (i + base).astype(np.int32), v


def expand_positions(ptr, base=0):
    """The outer coordinate (with origin) of every entry of a compressed level."""
    ptr = np.asarray(ptr, np.int64) - base
    return (np.repeat(np.arange(ptr.shape[0] - 1), np.diff(ptr)) + base).astype(np.int32)


def coo_to_csr(m, n, rows, cols, val, base=0):
    """COO -> CSR: the COO's levels are ordered, so no sort (convert.jl:346-355)."""
    return compose_compressed(m, n, rows, cols, val, base, sort=False)


def csr_to_csr(m, n, rowptr, colind, val, base=0):
    return compose_compressed(m, n, expand_positions(rowptr, base), colind, val, base, sort=False)


def to_coo(rows, cols, val):
    """COO target from an ordered source (convert.jl:316, 346-355): the
    explicit zeros dropped, nothing sorted or merged (COO's row level is not
    unique).  Coordinates keep their origin."""
    rows, cols, val = np.asarray(rows, np.int32), np.asarray(cols, np.int32), np.asarray(val)
    nz = (val & 0x7FFF) != 0 if val.dtype == np.uint16 else val != 0
    return rows[nz], cols[nz], val[nz]


def coo_to_csc(m, n, rows, cols, val, base=0):
    """COO -> CSC (colptr, rowind, val): the level order changes, so sorted."""
    return compose_compressed(n, m, cols, rows, val, base, sort=True)


def csr_to_csc(m, n, rowptr, colind, val, base=0):
    return compose_compressed(n, m, colind, expand_positions(rowptr, base), val, base, sort=True)


def csc_to_csr(m, n, colptr, rowind, val, base=0):
    return compose_compressed(m, n, rowind, expand_positions(colptr, base), val, base, sort=True)


# ------------------------------------------------------ block sparse matrix --
def bsm_assemble(row_sizes, col_sizes, blocks):
    """The one CSR the reference compiles a BlockSparseMatrix of CSR blocks to
    (ext/CUDAExt/ops/block_mul.jl:128-229): blocks = {(i, j): (rowptr,
    colind, val, base)} with 0-based block indices; rows of block row i
    follow row_off[i], and block (i, j)'s entries of each of its rows are
    appended, blocks visited in (i, j) order, columns shifted by col_off[j].
    Returns (rowptr, colind, val), 0-based."""
    row_off = np.concatenate([[0], np.cumsum(row_sizes)]).astype(np.int64)
    col_off = np.concatenate([[0], np.cumsum(col_sizes)]).astype(np.int64)
    n_rows = int(row_off[-1])
    row_nnz = [0] * n_rows
    for (i, j), (rp, ci, v, base) in blocks.items():
        for r in range(row_sizes[i]):
            row_nnz[row_off[i] + r] += int(rp[r + 1]) - int(rp[r])
    rowptr = [0] * (n_rows + 1)
    for r in range(n_rows):
        rowptr[r + 1] = rowptr[r] + row_nnz[r]
    colind = [0] * rowptr[-1]
    dtype = next(iter(blocks.values()))[2].dtype
    val = np.zeros(rowptr[-1], dtype)
    cursor = list(rowptr[:-1])
    for (i, j) in sorted(blocks):
        rp, ci, v, base = blocks[(i, j)]
        for r in range(row_sizes[i]):
            for k in range(int(rp[r]) - base, int(rp[r + 1]) - base):
                slot = cursor[row_off[i] + r]
                cursor[row_off[i] + r] += 1
                colind[slot] = int(ci[k]) - base + int(col_off[j])
                val[slot] = v[k]
    return np.array(rowptr, np.int32), np.array(colind, np.int32), val


def _csr_mv64(rp, ci, v, x, base):
    rp = np.asarray(rp, np.int64) - base
    ci = np.asarray(ci, np.int64) - base
    t = np.asarray(v, np.float64) * np.asarray(x, np.float64)[ci]
    rows = np.repeat(np.arange(rp.shape[0] - 1), np.diff(rp))
    acc = np.zeros(rp.shape[0] - 1)
    mag = np.zeros(rp.shape[0] - 1)
    np.add.at(acc, rows, t)
    np.add.at(mag, rows, np.abs(t))
    return acc, mag


def bbm_spmv_ref64(diags, off, T, bw, n_diag_rows, n_off_rows, n_cols, x):
    """fp64 y = M x for a BlockBandedMatrix and the per-row bound, period by
    period as the reference's execute(BBMSpMVOp) (src/block_banded.jl:79-122):
    diags[t] and off[k-1][t] = (neg, pos) are host CSR tuples (rowptr, colind,
    val, base); period t's diagonal rows get D_t x_t, its level-k coupling
    rows neg x_t + pos x_{t+k}."""
    x = np.asarray(x, np.float64)
    cum = np.concatenate([[0], np.cumsum(n_off_rows)]).astype(np.int64)
    starts = [0]
    for t in range(1, T):
        starts.append(starts[-1] + n_diag_rows + int(cum[min(bw, T - t)]))
    m = T * n_diag_rows + sum((T - k) * n_off_rows[k - 1] for k in range(1, bw + 1))
    y, bound = np.zeros(m), np.zeros(m)
    for t in range(T):
        xt = x[t * n_cols:(t + 1) * n_cols]
        a, g = _csr_mv64(*diags[t][:3], xt, diags[t][3])
        y[starts[t]:starts[t] + n_diag_rows], bound[starts[t]:starts[t] + n_diag_rows] = a, g
        for k in range(1, min(bw, T - 1 - t) + 1):
            neg, pos = off[k - 1][t]
            r0 = starts[t] + n_diag_rows + int(cum[k - 1])
            a1, g1 = _csr_mv64(*neg[:3], xt, neg[3])
            a2, g2 = _csr_mv64(*pos[:3], x[(t + k) * n_cols:(t + k + 1) * n_cols], pos[3])
            y[r0:r0 + n_off_rows[k - 1]] = a1 + a2
            bound[r0:r0 + n_off_rows[k - 1]] = g1 + g2
    return y, bound


def bbm_periodic_spmv(T, n_diag, n_off, n_cols, diag, neg, pos, x, y=None, alpha=1.0, beta=0.0,
                      base=0, patches=()):
    """Periodic block-banded y = alpha*M*x + beta*y in the order of JLUST's
    fused periodic kernel (ext/KernelAbstractionsExt/ops/block_periodic.jl:
    114-163); diag is a (rowptr, colind, val) CSR tuple with selector
    `patches` (first row, last row, column of the first row, value; relative
    to the diagonal block), neg / pos each a CSR tuple or a ShiftedDiag
    selector ("shifted", shift, val)."""
    d = [_c(diag[0], np.int32), _c(diag[1], np.int32), _c(diag[2])]
    dt = d[2].dtype
    x = _c(x, dt)
    rows = T * n_diag + (T - 1) * n_off
    y = np.zeros(rows, dt) if y is None else _c(y, dt).copy()
    fn = {np.dtype(np.float64): lib().or_bbm_periodic_spmv_f64,
          np.dtype(np.float32): lib().or_bbm_periodic_spmv_f32}[dt]
    keep = []

    def blk(b):
        if isinstance(b[0], str):
            return [None, None, None, int(b[1]), float(b[2])]
        a = [_c(b[0], np.int32), _c(b[1], np.int32), _c(b[2], dt)]
        keep.extend(a)
        return [_ptr(a[0]), _ptr(a[1]), _ptr(a[2]), 0, 0.0]
    pr = _c(np.array([v for p in patches for v in (p[0], p[1])], np.int64))
    pc = _c(np.array([p[2] for p in patches], np.int64))
    pv = _c(np.array([p[3] for p in patches], np.float64))
    fn(T, n_diag, n_off, n_cols, _ptr(d[0]), _ptr(d[1]), _ptr(d[2]), len(patches), _ptr(pr),
       _ptr(pc), _ptr(pv), *blk(neg), *blk(pos), _ptr(x), _ptr(y), alpha, beta, base)
    return y


def bsm_compile(row_sizes, col_sizes, blocks, shifted=None):
    """The reference's full BlockSparseMatrix compile (ext/CUDAExt/ops/
    block_mul.jl:89-229): ShiftedDiag blocks (`shifted` = {(i, j): (shift,
    val)}) and CSR blocks that are a constant times the identity (one entry
    per row, at the row's own column, all equal) become selector patches
    (first row, last row, column of the first row, value), 0-based, in
    (i, j) order; the other CSR blocks are assembled by bsm_assemble.
    Returns (rowptr, colind, val, patches)."""
    row_off = np.concatenate([[0], np.cumsum(row_sizes)]).astype(np.int64)
    col_off = np.concatenate([[0], np.cumsum(col_sizes)]).astype(np.int64)
    shifted = shifted or {}
    keys = sorted(set(blocks) | set(shifted))
    csr, patches = {}, []
    for (i, j) in keys:
        r0, r1 = int(row_off[i]), int(row_off[i]) + row_sizes[i] - 1
        if (i, j) in shifted:
            sh, v = shifted[(i, j)]
            patches.append((r0, r1, int(col_off[j]) + sh, v))
            continue
        rp, ci, v, base = blocks[(i, j)]
        rp0 = np.asarray(rp, np.int64) - base
        ci0 = np.asarray(ci, np.int64) - base
        m = row_sizes[i]
        sel = (rp0.shape[0] == m + 1 and rp0[-1] - rp0[0] == m and np.all(np.diff(rp0) == 1)
               and np.all(ci0[rp0[:-1]] == np.arange(m)) and np.all(np.asarray(v) == v[0]))
        if sel:
            patches.append((r0, r1, int(col_off[j]), float(v[0])))
        else:
            csr[(i, j)] = blocks[(i, j)]
    dtype = next(iter(blocks.values()))[2].dtype
    if csr:
        rp, ci, v = bsm_assemble(row_sizes, col_sizes, csr)
    else:
        rp, ci, v = np.zeros(int(row_off[-1]) + 1, np.int32), np.zeros(0, np.int32), np.zeros(0, dtype)
    return rp, ci, v, patches


def csr_patched_spmv(rowptr, colind, val, patches, x, y=None, beta=0.0, alpha=1.0):
    """y = alpha (A x + (patches) x) (+ beta y) in the value type, in the
    order of JLUST's patched kernel (ext/KernelAbstractionsExt/ops/
    block_periodic.jl:40-79, alpha = 1 there): per row the CSR entries summed
    in storage order, the patches summed in patch order into a second sum,
    then the two added.  Plain loops: small cases only."""
    val = np.asarray(val)
    T = val.dtype.type
    x = np.asarray(x, val.dtype)
    m = len(rowptr) - 1
    out = np.zeros(m, val.dtype) if y is None else np.asarray(y, val.dtype).copy()
    b = T(beta)
    for r in range(m):
        acc = T(0)
        for k in range(int(rowptr[r]), int(rowptr[r + 1])):
            acc = T(acc + T(val[k] * x[colind[k]]))
        pacc = T(0)
        for (r0, r1, c0, v) in patches:
            if r0 <= r <= r1:
                pacc = T(pacc + T(T(v) * x[r - r0 + c0]))
        o = T(T(alpha) * T(acc + pacc))
        if b != 0:
            o = T(o + T(b * out[r]))
        out[r] = o
    return out
