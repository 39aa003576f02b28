"""GPU format conversion (src/convert.jl:302-388): BSRRight((b1, b2)) from CSR
and COO sources, CSR from COO and CSR (a stable compaction: the reference
does not sort a source whose levels are ordered), CSC from COO and CSR and CSR
from CSC (sorted compression: the reference lexsorts when the level order
changes), and the position-buffer scan (src/convert.jl:154-168).  Results are
bit-identical to the reference's CPU composer (with the block-row level
extent ceil(m / b1) for BSR).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from .backend import _DTYPE, _ptr, _same_device, _stream
from .errors import UnsupportedFormat, UnsupportedValueType
from .formats import TensorFormat
from .formats import Formats
from .tensor import (USTensor, bsr_tensor, coo_tensor, coordinates, csr_tensor, nonzeros,
                     positions)


def exclusive_scan(counts: torch.Tensor, base: int = 0) -> torch.Tensor:
    """Position buffer of int32 counts: out[0] = base, out[i+1] = out[i] + counts[i]."""
    dev = _same_device(counts)
    n = counts.numel()
    out = torch.empty(n + 1, dtype=torch.int32, device=dev)
    ws_bytes = _lib.load().jlb_scan_workspace_size(n)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    _lib.call("jlb_exclusive_scan_i32", _stream(dev), n, _ptr(counts), _ptr(out), int(base),
              _ptr(ws), ws_bytes)
    return out


def _to_bsr(u: USTensor, b1: int, b2: int) -> USTensor:
    val = nonzeros(u)
    if val.dtype not in _DTYPE:
        raise UnsupportedValueType(f"convert_format: value type {val.dtype}")
    dt = _DTYPE[val.dtype]
    m, n = u.extents
    base = u.origin.offset
    mb = -(-m // b1)
    L = _lib.load()
    if u.format.family == "CSR":
        rowptr, colind = positions(u, 2), coordinates(u, 2)
        dev = _same_device(rowptr, colind, val)
        st = _stream(dev)
        nnz = val.numel()
        ws_bytes = L.jlb_csr_to_bsr_workspace_size(m, n, nnz, b1, b2)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
        browptr = torch.empty(mb + 1, dtype=torch.int32, device=dev)
        nnzb = C.c_int64()
        _lib.call("jlb_csr_to_bsr_count", st, dt, base, m, n, nnz, _ptr(rowptr), _ptr(colind),
                  _ptr(val), b1, b2, _ptr(browptr), C.byref(nnzb), _ptr(ws), ws_bytes)
        bcolind = torch.empty(nnzb.value, dtype=torch.int32, device=dev)
        bval = torch.empty(nnzb.value * b1 * b2, dtype=val.dtype, device=dev)
        _lib.call("jlb_csr_to_bsr_fill", st, dt, base, m, n, nnz, _ptr(rowptr), _ptr(colind),
                  _ptr(val), b1, b2, _ptr(browptr), nnzb.value, _ptr(bcolind), _ptr(bval),
                  _ptr(ws), ws_bytes)
    elif u.format.family == "COO":
        rows, cols = coordinates(u, 1), coordinates(u, 2)
        dev = _same_device(rows, cols, val)
        st = _stream(dev)
        nnz = val.numel()
        ws_bytes = L.jlb_coo_to_bsr_workspace_size(m, n, nnz, b1, b2, 0)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
        browptr = torch.empty(mb + 1, dtype=torch.int32, device=dev)
        nnzb = C.c_int64()
        _lib.call("jlb_coo_to_bsr_count", st, dt, base, m, n, nnz, _ptr(rows), _ptr(cols),
                  _ptr(val), b1, b2, _ptr(browptr), C.byref(nnzb), _ptr(ws), ws_bytes)
        ws_bytes = L.jlb_coo_to_bsr_workspace_size(m, n, nnz, b1, b2, nnzb.value)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
        bcolind = torch.empty(nnzb.value, dtype=torch.int32, device=dev)
        bval = torch.empty(nnzb.value * b1 * b2, dtype=val.dtype, device=dev)
        _lib.call("jlb_coo_to_bsr_fill", st, dt, base, m, n, nnz, _ptr(rows), _ptr(cols),
                  _ptr(val), b1, b2, _ptr(browptr), nnzb.value, _ptr(bcolind), _ptr(bval),
                  _ptr(ws), ws_bytes)
    else:
        raise UnsupportedFormat(f"convert_format: {u.format.name} -> BSR is not on B200Backend")
    return bsr_tensor(browptr, bcolind, bval, (m, n), (b1, b2), origin=u.origin)


def convert_format(u: USTensor, fmt: TensorFormat) -> USTensor:
    """convert_format(u, fmt) for the conversions the backend runs on the GPU."""
    if fmt.family == "BSR" and fmt.keys[2].dim == "i":
        return _to_bsr(u, *fmt.block)
    if fmt == Formats.CSR and u.format.family in ("COO", "CSR", "CSC"):
        return _to_csr(u)
    if fmt == Formats.CSC and u.format.family in ("COO", "CSR", "CSC"):
        return _to_csc(u)
    if fmt == Formats.COO and u.format.family in ("COO", "CSR"):
        return _to_coo(u)
    if fmt == u.format:
        return u
    raise UnsupportedFormat(f"convert_format: {u.format.name} -> {fmt.name} is not on B200Backend")


def _expand(ptr, n_outer, nnz, base, dev):
    """The outer coordinate of every entry of a compressed level."""
    out = torch.empty(max(nnz, 1), dtype=torch.int32, device=dev)
    _lib.call("jlb_positions_to_coordinates", _stream(dev), base, n_outer, nnz, _ptr(ptr),
              _ptr(out))
    return out[:nnz]


def _coo_to_csr(m, n, rows, cols, val, base, dev):
    """Stable compaction of row-ordered COO entries into CSR buffers."""
    dt = _DTYPE[val.dtype]
    st = _stream(dev)
    nnz = val.numel()
    ws_bytes = _lib.load().jlb_coo_to_csr_workspace_size(m, n, nnz)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    rowptr = torch.empty(m + 1, dtype=torch.int32, device=dev)
    nout = C.c_int64()
    _lib.call("jlb_coo_to_csr_count", st, dt, base, m, n, nnz, _ptr(rows), _ptr(cols), _ptr(val),
              _ptr(rowptr), C.byref(nout), _ptr(ws), ws_bytes)
    colind = torch.empty(nout.value, dtype=torch.int32, device=dev)
    out = torch.empty(nout.value, dtype=val.dtype, device=dev)
    _lib.call("jlb_coo_to_csr_fill", st, dt, base, m, n, nnz, _ptr(rows), _ptr(cols), _ptr(val),
              nout.value, _ptr(colind), _ptr(out), _ptr(ws), ws_bytes)
    return rowptr, colind, out


def _sorted_compress(n_outer, n_inner, outer, inner, val, base, dev):
    """Entries lexsorted by (outer, inner, storage index) and compressed
    along the outer coordinate."""
    dt = _DTYPE[val.dtype]
    st = _stream(dev)
    nnz = val.numel()
    ws_bytes = _lib.load().jlb_sorted_compress_workspace_size(n_outer, nnz)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    ptr = torch.empty(n_outer + 1, dtype=torch.int32, device=dev)
    nout = C.c_int64()
    _lib.call("jlb_sorted_compress_count", st, dt, base, n_outer, n_inner, nnz, _ptr(outer),
              _ptr(inner), _ptr(val), _ptr(ptr), C.byref(nout), _ptr(ws), ws_bytes)
    inner_out = torch.empty(nout.value, dtype=torch.int32, device=dev)
    out = torch.empty(nout.value, dtype=val.dtype, device=dev)
    _lib.call("jlb_sorted_compress_fill", st, dt, base, n_outer, n_inner, nnz, _ptr(outer),
              _ptr(inner), _ptr(val), _ptr(ptr), nout.value, _ptr(inner_out), _ptr(out),
              _ptr(ws), ws_bytes)
    return ptr, inner_out, out


def _entries(u: USTensor):
    """(rows, cols, values, device) of a CSR, CSC or COO tensor, rows or
    columns of a compressed level expanded on the device."""
    val = nonzeros(u)
    if val.dtype not in _DTYPE:
        raise UnsupportedValueType(f"convert_format: value type {val.dtype}")
    m, n = u.extents
    base, nnz = u.origin.offset, val.numel()
    fam = u.format.family
    if fam == "COO":
        rows, cols = coordinates(u, 1), coordinates(u, 2)
        dev = _same_device(rows, cols, val)
    elif fam == "CSR":
        rowptr, cols = positions(u, 2), coordinates(u, 2)
        dev = _same_device(rowptr, cols, val)
        rows = _expand(rowptr, m, nnz, base, dev)
    elif fam == "CSC":
        colptr, rows = positions(u, 2), coordinates(u, 2)
        dev = _same_device(colptr, rows, val)
        cols = _expand(colptr, n, nnz, base, dev)
    else:
        raise UnsupportedFormat(f"convert_format: {u.format.name} source is not on B200Backend")
    return rows, cols, val, dev


def _to_csr(u: USTensor) -> USTensor:
    m, n = u.extents
    rows, cols, val, dev = _entries(u)
    if u.format.family == "CSC":     # level order changes: the reference sorts
        rowptr, colind, out = _sorted_compress(m, n, rows, cols, val, u.origin.offset, dev)
    else:                            # ordered source: storage order kept
        rowptr, colind, out = _coo_to_csr(m, n, rows, cols, val, u.origin.offset, dev)
    return csr_tensor(rowptr, colind, out, (m, n), origin=u.origin)


def _to_csc(u: USTensor) -> USTensor:
    m, n = u.extents
    rows, cols, val, dev = _entries(u)
    colptr, rowind, out = _sorted_compress(n, m, cols, rows, val, u.origin.offset, dev)
    return USTensor((m, n), Formats.CSC, (None, colptr), (None, rowind), out, u.origin)


def _to_coo(u: USTensor) -> USTensor:
    """COO from an ordered source (COO, CSR): the explicit zeros dropped, the
    other entries in storage order."""
    m, n = u.extents
    rows, cols, val, dev = _entries(u)
    dt = _DTYPE[val.dtype]
    st = _stream(dev)
    nnz, base = val.numel(), u.origin.offset
    ws_bytes = _lib.load().jlb_coo_drop_zeros_workspace_size(nnz)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    nout = C.c_int64()
    _lib.call("jlb_coo_drop_zeros_count", st, dt, base, m, n, nnz, _ptr(rows), _ptr(cols),
              _ptr(val), C.byref(nout), _ptr(ws), ws_bytes)
    r = torch.empty(nout.value, dtype=torch.int32, device=dev)
    c = torch.empty(nout.value, dtype=torch.int32, device=dev)
    v = torch.empty(nout.value, dtype=val.dtype, device=dev)
    _lib.call("jlb_coo_drop_zeros_fill", st, dt, base, m, n, nnz, _ptr(rows), _ptr(cols),
              _ptr(val), nout.value, _ptr(r), _ptr(c), _ptr(v), _ptr(ws), ws_bytes)
    return coo_tensor(r, c, v, (m, n), origin=u.origin)
