"""GPU format conversion: convert_format(u, Formats.BSRRight((b1, b2))) for
CSR and COO sources (src/convert.jl:302-388), and the position-buffer scan
(src/convert.jl:154-168).  Results are bit-identical to the reference's CPU
composer with the block-row level extent ceil(m / b1).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from .backend import _DTYPE, _ptr, _same_device, _stream
from .errors import UnsupportedFormat, UnsupportedValueType
from .formats import TensorFormat
from .tensor import USTensor, bsr_tensor, coordinates, nonzeros, positions


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
    if fmt == u.format:
        return u
    raise UnsupportedFormat(f"convert_format: {u.format.name} -> {fmt.name} is not on B200Backend")
