"""ctypes binding of libjlust_b200.so (declarations mirror include/jlust_b200.h).

The library is loaded from jlust_b200/_lib/libjlust_b200.so, built in-tree by
`python -m jlust_b200.build`.  There is no fallback: if the library is missing
every operation raises, so a GPU run can never silently use another path.
"""
from __future__ import annotations

import ctypes as C
import os
import re

from . import errors

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libjlust_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "jlust_b200.h")

# enums (include/jlust_b200.h)
F32, F64, BF16 = 0, 1, 2
ROW_MAJOR, COL_MAJOR = 0, 1
SDDMM_ADD, SDDMM_MUL = 0, 1

_p, _i, _i64, _d, _sz = C.c_void_p, C.c_int, C.c_int64, C.c_double, C.c_size_t
_pi64 = C.POINTER(C.c_int64)

# name -> (restype, argtypes)
SIGNATURES = {
    "jlb_version": (_i, []),
    "jlb_status_string": (C.c_char_p, [_i]),
    "jlb_last_error": (_i, [C.c_char_p, _sz]),
    "jlb_init": (_i, [_i]),
    "jlb_device_status": (_i, [_p]),
    "jlb_csr_validate": (_i, [_p, _i, _i64, _i64, _i64, _p, _p, _i]),
    "jlb_csr_spmv": (_i, [_p, _i, _i, _i64, _i64, _i64, _p, _p, _p, _p, _p, _d, _d]),
    "jlb_dcsr_spmv": (_i, [_p, _i, _i, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _d, _d]),
    "jlb_coo_spmv": (_i, [_p, _i, _i, _i64, _i64, _i64, _p, _p, _p, _p, _p, _d, _d]),
    "jlb_csc_spmv": (_i, [_p, _i, _i, _i64, _i64, _i64, _p, _p, _p, _p, _p, _d, _d]),
    "jlb_csr_patched_spmv": (_i, [_p, _i, _i, _i64, _i64, _i64, _p, _p, _p, _i, _p, _p, _p, _p, _p, _d, _d]),
    "jlb_bbm_periodic_spmv": (_i, [_p, _i, _i, _i64, _i64, _i64, _i64, _p, _p, _p, _i, _p, _p, _p,
                                    _p, _p, _p, _i64, _d, _p, _p, _p, _i64, _d, _p, _p, _d, _d]),
    "jlb_spmv_plan_create": (_i, [C.POINTER(_p), _p, _i, _i, _i64, _i64, _i64, _p, _p]),
    "jlb_spmv_plan_execute": (_i, [_p, _p, _p, _p, _p, _d, _d]),
    "jlb_spmv_plan_info": (_i, [_p, _pi64, C.POINTER(_d), C.POINTER(_i)]),
    "jlb_spmv_plan_destroy": (_i, [_p]),
    "jlb_spmv_plan_set_variant": (_i, [_p, _i]),
    "jlb_csr_spmm": (_i, [_p, _i, _i, _i64, _i64, _i64, _p, _p, _p, _i64, _p, _i64, _i, _p,
                          _i64, _i, _d, _d]),
    "jlb_csr_spmm_workspace_size": (_sz, [_i, _i64, _i64, _i64, _i, _i]),
    "jlb_csr_spmm_ws": (_i, [_p, _i, _i, _i64, _i64, _i64, _p, _p, _p, _i64, _p, _i64, _i, _p,
                             _i64, _i, _d, _d, _p, _sz]),
    "jlb_sddmm": (_i, [_p, _i, _i, _i64, _i64, _i64, _p, _p, _i64, _p, _i64, _i, _p, _i64, _i,
                       _p, _p, _i, _d, _d]),
    "jlb_bsr_spmm": (_i, [_p, _i, _i64, _i64, _i64, _i, _p, _p, _p, _i64, _p, _i64, _p, _i64,
                          _d, _d]),
    "jlb_scan_workspace_size": (_sz, [_i64]),
    "jlb_exclusive_scan_i32": (_i, [_p, _i64, _p, _p, _i, _p, _sz]),
    "jlb_exclusive_scan_i32_noalloc": (_i, [_p, _i64, _p, _p, _i]),
    "jlb_csr_to_bsr_workspace_size": (_sz, [_i64, _i64, _i64, _i, _i]),
    "jlb_csr_to_bsr_count": (_i, [_p, _i, _i, _i64, _i64, _i64, _p, _p, _p, _i, _i, _p, _pi64,
                                  _p, _sz]),
    "jlb_csr_to_bsr_fill": (_i, [_p, _i, _i, _i64, _i64, _i64, _p, _p, _p, _i, _i, _p, _i64, _p,
                                 _p, _p, _sz]),
    "jlb_coo_to_bsr_workspace_size": (_sz, [_i64, _i64, _i64, _i, _i, _i64]),
    "jlb_coo_to_bsr_count": (_i, [_p, _i, _i, _i64, _i64, _i64, _p, _p, _p, _i, _i, _p, _pi64,
                                  _p, _sz]),
    "jlb_coo_to_bsr_fill": (_i, [_p, _i, _i, _i64, _i64, _i64, _p, _p, _p, _i, _i, _p, _i64, _p,
                                 _p, _p, _sz]),
    "jlb_spgemm_plan_create": (_i, [C.POINTER(_p), _p, _i, _i, _i64, _i64, _i64, _i64, _p, _p,
                                    _i64, _p, _p, _pi64, _pi64]),
    "jlb_spgemm_plan_structure": (_i, [_p, _p, _p, _p]),
    "jlb_spgemm_plan_execute": (_i, [_p, _p, _p, _p, _p, _d]),
    "jlb_spgemm_plan_destroy": (_i, [_p]),
    "jlb_coo_drop_zeros_workspace_size": (_sz, [_i64]),
    "jlb_coo_drop_zeros_count": (_i, [_p, _i, _i, _i64, _i64, _i64, _p, _p, _p, _pi64, _p, _sz]),
    "jlb_coo_drop_zeros_fill": (_i, [_p, _i, _i, _i64, _i64, _i64, _p, _p, _p, _i64, _p, _p, _p,
                                     _p, _sz]),
    "jlb_coo_to_csr_workspace_size": (_sz, [_i64, _i64, _i64]),
    "jlb_coo_to_csr_count": (_i, [_p, _i, _i, _i64, _i64, _i64, _p, _p, _p, _p, _pi64, _p, _sz]),
    "jlb_coo_to_csr_fill": (_i, [_p, _i, _i, _i64, _i64, _i64, _p, _p, _p, _i64, _p, _p, _p,
                                 _sz]),
    "jlb_sorted_compress_workspace_size": (_sz, [_i64, _i64]),
    "jlb_sorted_compress_count": (_i, [_p, _i, _i, _i64, _i64, _i64, _p, _p, _p, _p, _pi64, _p,
                                       _sz]),
    "jlb_sorted_compress_fill": (_i, [_p, _i, _i, _i64, _i64, _i64, _p, _p, _p, _p, _i64, _p, _p,
                                      _p, _sz]),
    "jlb_positions_to_coordinates": (_i, [_p, _i, _i64, _i64, _p, _p]),
    "jlb_halo_spmv_steps": (_i, [_p, _i, _i, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p,
                                 _p, _p, _i, _i, C.c_uint64]),
    "jlb_ipc_handle": (_i, [_p, _p, C.POINTER(C.c_uint64)]),
    "jlb_ipc_open": (_i, [_p, C.POINTER(_p)]),
    "jlb_ipc_close": (_i, [_p]),
    "jlb_l2_persist": (_i, [_p, _p, _sz, C.POINTER(_sz)]),
}

_lib = None


def header_symbols() -> list[str]:
    """Every entry point declared with JLB_API in include/jlust_b200.h."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"JLB_API\s+[\w\s\*]*?\b(jlb_\w+)\s*\(", text)))


def load(path: str = LIB_PATH):
    """Load the library (once) and declare every signature."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise errors.CudaError(
                f"libjlust_b200.so is not built ({path}); run `python -m jlust_b200.build`")
        lib = C.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def last_error() -> str:
    buf = C.create_string_buffer(512)
    load().jlb_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int, what: str = "") -> None:
    """Raise the JLUST exception that a nonzero status maps to."""
    if status != 0:
        msg = last_error()
        raise errors.from_status(status, f"{what}: {msg}" if what else msg)


def call(name: str, *args):
    st = getattr(load(), name)(*args)
    check(st, name)
    return st
