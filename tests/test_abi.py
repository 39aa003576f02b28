"""The C ABI library loads without a GPU, exports every symbol the header
declares, and rejects bad arguments with the documented status codes before
touching a device."""
import ctypes as C
import subprocess

import pytest

from jlust_b200 import _lib, errors


def test_header_symbols_exported():
    L = _lib.load()
    syms = _lib.header_symbols()
    assert len(syms) >= 20
    for s in syms:
        assert hasattr(L, s), f"{s} declared in include/jlust_b200.h but not exported"
    assert set(_lib.SIGNATURES) == set(syms), "ctypes table out of sync with the header"


def test_dynamic_symbol_table_has_only_the_abi():
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    jlb = {s for s in exported if s.startswith("jlb_")}
    assert jlb == set(_lib.header_symbols())


def test_version_and_status_strings():
    L = _lib.load()
    assert L.jlb_version() >= 100
    assert L.jlb_status_string(7) == b"NonCanonicalStorage"
    assert L.jlb_status_string(1) == b"UnsupportedFormat"


@pytest.mark.parametrize("args,status", [
    # bad dtype -> UnsupportedValueType
    ((None, 2, 0, 3, 3, 5, None, None, None, None, None, 1.0, 0.0), 3),
    # bad origin -> InvalidArgument
    ((None, 1, 7, 3, 3, 5, None, None, None, None, None, 1.0, 0.0), 8),
    # negative extent -> IncompatibleExtents
    ((None, 1, 0, -1, 3, 5, None, None, None, None, None, 1.0, 0.0), 6),
    # null buffers with work to do -> InvalidArgument
    ((None, 1, 0, 3, 3, 5, None, None, None, None, None, 1.0, 0.0), 8),
])
def test_spmv_argument_errors(args, status):
    L = _lib.load()
    st = L.jlb_csr_spmv(*args)
    assert st == status
    buf = C.create_string_buffer(256)
    assert L.jlb_last_error(buf, 256) == status
    assert len(buf.value) > 0
    with pytest.raises(errors.JLUSTError):
        _lib.check(st)


def test_error_classes_map_statuses():
    assert isinstance(errors.from_status(7, "x"), errors.NonCanonicalStorage)
    assert isinstance(errors.from_status(3, "x"), errors.UnsupportedValueType)
    assert isinstance(errors.from_status(10, "x"), errors.DeviceTimeout)


def test_workspace_queries_are_host_only():
    L = _lib.load()
    assert L.jlb_scan_workspace_size(0) > 0
    assert L.jlb_scan_workspace_size(10_000_000) >= 8 * (10_000_000 // 4096)   # one int64 per tile
    assert L.jlb_coo_to_bsr_workspace_size(100, 100, 1000, 4, 4, 10) > \
        L.jlb_coo_to_bsr_workspace_size(100, 100, 1000, 4, 4, 0)
