"""GPU conversions to CSR and CSC (convert_format with Formats.CSR /
Formats.CSC) against the oracle's restatement of the reference's composer:
bit-exact positions, coordinates and values.  COO -> CSR and CSR -> CSR keep
storage order (a stable compaction: explicit zeros dropped, adjacent equal
coordinates merged keeping the first value); CSC targets and CSC -> CSR are
lexsorted by (outer, inner, storage index), which on the device is a per
bucket bitonic sort (one warp up to 256 entries, one CTA in shared memory up
to 16,384, one CTA in global memory beyond)."""
import numpy as np
import pytest
import torch

import jlust_b200 as J
from oracle import oracle as O
from _helpers import DEV, bf16_dev, random_csr, to_dev

pytestmark = pytest.mark.gpu


def _host(t):
    t = t.cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def _dev_vals(v):
    return bf16_dev(v) if v.dtype == np.uint16 else to_dev(v)


def _vals(rng, k, dtype, zero_frac=0.1):
    v = rng.uniform(-1, 1, k)
    v[rng.random(k) < zero_frac] = 0.0
    if dtype == np.uint16:
        return (v.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    return v.astype(dtype)


def _same(got, ref):
    assert np.array_equal(_host(J.positions(got, 2)), ref[0])
    assert np.array_equal(_host(J.coordinates(got, 2)), ref[1])
    assert np.array_equal(_host(J.nonzeros(got)).view(np.uint8), np.asarray(ref[2]).view(np.uint8))


def _coo(m, n, rows, cols, val, base):
    return J.coo_tensor(to_dev((rows + base).astype(np.int32)), to_dev((cols + base).astype(np.int32)),
                        _dev_vals(val), (m, n), origin=base)


def test_fixture_kats(golden):
    g = golden["convert_fixture_3x4"]
    a = g["A"]
    rp, ci = np.array(a["rowptr"], np.int32), np.array(a["colind"], np.int32)
    v = np.array(a["val"], np.float32)
    A = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(v), (3, 4), origin=0)
    Cc = J.convert_format(A, J.Formats.CSC)
    J.device_status()
    assert Cc.format == J.Formats.CSC
    assert _host(J.positions(Cc, 2)).tolist() == g["csc"]["colptr"]
    assert _host(J.coordinates(Cc, 2)).tolist() == g["csc"]["rowind"]
    assert _host(J.nonzeros(Cc)).tolist() == g["csc"]["val"]
    back = J.convert_format(Cc, J.Formats.CSR)
    J.device_status()
    _same(back, (rp, ci, v))
    same = J.convert_format(A, J.Formats.CSR)
    _same(same, (rp, ci, v))
    A1 = J.csr_tensor(to_dev(rp + 1), to_dev(ci + 1), to_dev(v), (3, 4), origin=1)
    C1 = J.convert_format(A1, J.Formats.CSC)
    assert C1.origin == A1.origin
    assert _host(J.positions(C1, 2)).tolist() == [x + 1 for x in g["csc"]["colptr"]]


@pytest.mark.parametrize("dtype", [np.float64, np.float32, np.uint16])
@pytest.mark.parametrize("base", [0, 1])
def test_coo_to_csr_stable_compaction(dtype, base):
    """Row-ordered COO with unsorted columns, runs of duplicates, explicit
    zeros (also between duplicates) and empty rows."""
    rng = np.random.default_rng(200)
    m, n = 6000, 5000
    lens = rng.integers(0, 40, m)
    lens[rng.random(m) < 0.2] = 0
    rows = np.repeat(np.arange(m), lens)
    cols = rng.integers(0, 60, rows.shape[0])      # narrow: many equal neighbours
    dup = rng.random(rows.shape[0]) < 0.3
    cols[1:][dup[1:] & (rows[1:] == rows[:-1])] = cols[:-1][dup[1:] & (rows[1:] == rows[:-1])]
    val = _vals(rng, rows.shape[0], dtype, 0.15)
    U = J.convert_format(_coo(m, n, rows, cols, val, base), J.Formats.CSR)
    J.device_status()
    ref = O.coo_to_csr(m, n, rows + base, cols + base, val, base)
    _same(U, ref)
    assert U.origin.offset == base


@pytest.mark.parametrize("dtype", [np.float64, np.float32, np.uint16])
@pytest.mark.parametrize("offset", [0, 1])
def test_coo_to_csr_vector_and_scalar_keep(dtype, offset):
    """The keep pass takes four entries a thread when the COO arrays are
    16-byte aligned and one entry otherwise (offset 1: views one element
    in).  Dense rows and rows spread wider than a tile's 4096-row window,
    zero runs across lanes, warps and a tile boundary with equal coordinates
    on either side (merged across the zeros), and a ragged last tile."""
    rng = np.random.default_rng(207 + offset)
    m, n, k = 3_000_000, 50, 3 * 4096 + 1237
    dense = np.sort(rng.integers(100, 100 + k // 8, k // 2))
    rows = np.sort(np.concatenate([dense, rng.integers(0, m, k - k // 2)]))
    cols = rng.integers(0, n, k)
    val = _vals(rng, k, dtype, 0.05)
    nz = np.uint16(0x3f80) if dtype == np.uint16 else dtype(1.5)
    for a, b in ((4089, 4101), (4999, 5301), (127, 131), (8190, 8195)):
        rows[a:b + 1] = rows[a]
        cols[b] = cols[a]
        val[a + 1:b] = 0
        val[a] = val[b] = nz
    rows = np.maximum.accumulate(rows)

    def dev(x):
        t = _dev_vals(np.concatenate([x[:1], x])) if offset else _dev_vals(x)
        return t[offset:]
    A = J.coo_tensor(dev((rows + 1).astype(np.int32)), dev((cols + 1).astype(np.int32)), dev(val),
                     (m, n), origin=1)
    U = J.convert_format(A, J.Formats.CSR)
    J.device_status()
    _same(U, O.coo_to_csr(m, n, rows + 1, cols + 1, val, 1))


def test_coo_to_csr_rejects_decreasing_rows():
    A = _coo(4, 4, np.array([0, 2, 1]), np.array([0, 0, 0]), np.ones(3), 0)
    with pytest.raises(J.NonCanonicalStorage):
        J.convert_format(A, J.Formats.CSR)


@pytest.mark.parametrize("dtype", [np.float64, np.uint16])
def test_csr_to_csr_drops_zeros(dtype):
    rng = np.random.default_rng(201)
    m, n = 3000, 4000
    rp, ci, v = random_csr(m, n, rng.integers(0, 30, m), seed=202, dtype=np.float64)
    val = _vals(rng, v.shape[0], dtype, 0.2)
    A = J.csr_tensor(to_dev(rp), to_dev(ci), _dev_vals(val), (m, n), origin=0)
    U = J.convert_format(A, J.Formats.CSR)
    J.device_status()
    _same(U, O.csr_to_csr(m, n, rp, ci, val, 0))


@pytest.mark.parametrize("dtype", [np.float64, np.float32, np.uint16])
@pytest.mark.parametrize("base", [0, 1])
def test_coo_to_csc_sorted(dtype, base):
    """Unordered COO with duplicates to CSC: columns from empty to ~110,000
    entries (all three sorts), bit-exact with the stable lexsort."""
    rng = np.random.default_rng(203)
    m, n, nnz = 20000, 3000, 250000
    rows = rng.integers(0, m, nnz)
    cols = (rng.zipf(1.6, nnz) - 1) % n            # a few heavy columns
    rows[rng.random(nnz) < 0.05] = 7               # duplicates in row 7
    val = _vals(rng, nnz, dtype, 0.05)
    C = J.convert_format(_coo(m, n, rows, cols, val, base), J.Formats.CSC)
    J.device_status()
    _same(C, O.coo_to_csc(m, n, rows + base, cols + base, val, base))


def test_csr_csc_round_trip_long_columns():
    """CSR -> CSC with columns of up to ~40,000 entries (the global-memory
    sort) and back to CSR."""
    rng = np.random.default_rng(204)
    m, n = 60000, 2000
    lens = rng.integers(1, 8, m)
    rp = np.zeros(m + 1, np.int64)
    np.cumsum(lens, out=rp[1:])
    ci = np.empty(rp[-1], np.int64)
    for r in range(m):     # column 0 and 5 in most rows: long columns
        c = rng.choice(n - 10, lens[r], replace=False) + 10
        c[0] = 0
        if lens[r] > 1:
            c[1] = 5
        ci[rp[r]:rp[r + 1]] = np.sort(c)
    rp, ci = rp.astype(np.int32), ci.astype(np.int32)
    v = rng.uniform(-1, 1, rp[-1])
    A = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(v), (m, n), origin=0)
    C = J.convert_format(A, J.Formats.CSC)
    J.device_status()
    ref = O.csr_to_csc(m, n, rp, ci, v, 0)
    assert np.diff(ref[0]).max() > 16384
    _same(C, ref)
    B = J.convert_format(C, J.Formats.CSR)
    J.device_status()
    _same(B, O.csc_to_csr(m, n, *ref, 0))
    _same(B, (rp, ci, v))


def test_sorted_fill_needs_count_workspace():
    import ctypes as C

    from jlust_b200 import _lib
    from jlust_b200.backend import _DTYPE, _stream
    from jlust_b200.errors import JLUSTError
    rows = to_dev(np.array([0, 1], np.int32))
    cols = to_dev(np.array([1, 0], np.int32))
    val = to_dev(np.ones(2))
    L = _lib.load()
    wsb = L.jlb_sorted_compress_workspace_size(2, 2)
    ws = torch.zeros(wsb, dtype=torch.uint8, device=DEV)
    ptr = torch.empty(3, dtype=torch.int32, device=DEV)
    out_i = torch.empty(2, dtype=torch.int32, device=DEV)
    out_v = torch.empty(2, dtype=torch.float64, device=DEV)

    def p(t):
        return C.c_void_p(t.data_ptr())
    with pytest.raises(JLUSTError, match="workspace its count phase filled"):
        _lib.call("jlb_sorted_compress_fill", _stream(torch.device(DEV)), _DTYPE[torch.float64],
                  0, 2, 2, 2, p(cols),
                  p(rows), p(val), p(ptr), 2, p(out_i), p(out_v), p(ws), wsb)


@pytest.mark.parametrize("same_ws", [True, False])
def test_coo_to_csr_fill_workspace(same_ws):
    """Fill reuses the flags count stamped into its workspace; a fresh
    workspace makes it recompute them, with the same result."""
    import ctypes as C

    from jlust_b200 import _lib
    from jlust_b200.backend import _DTYPE, _stream
    rng = np.random.default_rng(205)
    m, n = 4000, 3000
    rows = np.sort(rng.integers(0, m, 60000))
    cols = rng.integers(0, 40, rows.shape[0])
    val = _vals(rng, rows.shape[0], np.float64, 0.1)
    r_d, c_d, v_d = to_dev(rows.astype(np.int32)), to_dev(cols.astype(np.int32)), to_dev(val)
    L = _lib.load()
    wsb = L.jlb_coo_to_csr_workspace_size(m, n, rows.shape[0])
    ws = torch.empty(wsb, dtype=torch.uint8, device=DEV)
    rowptr = torch.empty(m + 1, dtype=torch.int32, device=DEV)
    st = _stream(torch.device(DEV))

    def p(t):
        return C.c_void_p(t.data_ptr())
    nout = C.c_int64()
    dt = _DTYPE[torch.float64]
    _lib.call("jlb_coo_to_csr_count", st, dt, 0, m, n, rows.shape[0], p(r_d), p(c_d), p(v_d),
              p(rowptr), C.byref(nout), p(ws), wsb)
    ws2 = ws if same_ws else torch.zeros(wsb, dtype=torch.uint8, device=DEV)
    ci = torch.empty(nout.value, dtype=torch.int32, device=DEV)
    vo = torch.empty(nout.value, dtype=torch.float64, device=DEV)
    _lib.call("jlb_coo_to_csr_fill", st, dt, 0, m, n, rows.shape[0], p(r_d), p(c_d), p(v_d),
              nout.value, p(ci), p(vo), p(ws2), wsb)
    J.device_status()
    ref = O.coo_to_csr(m, n, rows, cols, val, 0)
    assert np.array_equal(rowptr.cpu().numpy(), ref[0])
    assert np.array_equal(ci.cpu().numpy(), ref[1])
    assert np.array_equal(vo.cpu().numpy(), ref[2])


def test_csr_to_coo_kat_and_round_trip(golden):
    g = golden["convert_fixture_3x4"]
    a = g["A"]
    rp, ci = np.array(a["rowptr"], np.int32), np.array(a["colind"], np.int32)
    v = np.array(a["val"], np.float32)
    A = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(v), (3, 4), origin=0)
    U = J.convert_format(A, J.Formats.COO)
    J.device_status()
    assert U.format == J.Formats.COO
    assert _host(J.coordinates(U, 1)).tolist() == [0, 0, 1, 2, 2]
    assert _host(J.coordinates(U, 2)).tolist() == [0, 2, 1, 0, 2]
    assert _host(J.nonzeros(U)).tolist() == [1, 2, 3, 4, 5]
    _same(J.convert_format(U, J.Formats.CSR), (rp, ci, v))


@pytest.mark.parametrize("dtype", [np.float64, np.uint16])
def test_to_coo_drops_zeros(dtype):
    rng = np.random.default_rng(206)
    m, n = 3000, 2000
    rp, ci, _ = random_csr(m, n, rng.integers(0, 25, m), seed=207, base=1)
    val = _vals(rng, ci.shape[0], dtype, 0.3)
    A = J.csr_tensor(to_dev(rp), to_dev(ci), _dev_vals(val), (m, n), origin=1)
    U = J.convert_format(A, J.Formats.COO)
    J.device_status()
    r, c, vv = O.to_coo(O.expand_positions(rp, 1), ci, val)
    assert np.array_equal(_host(J.coordinates(U, 1)), r)
    assert np.array_equal(_host(J.coordinates(U, 2)), c)
    assert np.array_equal(_host(J.nonzeros(U)).view(np.uint8), vv.view(np.uint8))
    # COO -> COO of an unordered COO only drops zeros too
    p = rng.permutation(r.shape[0])
    vz = vv[p].copy()
    vz[::7] = 0
    U2 = J.convert_format(J.coo_tensor(to_dev(r[p]), to_dev(c[p]), _dev_vals(vz), (m, n), origin=1),
                          J.Formats.COO)
    r2, c2, v2 = O.to_coo(r[p], c[p], vz)
    assert np.array_equal(_host(J.coordinates(U2, 1)), r2)
    assert np.array_equal(_host(J.nonzeros(U2)).view(np.uint8), v2.view(np.uint8))
