"""GPU CSR/COO -> BSR conversion and position scans: bit-exact against the
CPU composer restatement (indices, patterns and values)."""
import numpy as np
import pytest
import torch

import jlust_b200 as J
from jlust_b200 import synth
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


def check_csr(m, n, rp, ci, val, b1, b2, base):
    A = J.csr_tensor(to_dev(rp), to_dev(ci), _dev_vals(val), (m, n), origin=base)
    Bt = J.convert_format(A, J.Formats.BSRRight((b1, b2)))
    J.device_status()
    bp, bc, bv = O.csr_to_bsr(m, n, rp, ci, val, b1, b2, base=base)
    assert np.array_equal(_host(J.positions(Bt, 2)), bp)
    assert np.array_equal(_host(J.coordinates(Bt, 2)), bc)
    assert np.array_equal(_host(J.nonzeros(Bt)).view(np.uint8), bv.view(np.uint8))
    assert Bt.origin == A.origin and Bt.extents == (m, n)


def test_fixture(golden):
    g = golden["convert_fixture_3x4"]["A"]
    check_csr(3, 4, np.array(g["rowptr"], np.int32), np.array(g["colind"], np.int32),
              np.array(g["val"], np.float32), 2, 2, 0)


@pytest.mark.parametrize("dtype", [np.float64, np.float32, np.uint16])
@pytest.mark.parametrize("base", [0, 1])
@pytest.mark.parametrize("b1,b2", [(4, 4), (3, 5), (64, 64), (1, 7)])
def test_csr_random(dtype, base, b1, b2):
    rng = np.random.default_rng(61)
    m, n = 301, 257                                    # not multiples of the block size
    rp, ci, val = random_csr(m, n, rng.integers(0, 25, size=m), seed=62, base=base,
                             zero_frac=0.2)
    if dtype == np.uint16:
        val = synth.f32_to_bf16_bits(val.astype(np.float32))
    else:
        val = val.astype(dtype)
    val[::17] = -0.0 if dtype != np.uint16 else np.uint16(0x8000)   # negative zeros drop too
    check_csr(m, n, rp, ci, val, b1, b2, base)


def _dense_tile_csr(m, n, b1, b2, dtype, seed, base):
    """CSR whose rows are mostly whole tile rows of dense blocks (the fill's
    tile-row path), with the cases that leave it: rows thinned inside a block,
    blocks missing from single rows, explicit zeros of both signs, a block
    holding only zeros, rows of odd length (later rows start at odd entries)
    and a partial last block row."""
    rng = np.random.default_rng(seed)
    mb, nb = -(-m // b1), -(-n // b2)
    rows_cols = []
    for I in range(mb):
        blocks = np.sort(rng.choice(nb, size=min(nb, 5), replace=False))
        for i in range(I * b1, min(m, I * b1 + b1)):
            cols = []
            for J_ in blocks:
                c = np.arange(J_ * b2, min(n, J_ * b2 + b2))
                u = rng.random()
                if u < 0.1:
                    continue                                   # block absent from this row
                if u < 0.3:
                    c = np.sort(rng.choice(c, size=rng.integers(1, c.size + 1), replace=False))
                cols.append(c)
            if i % 7 == 3:
                cols.append(np.array([n - 1]))               # odd lengths, ragged starts
            rows_cols.append(np.unique(np.concatenate(cols)) if cols else np.zeros(0, np.int64))
    lens = np.array([c.size for c in rows_cols])
    rp = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    ci = np.concatenate(rows_cols).astype(np.int32)
    val = rng.uniform(0.5, 2.0, size=ci.size) * rng.choice([-1.0, 1.0], size=ci.size)
    if dtype == np.uint16:
        val = synth.f32_to_bf16_bits(val.astype(np.float32))
        neg0, pos0 = np.uint16(0x8000), np.uint16(0)
    else:
        val = val.astype(dtype)
        neg0, pos0 = dtype(-0.0), dtype(0.0)
    val[rng.random(val.size) < 0.03] = neg0
    val[rng.random(val.size) < 0.03] = pos0
    # block row 1: its first block column holds only zeros
    if mb > 1:
        I, J0 = 1, None
        for i in range(b1, min(m, 2 * b1)):
            seg = np.arange(rp[i], rp[i + 1])
            if J0 is None and seg.size:
                J0 = ci[seg[0]] // b2
            if J0 is not None:
                val[seg[ci[seg] // b2 == J0]] = neg0
    return (rp + base).astype(np.int32), (ci + base).astype(np.int32), val


@pytest.mark.parametrize("dtype", [np.float64, np.float32, np.uint16])
@pytest.mark.parametrize("b1,b2", [(64, 64), (8, 8), (3, 5), (16, 32)])
@pytest.mark.parametrize("base", [0, 1])
def test_csr_dense_tile_rows(dtype, b1, b2, base):
    m, n = 5 * b1 - 1, 11 * b2 - 2
    rp, ci, val = _dense_tile_csr(m, n, b1, b2, dtype, 70 + b1, base)
    check_csr(m, n, rp, ci, val, b1, b2, base)


@pytest.mark.parametrize("dtype", [np.float32, np.uint16])
def test_csr_unsorted_rows(dtype):
    """Rows whose columns are not ascending take the entry-by-entry fill; the
    result is the composer's (which sorts)."""
    rng = np.random.default_rng(80)
    m, n, b1, b2 = 200, 300, 16, 16
    rp, ci, val = _dense_tile_csr(m, n, b1, b2, dtype, 81, 0)
    for i in range(0, m, 3):                                # every third row shuffled
        s = slice(rp[i], rp[i + 1])
        perm = rng.permutation(rp[i + 1] - rp[i])
        ci[s], val[s] = ci[s][perm], val[s][perm]
    check_csr(m, n, rp, ci, val, b1, b2, 0)


def test_csr_wide_matrix_windows():
    """More block columns than one shared-memory bitmap window holds."""
    rng = np.random.default_rng(63)
    m, n = 40, 400_000
    rp, ci, val = random_csr(m, n, rng.integers(0, 200, size=m), seed=64)
    check_csr(m, n, rp, ci, val, 2, 1, 0)


def test_config5_round_trip():
    bp, bc, bv, _ = synth.config5(nbr=128)
    rp, ci, vals = synth.bsr_to_csr(bp, bc, bv, 64, 128)
    A = J.csr_tensor(to_dev(rp), to_dev(ci), bf16_dev(vals), (8192, 8192), origin=0)
    Bt = J.convert_format(A, J.Formats.BSRRight((64, 64)))
    J.device_status()
    assert np.array_equal(_host(J.positions(Bt, 2)), bp)
    assert np.array_equal(_host(J.coordinates(Bt, 2)), bc)
    assert np.array_equal(_host(J.nonzeros(Bt)), bv)


@pytest.mark.parametrize("base", [0, 1])
def test_coo_duplicates_and_order(base):
    rng = np.random.default_rng(65)
    m, n, nnz = 200, 150, 6000                          # many duplicate coordinates
    rows = rng.integers(0, m, nnz).astype(np.int32)
    cols = rng.integers(0, n, nnz).astype(np.int32)
    vals = rng.uniform(-1, 1, nnz)
    vals[rng.random(nnz) < 0.1] = 0
    A = J.coo_tensor(to_dev(rows + base), to_dev(cols + base), to_dev(vals), (m, n), origin=base)
    Bt = J.convert_format(A, J.Formats.BSRRight((8, 4)))
    J.device_status()
    bp, bc, bv = O.coo_to_bsr(m, n, rows + base, cols + base, vals, 8, 4, base=base)
    assert np.array_equal(_host(J.positions(Bt, 2)), bp)
    assert np.array_equal(_host(J.coordinates(Bt, 2)), bc)
    assert np.array_equal(_host(J.nonzeros(Bt)), bv)


def test_coo_bounds_error():
    A = J.coo_tensor(to_dev(np.array([0, 9], np.int32)), to_dev(np.array([0, 1], np.int32)),
                     to_dev(np.ones(2)), (4, 4), origin=0)
    with pytest.raises(J.NonCanonicalStorage):
        J.convert_format(A, J.Formats.BSRRight((2, 2)))
    J.device_status()


@pytest.mark.parametrize("n", [0, 1, 2047, 2048, 2049, 4095, 4096, 4097, 3_000_001,
                               16_777_217])
def test_scan(n):
    rng = np.random.default_rng(66)
    c = rng.integers(0, 300 if n < 5_000_000 else 100, size=n).astype(np.int32)
    out = J.exclusive_scan(to_dev(c), base=1)
    J.device_status()
    assert np.array_equal(out.cpu().numpy(), O.exclusive_scan(c, base=1))


def test_empty_matrix():
    A = J.csr_tensor(to_dev(np.zeros(11, np.int32)), to_dev(np.zeros(0, np.int32)),
                     to_dev(np.zeros(0)), (10, 10), origin=0)
    Bt = J.convert_format(A, J.Formats.BSRRight((4, 4)))
    assert _host(J.positions(Bt, 2)).tolist() == [0, 0, 0, 0] and J.nnz(Bt) == 0


def test_distributed_scan_single_process_gpu():
    """jlust_b200.dist.exclusive_scan with one rank runs the library scan on
    the GPU and equals the oracle (the multi-rank offsets are covered on gloo)."""
    from jlust_b200 import dist as D
    counts = np.random.default_rng(61).integers(0, 9, size=300_001).astype(np.int32)
    got = D.exclusive_scan(torch.from_numpy(counts).to(DEV), base=1)
    assert np.array_equal(got.cpu().numpy(), O.exclusive_scan(counts, 1))


@pytest.mark.parametrize("fill_ws", ["same", "fresh", "small"])
def test_csr_fill_workspace_handover(fill_ws):
    """The fill phase reuses the count phase's bitmaps only from the same
    workspace; a fresh (zeroed) workspace or one too small to hold them makes
    it rebuild them -- all three give the oracle's bits."""
    import ctypes as C
    from jlust_b200 import _lib
    rng = np.random.default_rng(65)
    m, n, b1, b2 = 700, 900, 16, 16
    rp, ci, val = random_csr(m, n, rng.integers(0, 40, size=m), seed=66, zero_frac=0.1)
    val = val.astype(np.float32)
    rpd, cid, vd = to_dev(rp), to_dev(ci), to_dev(val)
    mb = -(-m // b1)
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    L = _lib.load()
    wsb = L.jlb_csr_to_bsr_workspace_size(m, n, ci.shape[0], b1, b2)
    ws = torch.zeros(wsb, dtype=torch.uint8, device=DEV)
    browptr = torch.empty(mb + 1, dtype=torch.int32, device=DEV)
    nnzb = C.c_int64()

    def P(t):
        return C.c_void_p(t.data_ptr())

    _lib.call("jlb_csr_to_bsr_count", st, _lib.F32, 0, m, n, ci.shape[0], P(rpd), P(cid), P(vd),
              b1, b2, P(browptr), C.byref(nnzb), P(ws), wsb)
    if fill_ws == "fresh":
        ws = torch.zeros(wsb, dtype=torch.uint8, device=DEV)
    elif fill_ws == "small":
        wsb = 4096
        ws = torch.zeros(wsb, dtype=torch.uint8, device=DEV)
    bcol = torch.empty(nnzb.value, dtype=torch.int32, device=DEV)
    bval = torch.empty(nnzb.value * b1 * b2, dtype=torch.float32, device=DEV)
    _lib.call("jlb_csr_to_bsr_fill", st, _lib.F32, 0, m, n, ci.shape[0], P(rpd), P(cid), P(vd),
              b1, b2, P(browptr), nnzb.value, P(bcol), P(bval), P(ws), wsb)
    J.device_status()
    bp, bc, bv = O.csr_to_bsr(m, n, rp, ci, val, b1, b2)
    assert np.array_equal(browptr.cpu().numpy(), bp)
    assert np.array_equal(bcol.cpu().numpy(), bc)
    assert np.array_equal(bval.cpu().numpy().view(np.uint8), bv.view(np.uint8))


def test_scan_in_place_shifted():
    """counts given as out + 1 (the row-pointer layout the conversions use):
    each tile reads only the counts whose outputs it writes."""
    import ctypes as C

    from jlust_b200 import _lib
    from jlust_b200.backend import _stream
    rng = np.random.default_rng(67)
    n = 1_000_003
    c = rng.integers(0, 50, size=n).astype(np.int32)
    buf = torch.zeros(n + 1, dtype=torch.int32, device=DEV)
    buf[1:] = to_dev(c)
    L = _lib.load()
    wsb = L.jlb_scan_workspace_size(n)
    ws = torch.empty(wsb, dtype=torch.uint8, device=DEV)
    _lib.call("jlb_exclusive_scan_i32", _stream(torch.device(DEV)), n,
              C.c_void_p(buf.data_ptr() + 4), C.c_void_p(buf.data_ptr()), 0,
              C.c_void_p(ws.data_ptr()), wsb)
    J.device_status()
    assert np.array_equal(buf.cpu().numpy(), O.exclusive_scan(c))


def test_scan_total_past_int32_reported():
    """A running total past Int32 cannot be a position: the scan flags it and
    jlb_device_status reports it; the context stays usable."""
    c = np.full(3_000_000, 1000, np.int32)          # 3e9 in all
    J.exclusive_scan(to_dev(c))
    with pytest.raises(J.NonCanonicalStorage):
        J.device_status()
    out = J.exclusive_scan(to_dev(np.ones(10, np.int32)))
    J.device_status()
    assert out.cpu().tolist() == list(range(11))


@pytest.mark.parametrize("n", [3 * 4096, 3 * 4096 + 5])
@pytest.mark.parametrize("shift", [0, 1])
def test_scan_aligned_and_unaligned_buffers(n, shift):
    """Separate, 16-byte-aligned counts and output take the vector final pass
    (tile t writes out[t0 ..] with 16-byte stores, the last tile out[n]);
    buffers one element off a 16-byte boundary take the scalar pass; a whole
    number of tiles and a ragged last tile."""
    import ctypes as C

    from jlust_b200 import _lib
    from jlust_b200.backend import _stream
    rng = np.random.default_rng(68 + n + shift)
    c = rng.integers(0, 1000, size=n).astype(np.int32)
    cbuf = torch.zeros(n + 4, dtype=torch.int32, device=DEV)
    obuf = torch.full((n + 5,), -7, dtype=torch.int32, device=DEV)
    counts, out = cbuf[shift:shift + n], obuf[shift:shift + n + 1]
    counts.copy_(to_dev(c))
    L = _lib.load()
    wsb = L.jlb_scan_workspace_size(n)
    ws = torch.empty(wsb, dtype=torch.uint8, device=DEV)
    _lib.check(L.jlb_exclusive_scan_i32(_stream(DEV), n, C.c_void_p(counts.data_ptr()),
                                        C.c_void_p(out.data_ptr()), 1, C.c_void_p(ws.data_ptr()),
                                        wsb))
    J.device_status()
    assert np.array_equal(out.cpu().numpy(), O.exclusive_scan(c, base=1))
    assert int(obuf[shift + n + 1:].eq(-7).all()) and (shift == 0 or int(obuf[0]) == -7)
