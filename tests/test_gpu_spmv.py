"""CSR SpMV on the GPU against the CPU oracle: bit-exact for rows of up to 32
entries (same operations in the same order), within tolerance for longer rows."""
import numpy as np
import pytest
import torch

import jlust_b200 as J
from jlust_b200 import synth
from oracle import oracle as O
from _helpers import DEV, assert_within, random_csr, to_dev

pytestmark = pytest.mark.gpu
TOL = {np.float64: 1e-12, np.float32: 1e-5}


def run_spmv(rp, ci, val, x, m, n, base, y0=None, alpha=1.0, beta=0.0, prepared=False):
    A = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(val), (m, n), origin=base)
    xd = to_dev(x)
    yd = to_dev(y0) if y0 is not None else torch.zeros(m, dtype=xd.dtype, device=DEV)
    if prepared:
        h = J.prepare(J.B200Backend(), J.SpMVOp, A)
        J.execute(J.SpMVOp, h, xd, yd, alpha=alpha, beta=beta)
    else:
        J.execute(J.SpMVOp, A, xd, yd, alpha=alpha, beta=beta)
    J.device_status()
    return yd.cpu().numpy()


def test_kat(golden):
    for name in ("spmv_csr_onebased", "spmv_csr_zerobased"):
        g = golden[name]
        A = g["A"]
        y = run_spmv(np.array(A["rowptr"], np.int32), np.array(A["colind"], np.int32),
                     np.array(A["val"]), np.array(g["x"]), 3, 3, A["base"])
        assert y.tolist() == g["y"]


@pytest.mark.parametrize("dtype", [np.float64, np.float32])
@pytest.mark.parametrize("base", [0, 1])
@pytest.mark.parametrize("ab", [(1.0, 0.0), (0.5, 0.0), (-1.5, 2.0), (1.0, 1.0)])
def test_short_rows_bit_exact(dtype, base, ab):
    rng = np.random.default_rng(11)
    m, n = 5000, 3000
    lengths = rng.integers(0, 33, size=m)
    lengths[::97] = 0                                  # empty rows
    rp, ci, val = random_csr(m, n, lengths, seed=12, base=base, dtype=dtype)
    x = rng.uniform(-1, 1, n).astype(dtype)
    y0 = rng.uniform(-1, 1, m).astype(dtype)
    alpha, beta = ab
    got = run_spmv(rp, ci, val, x, m, n, base, y0, alpha, beta)
    ref = O.spmv(rp, ci, val, x, y0, alpha, beta, base)
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("dtype", [np.float64, np.float32])
def test_long_rows_within_tolerance(dtype):
    rng = np.random.default_rng(13)
    m, n = 3000, 20000
    lengths = rng.integers(0, 20, size=m)
    lengths[::50] = rng.integers(33, 3000, size=lengths[::50].shape[0])   # warp rows
    lengths[7] = 12000                                                      # unstaged tile
    rp, ci, val = random_csr(m, n, lengths, seed=14, dtype=dtype)
    x = rng.uniform(-1, 1, n).astype(dtype)
    got = run_spmv(rp, ci, val, x, m, n, 0, alpha=2.0)
    ref, bound = O.spmv_ref64(rp, ci, val, x, alpha=2.0)
    assert_within(got, ref, bound, TOL[dtype])
    # rows of up to 32 entries are summed by one thread in storage order
    short = np.diff(rp) <= 32
    exact = O.spmv(rp, ci, val, x, alpha=2.0)
    assert np.array_equal(got[short], exact[short])


def test_prepared_handle_and_update_values():
    rp, ci, val, x = synth.config1(seed=21, n=20000, k=10)
    A = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(val), (20000, 20000), origin=0)
    h = J.prepare(J.B200Backend(), J.SpMVOp, A)
    info = h.info()
    assert info["max_row"] == 10 and info["variant"] == 0
    y = torch.zeros(20000, dtype=torch.float64, device=DEV)
    J.execute(J.SpMVOp, h, to_dev(x), y)
    assert np.array_equal(y.cpu().numpy(), O.spmv(rp, ci, val, x))
    val2 = val * 3
    J.update_values(h, J.csr_tensor(A.pos[1], A.crd[1], to_dev(val2), (20000, 20000), origin=0))
    J.execute(h, to_dev(x), y)
    assert np.array_equal(y.cpu().numpy(), O.spmv(rp, ci, val2, x))


def test_validation_rejects_noncanonical():
    rp = np.array([0, 2, 1, 3], np.int32)       # decreasing row pointer
    ci = np.array([0, 1, 2], np.int32)
    A = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(np.ones(3)), (3, 3), origin=0)
    with pytest.raises(J.NonCanonicalStorage):
        J.validate_storage(A)
    with pytest.raises(J.NonCanonicalStorage):
        J.prepare(J.B200Backend(), J.SpMVOp, A)
    ci_bad = np.array([0, 5, 2], np.int32)      # column out of range
    A2 = J.csr_tensor(to_dev(np.array([0, 2, 2, 3], np.int32)), to_dev(ci_bad),
                      to_dev(np.ones(3)), (3, 3), origin=0)
    with pytest.raises(J.NonCanonicalStorage):
        J.validate_storage(A2)
    J.validate_storage(J.csr_tensor(to_dev(np.array([0, 2, 2, 3], np.int32)),
                                    to_dev(np.array([0, 2, 1], np.int32)), to_dev(np.ones(3)),
                                    (3, 3), origin=0))


def test_empty_and_degenerate():
    # m = 0
    got = run_spmv(np.array([0], np.int32), np.zeros(0, np.int32), np.zeros(0), np.ones(4), 0, 4, 0)
    assert got.shape == (0,)
    # nnz = 0 with beta
    y0 = np.arange(5, dtype=np.float64)
    got = run_spmv(np.zeros(6, np.int32), np.zeros(0, np.int32), np.zeros(0), np.ones(3), 5, 3, 0,
                   y0, 1.0, 2.0)
    assert got.tolist() == (2 * y0).tolist()


def test_config1_full_size_bit_exact():
    rp, ci, val, x = synth.config1()
    got = run_spmv(rp, ci, val, x, 100_000, 100_000, 0)
    assert np.array_equal(got, O.spmv(rp, ci, val, x))


def test_laplacian_iterations_bit_exact():
    """20 iterations x <- A x on a 1024^2 grid stay bit-identical to the oracle."""
    rp, ci, val, x = synth.config2(g=1024)
    n = 1024 * 1024
    A = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(val), (n, n), origin=0)
    xa, xb = to_dev(x), torch.empty(n, dtype=torch.float64, device=DEV)
    xr = x.copy()
    for _ in range(20):
        J.execute(J.SpMVOp, A, xa, xb)
        xa, xb = xb, xa
        xr = O.spmv(rp, ci, val, xr)
    J.device_status()
    assert np.array_equal(xa.cpu().numpy(), xr)


def test_l2_persisting_window_same_results():
    """Iterations under a persisting L2 window over the matrix (jlb_l2_persist)
    give the same bits as without it; clearing the window releases the
    set-aside."""
    rp, ci, val, x = synth.config2(g=1024)
    n = 1024 * 1024
    A = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(val), (n, n), origin=0)
    persisted = J.l2_persist(A.val, val.nbytes)
    assert persisted > 0
    try:
        xa, xb = to_dev(x), torch.empty(n, dtype=torch.float64, device=DEV)
        xr = x.copy()
        for _ in range(10):
            J.execute(J.SpMVOp, A, xa, xb)
            xa, xb = xb, xa
            xr = O.spmv(rp, ci, val, xr)
        J.device_status()
        assert np.array_equal(xa.cpu().numpy(), xr)
    finally:
        assert J.l2_persist(0, 0) == 0


def test_row_range_views_match_whole():
    """SpMV through row-range views of one CSR (row pointer slices over the
    same columns and values, as a chunked pipeline uses them) gives the same
    bits as the whole matrix."""
    rp, ci, val, x = synth.config2(g=512)
    n = 512 * 512
    rpd, cid, vd, xd = to_dev(rp), to_dev(ci), to_dev(val), to_dev(x)
    whole = torch.empty(n, dtype=torch.float64, device=DEV)
    J.execute(J.SpMVOp, J.csr_tensor(rpd, cid, vd, (n, n), origin=0), xd, whole)
    parts = torch.empty(n, dtype=torch.float64, device=DEV)
    b = [n * c // 7 for c in range(8)]
    for lo, hi in zip(b[:-1], b[1:]):
        J.execute(J.SpMVOp, J.csr_tensor(rpd[lo:hi + 1], cid, vd, (hi - lo, n), origin=0), xd,
                  parts[lo:hi])
    J.device_status()
    assert torch.equal(whole, parts)


@pytest.mark.parametrize("variant", [2, 4, 8, 16, 32])
@pytest.mark.parametrize("dtype", [np.float64, np.float32])
@pytest.mark.parametrize("base", [0, 1])
def test_vector_variants_within_tolerance(variant, dtype, base):
    """Groups of W lanes per row (16-byte loads of four columns and values,
    quads straddling row boundaries masked, the array's last partial quad
    loaded entry by entry): within tolerance of the fp64 restatement for
    empty, short, medium and very long rows, alpha and beta != 0."""
    rng = np.random.default_rng(60 + variant)
    m, n = 4001, 7000
    lengths = rng.integers(0, 60, size=m)
    lengths[::31] = 0
    lengths[::97] = rng.integers(100, 3000, size=lengths[::97].shape[0])
    lengths[-1] = 3                     # the last quad ends inside the arrays' tail
    rp, ci, val = random_csr(m, n, lengths, seed=61, base=base, dtype=dtype)
    x = rng.uniform(-1, 1, n).astype(dtype)
    y0 = rng.uniform(-1, 1, m).astype(dtype)
    A = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(val), (m, n), origin=base)
    h = J.prepare(J.B200Backend(), J.SpMVOp, A).set_variant(variant)
    assert h.info()["variant"] == variant
    yd = to_dev(y0)
    J.execute(J.SpMVOp, h, to_dev(x), yd, alpha=1.5, beta=-0.5)
    J.device_status()
    ref, bound = O.spmv_ref64(rp - base, ci - base, val, x, y0, 1.5, -0.5)
    assert_within(yd.cpu().numpy(), ref, bound, TOL[dtype])


def test_plan_picks_vector_rows_for_uniform_rows():
    """Uniform rows of 16-40 entries: the plan takes groups of 4 lanes per row
    and agrees within tolerance with the restatement; the set_variant
    override refuses widths other than 0, 2, 4, 8, 16, 32."""
    rng = np.random.default_rng(70)
    m, n = 20000, 20000
    rp, ci, val = random_csr(m, n, rng.integers(16, 41, size=m), seed=71)
    x = rng.uniform(-1, 1, n)
    A = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(val), (m, n), origin=0)
    h = J.prepare(J.B200Backend(), J.SpMVOp, A)
    assert h.info()["variant"] == 4
    y = torch.zeros(m, dtype=torch.float64, device=DEV)
    J.execute(J.SpMVOp, h, to_dev(x), y)
    J.device_status()
    ref, bound = O.spmv_ref64(rp, ci, val, x)
    assert_within(y.cpu().numpy(), ref, bound, 1e-12)
    with pytest.raises(J.errors.InvalidArgument):
        h.set_variant(3)


def test_vector_variant_unaligned_values_fall_back():
    """A value array that is not 16-byte aligned (a view one element in)
    runs the thread-per-row kernel: bit-exact for short rows."""
    rng = np.random.default_rng(72)
    m, n = 3000, 3000
    rp, ci, val = random_csr(m, n, rng.integers(0, 20, size=m), seed=73)
    store = to_dev(np.concatenate([[0.0], val]))
    A = J.csr_tensor(to_dev(rp), to_dev(ci), store[1:], (m, n), origin=0)
    h = J.prepare(J.B200Backend(), J.SpMVOp, A).set_variant(8)
    x = rng.uniform(-1, 1, n)
    y = torch.zeros(m, dtype=torch.float64, device=DEV)
    J.execute(J.SpMVOp, h, to_dev(x), y)
    J.device_status()
    assert np.array_equal(y.cpu().numpy(), O.spmv(rp, ci, val, x))


def _banded_csr(m, lo_bw, hi_bw, seed, base=0, dtype=np.float64, drop=0.0):
    """Rows whose columns are [r - lo_bw, r + hi_bw] clipped to the matrix,
    a fraction `drop` of them left out."""
    rng = np.random.default_rng(seed)
    rows, cols = [], []
    for r in range(m):
        c = np.arange(max(0, r - lo_bw), min(m, r + hi_bw + 1))
        if drop:
            c = c[rng.random(c.shape[0]) >= drop]
        rows.append(np.full(c.shape[0], r))
        cols.append(c)
    cols = np.concatenate(cols).astype(np.int32)
    lens = np.array([len(r) for r in rows])
    rp = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    val = rng.uniform(-1, 1, cols.shape[0]).astype(dtype)
    return (rp + base).astype(np.int32), (cols + base).astype(np.int32), val


@pytest.mark.parametrize("dtype", [np.float64, np.float32])
@pytest.mark.parametrize("base", [0, 1])
def test_banded_staged_x_variant(dtype, base):
    """Variant 1 stages each 1024-row block's window of x in shared memory:
    bit-exact with the oracle for rows of up to 32 entries (the same sums in
    the same order as variant 0), beta != 0 included."""
    m = 5000
    rp, ci, val = _banded_csr(m, 9, 14, seed=80, base=base, dtype=dtype, drop=0.2)
    rng = np.random.default_rng(81)
    x = rng.uniform(-1, 1, m).astype(dtype)
    y0 = rng.uniform(-1, 1, m).astype(dtype)
    A = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(val), (m, m), origin=base)
    h = J.prepare(J.B200Backend(), J.SpMVOp, A).set_variant(1)
    assert h.info()["variant"] == 1
    y = to_dev(np.zeros(m, dtype))
    J.execute(J.SpMVOp, h, to_dev(x), y)
    J.device_status()
    assert np.array_equal(y.cpu().numpy(), O.spmv(rp - base, ci - base, val, x))
    yb = to_dev(y0)
    J.execute(J.SpMVOp, h, to_dev(x), yb, alpha=1.5, beta=-0.5)
    J.device_status()
    assert np.array_equal(yb.cpu().numpy(), O.spmv(rp - base, ci - base, val, x, y0, 1.5, -0.5))


def test_banded_staged_x_long_rows_and_laplacian():
    """Variant 1 on rows longer than 32 entries (the warp path, within
    tolerance) and on the 5-point Laplacian (bit-exact)."""
    m = 3000
    rp, ci, val = _banded_csr(m, 30, 25, seed=82)
    x = np.random.default_rng(83).uniform(-1, 1, m)
    A = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(val), (m, m), origin=0)
    h = J.prepare(J.B200Backend(), J.SpMVOp, A).set_variant(1)
    y = torch.zeros(m, dtype=torch.float64, device=DEV)
    J.execute(J.SpMVOp, h, to_dev(x), y)
    J.device_status()
    ref, bound = O.spmv_ref64(rp, ci, val, x)
    assert_within(y.cpu().numpy(), ref, bound, 1e-12)
    rp, ci, val, x = synth.config2(g=96)
    n = 96 * 96
    A = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(val), (n, n), origin=0)
    h = J.prepare(J.B200Backend(), J.SpMVOp, A).set_variant(1)
    y = torch.zeros(n, dtype=torch.float64, device=DEV)
    J.execute(J.SpMVOp, h, to_dev(x), y)
    J.device_status()
    assert np.array_equal(y.cpu().numpy(), O.spmv(rp, ci, val, x))


def test_banded_staged_x_falls_back_when_window_too_wide():
    """A matrix whose bandwidth gives a window larger than shared memory (one
    entry far from the diagonal) runs variant 0 under variant 1: bit-exact."""
    m = 40000
    rp, ci, val = _banded_csr(m, 2, 2, seed=84)
    ci = ci.copy()
    ci[rp[5]] = m - 1                  # row 5 reaches the last column
    order = np.argsort(ci[rp[5]:rp[6]], kind="stable")
    ci[rp[5]:rp[6]] = ci[rp[5]:rp[6]][order]
    val[rp[5]:rp[6]] = val[rp[5]:rp[6]][order]
    x = np.random.default_rng(85).uniform(-1, 1, m)
    A = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(val), (m, m), origin=0)
    h = J.prepare(J.B200Backend(), J.SpMVOp, A).set_variant(1)
    y = torch.zeros(m, dtype=torch.float64, device=DEV)
    J.execute(J.SpMVOp, h, to_dev(x), y)
    J.device_status()
    assert np.array_equal(y.cpu().numpy(), O.spmv(rp, ci, val, x))
