"""SpMV with DCSR, COO and CSC inputs on the GPU against the CPU oracle: the
reference's known answers, DCSR bit-exact for rows of up to 32 entries (rows
that are not stored keep y), COO and CSC within tolerance (their terms land
through atomic adds, in the reference as here)."""
import numpy as np
import pytest

import jlust_b200 as J
from oracle import oracle as O
from _helpers import DEV, assert_within, random_csr, to_dev

pytestmark = pytest.mark.gpu
TOL = {np.float64: 1e-12, np.float32: 1e-5}


def _origin(base):
    return J.OneBased() if base == 1 else J.ZeroBased()


def dcsr(m, n, fibptr, row_ids, colind, val, base):
    return J.USTensor((m, n), J.Formats.DCSR, (None, to_dev(fibptr)),
                      (to_dev(row_ids), to_dev(colind)), to_dev(val), _origin(base))


def csc(m, n, colptr, rowind, val, base):
    return J.USTensor((m, n), J.Formats.CSC, (None, to_dev(colptr)), (None, to_dev(rowind)),
                      to_dev(val), _origin(base))


def run(A, x, y0, alpha=1.0, beta=0.0):
    y = to_dev(y0)
    J.execute(J.SpMVOp, A, to_dev(x), y, alpha=alpha, beta=beta)
    J.device_status()
    return y.cpu().numpy()


def test_kats(golden):
    g = golden["spmv_dcsr_onebased"]
    A = dcsr(g["m"], g["n"], np.array(g["fibptr"], np.int32), np.array(g["row_ids"], np.int32),
             np.array(g["colind"], np.int32), np.array(g["val"]), 1)
    assert run(A, np.array(g["x"]), np.array(g["y0"])).tolist() == g["y"]
    g = golden["spmv_coo_onebased"]
    A = J.coo_tensor(to_dev(np.array(g["rows"], np.int32)), to_dev(np.array(g["cols"], np.int32)),
                     to_dev(np.array(g["val"])), (g["m"], g["n"]), origin=1)
    assert run(A, np.array(g["x"]), np.full(3, np.nan)).tolist() == g["y"]


def _dcsr_case(dtype, base, max_len, seed):
    rng = np.random.default_rng(seed)
    m, n = 5000, 3000
    stored = np.sort(rng.choice(m, size=1800, replace=False))
    rp, ci, val = random_csr(stored.shape[0], n, rng.integers(1, max_len + 1, stored.shape[0]),
                             seed=seed + 1, base=base, dtype=dtype)
    return m, n, rp, (stored + base).astype(np.int32), ci, val, rng


@pytest.mark.parametrize("dtype", [np.float64, np.float32])
@pytest.mark.parametrize("base", [0, 1])
@pytest.mark.parametrize("ab", [(1.0, 0.0), (0.5, -1.5)])
def test_dcsr_bit_exact(dtype, base, ab):
    m, n, rp, rows, ci, val, rng = _dcsr_case(dtype, base, 32, 71)
    x = rng.uniform(-1, 1, n).astype(dtype)
    y0 = rng.uniform(-1, 1, m).astype(dtype)
    got = run(dcsr(m, n, rp, rows, ci, val, base), x, y0, *ab)
    ref = O.dcsr_spmv(m, rp, rows, ci, val, x, y0, ab[0], ab[1], base)
    assert np.array_equal(got, ref)                       # stored rows and untouched rows


def test_dcsr_long_rows_within_tolerance():
    m, n, rp, rows, ci, val, rng = _dcsr_case(np.float64, 0, 200, 73)
    x = rng.uniform(-1, 1, n)
    got = run(dcsr(m, n, rp, rows, ci, val, 0), x, np.zeros(m))
    r = np.repeat(rows, np.diff(rp))
    ref, bound = O.entry_spmv_ref64(m, r, ci, val, x)
    assert_within(got, ref, bound, 1e-12)


@pytest.mark.parametrize("dtype", [np.float64, np.float32])
@pytest.mark.parametrize("base", [0, 1])
@pytest.mark.parametrize("shuffle", [False, True])
def test_coo_within_tolerance(dtype, base, shuffle):
    rng = np.random.default_rng(75)
    m, n = 4000, 3500
    rp, ci, val = random_csr(m, n, rng.integers(0, 60, m), seed=76, dtype=dtype)
    rows = np.repeat(np.arange(m, dtype=np.int32), np.diff(rp))
    # duplicate some coordinates: duplicates add
    dup = rng.choice(rows.shape[0], 500, replace=False)
    rows, ci = np.concatenate([rows, rows[dup]]), np.concatenate([ci, ci[dup]])
    val = np.concatenate([val, rng.uniform(-1, 1, 500).astype(dtype)])
    if shuffle:
        p = rng.permutation(rows.shape[0])
        rows, ci, val = rows[p], ci[p], val[p]
    x = rng.uniform(-1, 1, n).astype(dtype)
    y0 = rng.uniform(-1, 1, m).astype(dtype)
    A = J.coo_tensor(to_dev((rows + base).astype(np.int32)), to_dev((ci + base).astype(np.int32)),
                     to_dev(val), (m, n), origin=base)
    for alpha, beta in ((1.0, 0.0), (-0.5, 2.0)):
        got = run(A, x, y0, alpha, beta)
        ref, bound = O.entry_spmv_ref64(m, rows, ci, val, x, y0, alpha, beta)
        assert_within(got, ref, bound, TOL[dtype])


@pytest.mark.parametrize("dtype", [np.float64, np.float32])
@pytest.mark.parametrize("base", [0, 1])
def test_csc_within_tolerance(dtype, base):
    rng = np.random.default_rng(77)
    m, n = 3000, 4500
    # columns as the rows of a random CSR of the transpose
    cp, ri, val = random_csr(n, m, rng.integers(0, 30, n), seed=78, dtype=dtype)
    x = rng.uniform(-1, 1, n).astype(dtype)
    y0 = rng.uniform(-1, 1, m).astype(dtype)
    A = csc(m, n, (cp + base).astype(np.int32), (ri + base).astype(np.int32), val, base)
    got = run(A, x, y0, 1.5, 0.25)
    cols = np.repeat(np.arange(n), np.diff(cp))
    ref, bound = O.entry_spmv_ref64(m, ri, cols, val, x, y0, 1.5, 0.25)
    assert_within(got, ref, bound, TOL[dtype])
    assert_within(O.entry_spmv(m, n, ri, val, x, colptr=cp, y=y0, alpha=1.5, beta=0.25),
                  ref, bound, TOL[dtype])


def test_coo_out_of_range_row_reported():
    """A coordinate outside the extents is skipped on the device and reported
    as non-canonical storage; the context stays usable."""
    A = J.coo_tensor(to_dev(np.array([0, 7], np.int32)), to_dev(np.array([0, 1], np.int32)),
                     to_dev(np.array([1.0, 2.0])), (3, 3), origin=0)
    y = to_dev(np.zeros(3))
    J.execute(J.SpMVOp, A, to_dev(np.ones(3)), y)
    with pytest.raises(J.NonCanonicalStorage):
        J.device_status()
    assert y.cpu().tolist() == [1.0, 0.0, 0.0]
