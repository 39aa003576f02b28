"""CSR SpMM on the GPU against the CPU oracle: bit-exact per element for rows
of up to 256 entries (storage-order sums), within tolerance for longer rows;
generic layouts (column-major B and C, Julia's native order) bit-exact."""
import numpy as np
import pytest
import torch

import jlust_b200 as J
from jlust_b200 import synth
from oracle import oracle as O
from _helpers import DEV, assert_within, random_csr, to_dev

pytestmark = pytest.mark.gpu


def run(rp, ci, val, B, m, n, base, C0=None, alpha=1.0, beta=0.0, c_col_major=False):
    A = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(val), (m, n), origin=base)
    Bd = torch.from_numpy(np.asarray(B)).to(DEV)
    if np.asarray(B).flags.f_contiguous and not np.asarray(B).flags.c_contiguous:
        Bd = torch.from_numpy(np.ascontiguousarray(np.asarray(B).T)).to(DEV).t()
    k = B.shape[1]
    if C0 is None:
        C0 = np.zeros((m, k), val.dtype)
    if c_col_major:
        Cd = torch.from_numpy(np.ascontiguousarray(C0.T)).to(DEV).t()
    else:
        Cd = torch.from_numpy(np.ascontiguousarray(C0)).to(DEV)
    J.execute(J.SpMMOp, A, Bd, Cd, alpha=alpha, beta=beta)
    J.device_status()
    return Cd.cpu().numpy()


def test_kat(golden):
    g = golden["spmm_csr_onebased"]
    A = g["A"]
    C = run(np.array(A["rowptr"], np.int32), np.array(A["colind"], np.int32), np.array(A["val"]),
            np.array(g["B"]), 3, 3, 1)
    assert C.tolist() == g["C"]


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("k", [64, 8, 100, 192])
@pytest.mark.parametrize("base", [0, 1])
def test_rowmajor_bit_exact(dtype, k, base):
    rng = np.random.default_rng(31)
    m, n = 3000, 2500
    lengths = rng.integers(0, 40, size=m)
    lengths[::41] = 0
    lengths[::113] = rng.integers(100, 256, size=lengths[::113].shape[0])
    rp, ci, val = random_csr(m, n, lengths, seed=32, base=base, dtype=dtype)
    B = rng.uniform(-1, 1, size=(n, k)).astype(dtype)
    C0 = rng.uniform(-1, 1, size=(m, k)).astype(dtype)
    for alpha, beta in ((1.0, 0.0), (0.75, -1.25)):
        got = run(rp, ci, val, B, m, n, base, C0, alpha, beta)
        ref = O.spmm(rp, ci, val, B, C0, alpha, beta, base)
        assert np.array_equal(got, ref)


def test_long_rows_tolerance():
    rng = np.random.default_rng(33)
    m, n, k = 600, 20000, 64
    lengths = rng.integers(1, 8, size=m)
    lengths[::37] = rng.integers(257, 6000, size=lengths[::37].shape[0])
    rp, ci, val = random_csr(m, n, lengths, seed=34, dtype=np.float32)
    B = rng.uniform(-1, 1, size=(n, k)).astype(np.float32)
    got = run(rp, ci, val, B, m, n, 0)
    ref, bound = O.spmm_ref64(rp, ci, val, B)
    assert_within(got, ref, bound, 1e-5)
    short = np.diff(rp) <= 256
    assert np.array_equal(got[short], O.spmm(rp, ci, val, B)[short])


@pytest.mark.parametrize("k", [24, 7])
@pytest.mark.parametrize("b_f,c_f", [(True, True), (True, False), (False, True)])
def test_column_major_layouts_bit_exact(b_f, c_f, k):
    """JLUST's native column-major B and C: B transposed into a workspace and
    gathered by the streaming kernels, C stored column-major by them (k = 24);
    k = 7 (not a whole number of vectors) takes the generic kernel.  Both
    sum each row in storage order: bit-exact."""
    rng = np.random.default_rng(35)
    m, n = 700, 500
    rp, ci, val = random_csr(m, n, rng.integers(0, 30, size=m), seed=36)
    B = rng.uniform(-1, 1, size=(n, k))
    if b_f:
        B = np.asfortranarray(B)
    C0 = rng.uniform(-1, 1, size=(m, k))
    got = run(rp, ci, val, B, m, n, 0, C0, 1.5, 0.5, c_col_major=c_f)
    assert np.array_equal(got, O.spmm(rp, ci, val, B, C0, 1.5, 0.5))


@pytest.mark.parametrize("beta", [0.0, 0.5])
def test_column_major_long_rows(beta):
    """Column-major B and C (fp32, k = 64) with rows past the long-row
    threshold and 1-based storage: short rows bit-exact, long rows within
    1e-5."""
    rng = np.random.default_rng(37)
    m, n, k = 3000, 9000, 64
    lengths = rng.integers(0, 12, size=m)
    lengths[::53] = rng.integers(257, 3000, size=lengths[::53].shape[0])
    rp, ci, val = random_csr(m, n, lengths, seed=38, base=1, dtype=np.float32)
    B = np.asfortranarray(rng.uniform(-1, 1, size=(n, k)).astype(np.float32))
    C0 = rng.uniform(-1, 1, size=(m, k)).astype(np.float32)
    got = run(rp, ci, val, B, m, n, 1, C0, 1.0, beta, c_col_major=True)
    short = np.diff(rp) <= 256
    assert np.array_equal(got[short], O.spmm(rp, ci, val, B, C0, 1.0, beta, 1)[short])
    ref, bound = O.spmm_ref64(rp - 1, ci - 1, val, B, C0 if beta else None, 1.0, beta)
    assert_within(got[~short], ref[~short], bound[~short], 1e-5)


def test_column_major_b_without_workspace():
    """jlb_csr_spmm (no workspace) with a column-major B runs the generic
    kernel: bit-exact, no allocation."""
    import ctypes as C
    from jlust_b200 import _lib
    rng = np.random.default_rng(39)
    m, n, k = 400, 300, 16
    rp, ci, val = random_csr(m, n, rng.integers(0, 20, size=m), seed=40, dtype=np.float32)
    B = np.asfortranarray(rng.uniform(-1, 1, size=(n, k)).astype(np.float32))
    rpd, cid, vd = to_dev(rp), to_dev(ci), to_dev(val)
    Bd = torch.from_numpy(np.ascontiguousarray(B.T)).to(DEV)          # k x n row-major = B col-major
    Cd = torch.zeros(m, k, dtype=torch.float32, device=DEV)
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.call("jlb_csr_spmm", st, _lib.F32, 0, m, n, ci.shape[0], p(rpd), p(cid), p(vd), k, p(Bd),
              n, 1, p(Cd), k, 0, 1.0, 0.0)
    J.device_status()
    assert np.array_equal(Cd.cpu().numpy(), O.spmm(rp, ci, val, B))


def test_power_law_reduced_config3():
    """Config-3 structure (Zipf(2) out-degree up to 4096, k = 64) at 1/16 size."""
    rp, ci, val, B = synth.config3(m=262_144)
    got = run(rp, ci, val, B, 262_144, 262_144, 0)
    ref, bound = O.spmm_ref64(rp, ci, val, B)
    assert_within(got, ref, bound, 1e-5)
    short = np.diff(rp) <= 256
    assert np.array_equal(got[short], O.spmm(rp, ci, val, B)[short])


@pytest.mark.parametrize("pattern", ["empty", "all_long", "one_row", "edge256", "sparse_rows", "ragged"])
def test_row_patterns(pattern):
    """Row patterns the streaming kernel's partition and cursors must get right:
    no entries at all, only long rows, a single row, lengths at the long-row
    threshold (256 vs 257), runs of empty rows, and ragged lengths in 1-based
    storage with beta != 0."""
    rng = np.random.default_rng(41)
    n, k, base = 3000, 64, 0
    if pattern == "empty":
        lengths = np.zeros(5000, np.int64)
    elif pattern == "all_long":
        lengths = rng.integers(257, 700, size=40)
    elif pattern == "one_row":
        lengths = np.array([7])
    elif pattern == "edge256":
        lengths = rng.choice([0, 1, 255, 256, 257], size=400)
    elif pattern == "sparse_rows":
        lengths = np.where(rng.random(20000) < 0.02, rng.integers(1, 5, size=20000), 0)
    else:
        lengths = rng.integers(0, 60, size=9000)
        base = 1
    m = lengths.shape[0]
    rp, ci, val = random_csr(m, n, lengths, seed=42, base=base, dtype=np.float32)
    B = rng.uniform(-1, 1, size=(n, k)).astype(np.float32)
    C0 = rng.uniform(-1, 1, size=(m, k)).astype(np.float32)
    beta = 0.5 if pattern == "ragged" else 0.0
    got = run(rp, ci, val, B, m, n, base, C0, 1.0, beta)
    exact = O.spmm(rp, ci, val, B, C0, 1.0, beta, base)
    short = np.diff(rp) <= 256
    assert np.array_equal(got[short], exact[short])
    if (~short).any():
        ref, bound = O.spmm_ref64(rp - base, ci - base, val, B)
        assert_within(got[~short], ref[~short], bound[~short], 1e-5)
