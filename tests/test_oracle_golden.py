"""The CPU oracle against the reference's known-answer vectors, and its own
invariants (thread-count independence, fp64 agreement, conversion round trip)."""
import numpy as np
import pytest

from oracle import oracle as O
from jlust_b200 import synth


def _csr(d, dtype=np.float64):
    return (np.array(d["rowptr"], np.int32), np.array(d["colind"], np.int32),
            np.array(d["val"], dtype), d["base"])


@pytest.mark.parametrize("name", ["spmv_csr_onebased", "spmv_csr_zerobased"])
@pytest.mark.parametrize("dtype", [np.float64, np.float32])
def test_spmv_kat(golden, name, dtype):
    g = golden[name]
    rp, ci, v, base = _csr(g["A"], dtype)
    y = O.spmv(rp, ci, v, np.array(g["x"], dtype), alpha=g["alpha"], beta=g["beta"], base=base)
    assert np.array_equal(y, np.array(g["y"], dtype))


@pytest.mark.parametrize("order", ["C", "F"])
def test_spmm_kat(golden, order):
    g = golden["spmm_csr_onebased"]
    rp, ci, v, base = _csr(g["A"])
    B = np.array(g["B"], np.float64, order=order)
    C = O.spmm(rp, ci, v, B, base=base, c_order=0 if order == "C" else 1)
    assert np.array_equal(C, np.array(g["C"]))


def test_sddmm_kat(golden):
    g = golden["sddmm_csr_onebased"]
    rp, ci, v, base = _csr(g["C"], np.float32)
    A = np.array(g["A"], np.float32)
    B = np.array(g["B"], np.float32)      # K x n as the reference passes it
    out = O.sddmm(rp, ci, A, B, v, mode=0, alpha=g["alpha"], beta=g["beta"], base=base)
    assert np.array_equal(out, np.array(g["out"], np.float32))
    # sampled-product mode with S = 1 gives the same values
    out1 = O.sddmm(rp, ci, A, B, v, S=np.ones(5, np.float32), mode=1, base=base)
    assert np.array_equal(out1, out)


def test_conversion_fixture_blocks(golden):
    """CSR fixture of test_convert.jl to BSRRight((2,2)) with the level extents
    of dim2lvl(as_size=true): ceil(3/2) = 2 block rows."""
    g = golden["convert_fixture_3x4"]
    rp, ci, v, base = _csr(g["A"], np.float32)
    bp, bc, bv = O.csr_to_bsr(3, 4, rp, ci, v, 2, 2, base=base)
    assert bp.tolist() == [0, 2, 4]
    assert bc.tolist() == [0, 1, 0, 1]
    assert bv.tolist() == [1, 0, 0, 3, 2, 0, 0, 0, 4, 0, 0, 0, 5, 0, 0, 0]
    # the decomposer's visit set is recovered from the blocks
    visits = []
    for I in range(2):
        for q in range(bp[I], bp[I + 1]):
            tile = bv[q * 4:(q + 1) * 4].reshape(2, 2)
            for r in range(2):
                for c in range(2):
                    if tile[r, c] != 0:
                        visits.append([[I * 2 + r, int(bc[q]) * 2 + c], float(tile[r, c])])
    assert sorted(visits) == sorted(g["decomposer_visits"])


def test_conversion_origin_preserved():
    rp = np.array([1, 3, 4, 6], np.int32)
    ci = np.array([1, 3, 2, 1, 3], np.int32)
    v = np.array([1, 2, 3, 4, 5], np.float32)
    bp, bc, bv = O.csr_to_bsr(3, 4, rp, ci, v, 2, 2, base=1)
    assert bp.tolist() == [1, 3, 5] and bc.tolist() == [1, 2, 1, 2]


def test_coo_duplicates_first_wins_and_zeros_dropped():
    rows = np.array([2, 0, 0, 1, 0], np.int32)
    cols = np.array([3, 1, 1, 0, 1], np.int32)
    vals = np.array([5, 0, 7, 9, 8], np.float64)   # (0,1): 0 dropped, then 7 wins over 8
    bp, bc, bv = O.coo_to_bsr(3, 4, rows, cols, vals, 2, 2)
    assert bp.tolist() == [0, 1, 2]
    assert bc.tolist() == [0, 1]
    assert bv.tolist() == [0, 7, 9, 0, 0, 5, 0, 0]


def test_scan():
    c = np.array([3, 0, 2, 5], np.int32)
    assert O.exclusive_scan(c, base=1).tolist() == [1, 4, 4, 6, 11]


def test_thread_count_independent():
    rp, ci, v, x = synth.config1(seed=5, n=3000, k=7)
    outs = []
    for t in (1, 4):
        O.set_threads(t)
        outs.append(O.spmv(rp, ci, v, x))
    O.set_threads(O.max_threads())
    assert np.array_equal(outs[0], outs[1])


def test_spmv_matches_fp64_reference():
    rp, ci, v, x = synth.config1(seed=6, n=2000, k=9)
    y = O.spmv(rp, ci, v, x, alpha=0.5)
    y64, bound = O.spmv_ref64(rp, ci, v, x, alpha=0.5)
    assert np.all(np.abs(y - y64) <= 1e-14 * bound + 1e-300)


def test_bsr_oracle_vs_dense():
    bp, bc, bv, B = synth.config5(seed=7, nbr=6, bs=8, band=1, p_off=0.3, N=16)
    Y = O.bsr_spmm(bp, bc, bv, B, b1=8, b2=8)
    dense = np.zeros((48, 48), np.float64)
    for I in range(6):
        for q in range(bp[I], bp[I + 1]):
            dense[I * 8:(I + 1) * 8, bc[q] * 8:(bc[q] + 1) * 8] = synth.bf16_bits_to_f32(
                bv[q * 64:(q + 1) * 64]).reshape(8, 8)
    ref = dense @ synth.bf16_bits_to_f32(B).astype(np.float64)
    assert np.allclose(Y, ref, rtol=1e-5, atol=1e-5)
    y64, bound = O.bsr_spmm_ref64(bp, bc, bv, B, b1=8, b2=8)
    assert np.allclose(y64, ref, rtol=1e-12, atol=1e-12)


def test_csr_bsr_round_trip():
    bp, bc, bv, _ = synth.config5(seed=8, nbr=5, bs=4, band=1, p_off=0.4, N=8)
    rp, ci, vals = synth.bsr_to_csr(bp, bc, bv, 4, 5)
    bp2, bc2, bv2 = O.csr_to_bsr(20, 20, rp, ci, vals, 4, 4)
    # blocks whose values are all zero after bf16 rounding would vanish; none here
    assert np.array_equal(bp2, bp) and np.array_equal(bc2, bc) and np.array_equal(bv2, bv)


@pytest.mark.parametrize("dtype", [np.float64, np.float32])
def test_dcsr_and_coo_spmv_kats(golden, dtype):
    """The reference's DCSR (row 2 not stored, left as it was) and COO SpMV
    answers, and the same matrix stored as CSC."""
    g = golden["spmv_dcsr_onebased"]
    y = O.dcsr_spmv(g["m"], g["fibptr"], g["row_ids"], g["colind"], np.array(g["val"], dtype),
                    np.array(g["x"], dtype), np.array(g["y0"], dtype), g["alpha"], g["beta"],
                    g["base"])
    assert y.tolist() == g["y"]
    g = golden["spmv_coo_onebased"]
    y = O.entry_spmv(g["m"], g["n"], g["rows"], np.array(g["val"], dtype),
                     np.array(g["x"], dtype), cols=g["cols"], base=g["base"])
    assert y.tolist() == g["y"]
    # column-major storage of the same entries
    order = np.lexsort((g["rows"], g["cols"]))
    rows = np.array(g["rows"])[order]
    cols = np.array(g["cols"])[order]
    colptr = np.searchsorted(cols, np.arange(1, g["n"] + 2)) + 1
    y = O.entry_spmv(g["m"], g["n"], rows, np.array(g["val"], dtype)[order],
                     np.array(g["x"], dtype), colptr=colptr, base=1)
    assert y.tolist() == g["y"]


def test_dcsr_rows_not_stored_keep_y():
    """With beta != 0 the stored rows get alpha*A x + beta*y and the others
    keep y unscaled, as the reference's DCSR walk writes stored rows only."""
    y0 = np.array([10.0, 20.0, 30.0])
    y = O.dcsr_spmv(3, [0, 2, 4], [0, 2], [0, 2, 0, 2], [1.0, 2.0, 4.0, 5.0], [1.0, 2.0, 3.0],
                    y0, 1.0, 0.5)
    assert y.tolist() == [12.0, 20.0, 34.0]


def test_csr_csc_conversion_kats(golden):
    """The reference's CSR/CSC conversion tests on its 3x4 fixture
    (test_convert.jl:34-40 CSR -> CSR identity, :44-58 CSR -> CSC buffers,
    :97-106 CSR -> CSC -> CSR round trip, :110-116 the round trip through
    COO), restated by the oracle's composer."""
    g = golden["convert_fixture_3x4"]
    rp, ci, v, base = _csr(g["A"], np.float32)
    p2, i2, v2 = O.csr_to_csr(3, 4, rp, ci, v, base)
    assert p2.tolist() == rp.tolist() and i2.tolist() == ci.tolist() and v2.tolist() == v.tolist()
    cp, ri, cv = O.csr_to_csc(3, 4, rp, ci, v, base)
    assert cp.tolist() == g["csc"]["colptr"]
    assert ri.tolist() == g["csc"]["rowind"]
    assert cv.tolist() == g["csc"]["val"]
    p3, i3, v3 = O.csc_to_csr(3, 4, cp, ri, cv, base)
    assert p3.tolist() == rp.tolist() and i3.tolist() == ci.tolist() and v3.tolist() == v.tolist()
    rows = O.expand_positions(rp, base)
    p4, i4, v4 = O.coo_to_csr(3, 4, rows, ci, v, base)
    assert p4.tolist() == rp.tolist() and i4.tolist() == ci.tolist() and v4.tolist() == v.tolist()
    # origin preserved (test_convert.jl:161-168)
    p5, i5, _ = O.csr_to_csc(3, 4, rp + 1, ci + 1, v, 1)
    assert p5.tolist() == [x + 1 for x in g["csc"]["colptr"]]
    assert i5.tolist() == [x + 1 for x in g["csc"]["rowind"]]


def test_coo_to_csr_composer_semantics():
    """COO's levels are ordered, so COO -> CSR keeps storage order: columns
    stay unsorted within a row, adjacent equal coordinates (after dropping
    zeros) keep the first value, non-adjacent ones stay separate, and rows
    that decrease are refused (convert.jl:222-246, 316, 346-355)."""
    rows = np.array([0, 0, 0, 0, 0, 2, 2, 2], np.int32)
    cols = np.array([3, 1, 1, 1, 3, 0, 0, 2], np.int32)
    val = np.array([1.0, 2.0, 0.0, 5.0, 6.0, 7.0, 8.0, -0.0])
    rp, ci, v = O.coo_to_csr(3, 4, rows, cols, val)
    assert rp.tolist() == [0, 3, 3, 4]
    assert ci.tolist() == [3, 1, 3, 0]
    assert v.tolist() == [1.0, 2.0, 6.0, 7.0]
    with pytest.raises(ValueError):
        O.coo_to_csr(3, 4, np.array([1, 0], np.int32), np.array([0, 0], np.int32), np.ones(2))
    # the same entries to CSC are lexsorted by (column, row, storage index)
    cp, ri, cv = O.coo_to_csc(3, 4, rows, cols, val)
    assert cp.tolist() == [0, 1, 2, 2, 3]
    assert ri.tolist() == [2, 0, 0] and cv.tolist() == [7.0, 2.0, 1.0]


def test_spgemm_kat(golden):
    """C = A*A for the reference's 3x3 matrix (test_cuda.jl:436-451)."""
    g = golden["spgemm_csr"]
    rp, ci, v, base = _csr(g["A"], np.float32)
    crp, cci, cv = O.spgemm(3, 3, rp, ci, v, rp, ci, v, base=base)
    D = np.zeros((3, 3), np.float32)
    for r in range(3):
        for p in range(crp[r] - base, crp[r + 1] - base):
            D[r, cci[p] - base] = cv[p]
    assert D.tolist() == g["C_dense"]
    assert crp.tolist() == [1, 3, 4, 6]


def test_csr_to_coo_kat(golden):
    """CSR -> COO of the 3x4 fixture (test_convert.jl:62-79) and the round
    trip CSR -> COO -> CSR (:110-116)."""
    g = golden["convert_fixture_3x4"]
    rp, ci, v, base = _csr(g["A"], np.float32)
    r, c, vv = O.to_coo(O.expand_positions(rp, base), ci, v)
    assert r.tolist() == [0, 0, 1, 2, 2] and c.tolist() == [0, 2, 1, 0, 2]
    assert vv.tolist() == [1, 2, 3, 4, 5]
    p2, i2, v2 = O.coo_to_csr(3, 4, r, c, vv, base)
    assert p2.tolist() == rp.tolist() and i2.tolist() == ci.tolist() and v2.tolist() == v.tolist()


def _dense_csr(m, n, rp, ci, v, base=0):
    D = np.zeros((m, n))
    for r in range(m):
        for k in range(rp[r] - base, rp[r + 1] - base):
            D[r, ci[k] - base] += float(v[k])
    return D


def test_oracle_spgemm_against_dense():
    """The oracle's SpGEMM against a dense product: C's structure is every
    column reached by a product (explicit zeros included) and its values agree
    to fp64 rounding."""
    from _helpers import random_csr
    rng = np.random.default_rng(400)
    m, k, n = 120, 90, 150
    arp, aci, av = random_csr(m, k, rng.integers(0, 8, m), seed=401, zero_frac=0.1)
    brp, bci, bv = random_csr(k, n, rng.integers(0, 10, k), seed=402)
    crp, cci, cv = O.spgemm(m, n, arp, aci, av, brp, bci, bv, alpha=-0.5)
    A, B = _dense_csr(m, k, arp, aci, av), _dense_csr(k, n, brp, bci, bv)
    assert np.allclose(_dense_csr(m, n, crp, cci, cv), -0.5 * A @ B, rtol=1e-13, atol=1e-13)
    pattern = (np.abs(_dense_csr(m, k, arp, aci, np.ones_like(av))) @
               np.abs(_dense_csr(k, n, brp, bci, np.ones_like(bv)))) > 0
    got = np.zeros((m, n), bool)
    for r in range(m):
        got[r, cci[crp[r]:crp[r + 1]]] = True
        assert np.all(np.diff(cci[crp[r]:crp[r + 1]]) > 0)
    assert np.array_equal(got, pattern)


def test_oracle_periodic_bbm_with_selectors_against_dense():
    """The oracle's periodic block-banded product with diagonal patches and a
    ShiftedDiag coupling block against the dense T-period matrix."""
    from _helpers import random_csr
    rng = np.random.default_rng(410)
    T, nd, no, nc = 5, 40, 15, 50
    drp, dci, dv = random_csr(nd, nc, rng.integers(0, 6, nd), seed=411)
    prp, pci, pv = random_csr(no, nc, rng.integers(0, 4, no), seed=412)
    patches = [(0, 9, 20, 1.5), (10, 39, 3, -2.0)]
    x = rng.uniform(-1, 1, T * nc)
    y = O.bbm_periodic_spmv(T, nd, no, nc, (drp, dci, dv), ("shifted", 7, 0.25), (prp, pci, pv), x,
                            patches=patches)
    D = _dense_csr(nd, nc, drp, dci, dv)
    for r0, r1, c0, val in patches:
        D[np.arange(r0, r1 + 1), c0 + np.arange(r1 - r0 + 1)] += val
    N = np.zeros((no, nc))
    N[np.arange(no), 7 + np.arange(no)] = 0.25
    P = _dense_csr(no, nc, prp, pci, pv)
    rows = T * nd + (T - 1) * no
    M = np.zeros((rows, T * nc))
    r = 0
    for t in range(T):
        M[r:r + nd, t * nc:(t + 1) * nc] = D
        r += nd
        if t < T - 1:
            M[r:r + no, t * nc:(t + 1) * nc] = N
            M[r:r + no, (t + 1) * nc:(t + 2) * nc] = P
            r += no
    assert np.allclose(y, M @ x, rtol=1e-13, atol=1e-13)


def _kat_blocks(g):
    out = {}
    for key, b in g["blocks"].items():
        i, j = map(int, key.split(","))
        out[(i, j)] = (np.array(b["rowptr"], np.int32), np.array(b["colind"], np.int32),
                       np.array(b["val"]), b["base"])
    return out


@pytest.mark.parametrize("name", ["bsm_diagonal", "bsm_accumulate"])
def test_bsm_kats(golden, name):
    """The reference's BlockSparseMatrix KATs (test/test_emitter_cuda.jl:
    297-322) through the oracle's restatement of the compiled CSR
    (block_mul.jl:128-229) and its SpMV."""
    g = golden[name]
    blocks = _kat_blocks(g)
    nbr, nbc = g["grid"]
    row_sizes = [[g["blocks"][k]["m"] for k in g["blocks"] if int(k.split(",")[0]) == r][0]
                 for r in range(nbr)]
    col_sizes = [[g["blocks"][k]["n"] for k in g["blocks"] if int(k.split(",")[1]) == c][0]
                 for c in range(nbc)]
    rp, ci, v = O.bsm_assemble(row_sizes, col_sizes, blocks)
    assert O.spmv(rp, ci, v, np.array(g["x"])).tolist() == g["y"]
