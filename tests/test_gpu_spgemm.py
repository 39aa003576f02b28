"""SpGEMM C = alpha*A*B (CSR x CSR -> CSR) on the GPU: the reference's known
answer, and bit-exact against the oracle's restatement of the reference's
scatter-sort-reduce order (products of a row in A-entry then B-entry order,
sorted stably by column, runs summed left to right) for random matrices,
rows of C with up to ~20,000 products (all three sorts), empty rows, explicit
zeros (kept in the structure, as in the reference) and both origins; the
prepared handle recomputes values for new values of the same structures."""
import numpy as np
import pytest
import torch

import jlust_b200 as J
from oracle import oracle as O
from _helpers import DEV, random_csr, to_dev

pytestmark = pytest.mark.gpu


def _t(rp, ci, v, m, n, base):
    return J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(v), (m, n), origin=base)


def _check(C, ref):
    assert np.array_equal(J.positions(C, 2).cpu().numpy(), ref[0])
    assert np.array_equal(J.coordinates(C, 2).cpu().numpy(), ref[1])
    assert np.array_equal(J.nonzeros(C).cpu().numpy(), ref[2])


def test_kat(golden):
    g = golden["spgemm_csr"]
    a = g["A"]
    rp, ci = np.array(a["rowptr"], np.int32), np.array(a["colind"], np.int32)
    v = np.array(a["val"], np.float32)
    A = _t(rp, ci, v, 3, 3, 1)
    C0 = J.csr_tensor(to_dev(np.ones(4, np.int32)), to_dev(np.zeros(0, np.int32)),
                      to_dev(np.zeros(0, np.float32)), (3, 3), origin=1)
    C = J.execute(J.SpGEMMOp, A, A, C0)
    J.device_status()
    D = np.zeros((3, 3), np.float32)
    crp, cci, cv = (x.cpu().numpy() for x in (J.positions(C, 2), J.coordinates(C, 2), J.nonzeros(C)))
    for r in range(3):
        D[r, cci[crp[r] - 1:crp[r + 1] - 1] - 1] = cv[crp[r] - 1:crp[r + 1] - 1]
    assert D.tolist() == g["C_dense"]


@pytest.mark.parametrize("dtype", [np.float64, np.float32])
@pytest.mark.parametrize("base", [0, 1])
@pytest.mark.parametrize("alpha", [1.0, -0.75])
def test_random_bit_exact(dtype, base, alpha):
    rng = np.random.default_rng(300)
    m, k, n = 3000, 2500, 2000
    la = rng.integers(0, 12, m)
    la[rng.random(m) < 0.1] = 0
    lb = rng.integers(0, 20, k)
    lb[rng.random(k) < 0.1] = 0
    arp, aci, av = random_csr(m, k, la, seed=301, base=base, dtype=dtype, zero_frac=0.05)
    brp, bci, bv = random_csr(k, n, lb, seed=302, base=base, dtype=dtype)
    A, B = _t(arp, aci, av, m, k, base), _t(brp, bci, bv, k, n, base)
    C = J.execute(J.SpGEMMOp, A, B, A, alpha=alpha)
    J.device_status()
    assert C.origin.offset == base and C.extents == (m, n)
    _check(C, O.spgemm(m, n, arp, aci, av, brp, bci, bv, alpha=alpha, base=base))


def test_long_rows_of_products():
    """A few dense A rows against long B rows: rows of C with more than 256
    and more than 16,384 products, duplicates in every column."""
    rng = np.random.default_rng(310)
    m, k, n = 64, 400, 900
    la = rng.integers(1, 5, m)
    la[3], la[10], la[20] = 390, 120, 60
    arp, aci, av = random_csr(m, k, la, seed=311)
    brp, bci, bv = random_csr(k, n, rng.integers(20, 90, k), seed=312)
    A, B = _t(arp, aci, av, m, k, 0), _t(brp, bci, bv, k, n, 0)
    h = J.prepare(J.B200Backend(), J.SpGEMMOp, A, B)
    assert h.products > 0
    counts = [sum(int(brp[j + 1] - brp[j]) for j in aci[arp[r]:arp[r + 1]]) for r in range(m)]
    assert max(counts) > 16384 and sorted(counts)[-2] > 256
    C = J.execute(h, A, B)
    J.device_status()
    _check(C, O.spgemm(m, n, arp, aci, av, brp, bci, bv))


def test_handle_new_values_and_square():
    """The prepared handle: new values of the same structures recompute C
    without a new symbolic pass (update of the reference's handle path)."""
    rng = np.random.default_rng(320)
    m = 5000
    rp, ci, v = random_csr(m, m, rng.integers(0, 9, m), seed=321)
    A = _t(rp, ci, v, m, m, 0)
    h = J.prepare(J.B200Backend(), J.SpGEMMOp, A, A)
    C1 = J.execute(h, A, A)
    _check(C1, O.spgemm(m, m, rp, ci, v, rp, ci, v))
    v2 = rng.uniform(-2, 2, v.shape[0])
    A2 = _t(rp, ci, v2, m, m, 0)
    C2 = J.execute(h, A2, A, alpha=0.5)
    J.device_status()
    _check(C2, O.spgemm(m, m, rp, ci, v2, rp, ci, v, alpha=0.5))


def test_empty_and_errors():
    z = np.zeros(0, np.int32)
    A = J.csr_tensor(to_dev(np.zeros(5, np.int32)), to_dev(z), to_dev(np.zeros(0)), (4, 3), origin=0)
    B = J.csr_tensor(to_dev(np.zeros(4, np.int32)), to_dev(z), to_dev(np.zeros(0)), (3, 6), origin=0)
    C = J.execute(J.SpGEMMOp, A, B, A)
    assert J.positions(C, 2).cpu().tolist() == [0, 0, 0, 0, 0] and J.nonzeros(C).numel() == 0
    with pytest.raises(J.IncompatibleExtents):
        J.execute(J.SpGEMMOp, A, A, A)
    bad = J.csr_tensor(to_dev(np.array([0, 1], np.int32)), to_dev(np.array([7], np.int32)),
                       to_dev(np.ones(1)), (1, 3), origin=0)
    with pytest.raises(J.NonCanonicalStorage):
        J.execute(J.SpGEMMOp, bad, B, bad)
