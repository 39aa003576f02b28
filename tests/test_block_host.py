"""BlockSparseMatrix on the host: the reference's construction checks
(src/block_sparse.jl:34-73) and the assembled CSR of the compiled path
against the oracle's restatement of the reference's assembly
(ext/CUDAExt/ops/block_mul.jl:128-229), on CPU tensors."""
import numpy as np
import pytest
import torch

import jlust_b200 as J
from jlust_b200.block import _Compiled
from oracle import oracle as O
from _helpers import random_csr


def _blk(m, n, seed, base=0, dtype=np.float64, lens=None):
    rng = np.random.default_rng(seed)
    rp, ci, v = random_csr(m, n, rng.integers(0, 6, m) if lens is None else lens, seed=seed,
                           base=base, dtype=dtype)
    return (rp, ci, v, base), J.csr_tensor(torch.from_numpy(rp), torch.from_numpy(ci),
                                            torch.from_numpy(v), (m, n), origin=base)


def test_construction_checks():
    _, a = _blk(3, 4, 1)
    _, b = _blk(2, 4, 2)
    _, c = _blk(3, 5, 3)
    with pytest.raises(ValueError, match="inconsistent"):
        J.BlockSparseMatrix([[a, None], [b, None], [c, None]])
    with pytest.raises(ValueError, match="entirely nothing"):
        J.BlockSparseMatrix([[a, None], [None, None]])
    with pytest.raises(ValueError, match="all blocks are nothing"):
        J.BlockSparseMatrix([[None]])
    _, f = _blk(3, 4, 4, dtype=np.float32)
    with pytest.raises(ValueError, match="mixed element types"):
        J.BlockSparseMatrix([[a, f]])
    A = J.BlockSparseMatrix([[a, None], [None, c]])
    assert A.shape == (6, 9) and A.compilable()


def test_assembly_matches_reference_order():
    sizes_r, sizes_c = [5, 3, 7], [4, 6]
    host, blocks = {}, [[None, None], [None, None], [None, None]]
    for (i, j), base in {(0, 0): 0, (0, 1): 1, (1, 1): 0, (2, 0): 1, (2, 1): 0}.items():
        h, t = _blk(sizes_r[i], sizes_c[j], 10 + 3 * i + j, base=base)
        host[(i, j)], blocks[i][j] = h, t
    A = J.BlockSparseMatrix(blocks)
    c = _Compiled(A)
    rp, ci, v = O.bsm_assemble(sizes_r, sizes_c, host)
    assert np.array_equal(c.csr.pos[1].numpy(), rp)
    assert np.array_equal(c.csr.crd[1].numpy(), ci)
    assert np.array_equal(c.val.numpy(), v)


def _bbm_case(dev=None, dtype=np.float64):
    """T = 5 periods, bw = 2, per-period diagonal blocks, level 1 shared,
    level 2 per transition."""
    T, bw, nd, no, nc = 5, 2, 40, [7, 5], 30
    dh, dt = [], []
    for t in range(T):
        h, u = _blk(nd, nc, 200 + t, base=t % 2, dtype=dtype)
        dh.append(h), dt.append(u)
    n1h, n1 = _blk(no[0], nc, 300, dtype=dtype)
    p1h, p1 = _blk(no[0], nc, 301, base=1, dtype=dtype)
    lvl2h, lvl2 = [], []
    for t in range(T - 2):
        a, ua = _blk(no[1], nc, 400 + t, dtype=dtype)
        b, ub = _blk(no[1], nc, 500 + t, dtype=dtype)
        lvl2h.append((a, b)), lvl2.append((ua, ub))
    offh = [[(n1h, p1h)] * (T - 1), lvl2h]
    M = J.BlockBandedMatrix(dt, [(n1, p1), lvl2], T, bw, nd, no, nc)
    return M, dh, offh, (T, bw, nd, no, nc)


def test_bbm_shape_and_assembly():
    M, dh, offh, (T, bw, nd, no, nc) = _bbm_case()
    assert M.shape == (T * nd + (T - 1) * no[0] + (T - 2) * no[1], T * nc)
    from jlust_b200.block import _Assembled
    c = _Assembled(*M.shape, M.parts(), torch.float64)
    x = np.random.default_rng(9).uniform(-1, 1, M.shape[1])
    got = O.spmv(c.csr.pos[1].numpy(), c.csr.crd[1].numpy(), c.val.numpy(), x)
    ref, bound = O.bbm_spmv_ref64(dh, offh, T, bw, nd, no, nc, x)
    assert np.all(np.abs(got - ref) <= 1e-12 * bound + 1e-300)


def test_selector_patches_compile():
    """ShiftedDiag blocks and CSR blocks that are a constant times the
    identity leave the assembled CSR as selector patches (block_mul.jl:
    89-229), in (i, j) order, as the oracle's restatement of the compile
    has them; a block with a column shift past its columns is refused."""
    h00, b00 = _blk(4, 5, 21)
    sel = (np.arange(4, dtype=np.int32), np.arange(3, dtype=np.int32), np.full(3, 0.5), 0)
    b10 = J.csr_tensor(*(torch.from_numpy(a) for a in sel[:3]), (3, 5), origin=0)
    h11, b11 = _blk(3, 6, 22, base=1)
    sd = J.shifted_diag_tensor(torch.float64, 4, 6, shift=2, val=3.0)
    A = J.BlockSparseMatrix([[b00, sd], [b10, b11]])
    c = _Compiled(A)
    rp, ci, v, patches = O.bsm_compile([4, 3], [5, 6], {(0, 0): h00, (1, 0): sel, (1, 1): h11},
                                       {(0, 1): (2, 3.0)})
    assert c.patches == patches == [(0, 3, 7, 3.0), (4, 6, 0, 0.5)]
    assert np.array_equal(J.positions(c.csr, 2).numpy(), rp)
    assert np.array_equal(J.coordinates(c.csr, 2).numpy(), ci)
    assert np.array_equal(c.val.numpy(), v)
    bad = J.BlockSparseMatrix([[b00, J.shifted_diag_tensor(torch.float64, 4, 6, shift=3)],
                               [b10, b11]])
    with pytest.raises(J.IncompatibleExtents, match="ShiftedDiag"):
        _Compiled(bad)
    # the oracle's patched product against a dense product
    x = np.random.default_rng(23).uniform(-1, 1, 11)
    D = np.zeros((7, 11))
    for r in range(7):
        for k in range(rp[r], rp[r + 1]):
            D[r, ci[k]] += v[k]
    for r0, r1, c0, pv in patches:
        D[np.arange(r0, r1 + 1), c0 + np.arange(r1 - r0 + 1)] += pv
    assert np.allclose(O.csr_patched_spmv(rp, ci, v, patches, x), D @ x, rtol=1e-14, atol=1e-14)


def test_block_products_refuse_mismatched_vectors():
    """x and y of the compiled block products must be contiguous vectors of
    the matrix's value type: the kernels read and write value-sized elements
    at unit stride, so a float32 x with a float64 matrix, or a strided view,
    is refused before any device work."""
    _, a = _blk(6, 5, 31)
    _, b = _blk(6, 4, 32)
    A = J.BlockSparseMatrix([[a, b]])
    x64, y64 = torch.zeros(9, dtype=torch.float64), torch.zeros(6, dtype=torch.float64)
    with pytest.raises(J.UnsupportedValueType):
        J.mul(y64, A, torch.zeros(9, dtype=torch.float32))
    with pytest.raises(J.UnsupportedValueType):
        J.mul(torch.zeros(6, dtype=torch.float32), A, x64)
    with pytest.raises(J.IncompatibleExtents, match="contiguous"):
        J.mul(y64, A, torch.zeros(18, dtype=torch.float64)[::2])
    M, *_ = _bbm_case()
    m, n = M.shape
    with pytest.raises(J.UnsupportedValueType):
        J.mul(torch.zeros(m, dtype=torch.float64), M, torch.zeros(n, dtype=torch.float32))
    with pytest.raises(J.IncompatibleExtents, match="contiguous"):
        J.mul(torch.zeros(2 * m, dtype=torch.float64)[::2], M, torch.zeros(n, dtype=torch.float64))


def test_bbm_bw1_constructor():
    """The reference's bw = 1 form BlockBandedMatrix(diag, neg_off, pos_off,
    T, n_diag_rows, n_off_rows, n_cols) (src/block_banded.jl:56-62) builds
    the same matrix as the general form with one shared coupling pair."""
    _, d = _blk(8, 6, 41)
    _, neg = _blk(3, 6, 42)
    _, pos = _blk(3, 6, 43)
    M1 = J.BlockBandedMatrix(d, neg, pos, 4, 8, 3, 6)
    M2 = J.BlockBandedMatrix(d, [(neg, pos)], 4, 1, 8, [3], 6)
    assert M1.shape == M2.shape == (4 * 8 + 3 * 3, 24)
    assert (M1.bw, M1.n_off_rows, M1.starts) == (M2.bw, M2.n_off_rows, M2.starts)
    assert [(k, r, c) for k, r, c, _ in M1.parts()] == [(k, r, c) for k, r, c, _ in M2.parts()]
    with pytest.raises(ValueError, match="n_off_rows an Int"):
        J.BlockBandedMatrix(d, neg, pos, 4, 8, [3], 6)
    _, f32 = _blk(3, 6, 44, dtype=np.float32)
    with pytest.raises(ValueError, match="mixed element types"):
        J.BlockBandedMatrix(d, neg, f32, 4, 8, 3, 6)
