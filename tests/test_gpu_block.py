"""BlockSparseMatrix products on the GPU. All-CSR matrices take the compiled
path (one assembled CSR, its SpMV replayed from a CUDA graph): bit-exact with
the oracle's SpMV of the reference's assembly (rows of up to 32 entries),
also after new buffers, after update_block_values and inside a capture the
caller started. Other block formats take the per-block path, and BlockSpMM
adds every block into its slice of Y: both within tolerance of fp64. A
BlockBandedMatrix is assembled the same way."""
import numpy as np
import pytest
import torch

import jlust_b200 as J
from oracle import oracle as O
from _helpers import DEV, assert_within, random_csr, to_dev

pytestmark = pytest.mark.gpu

SIZES_R, SIZES_C = [700, 300, 1100], [500, 900]
LAYOUT = {(0, 0): 0, (0, 1): 1, (1, 1): 0, (2, 0): 1, (2, 1): 0}


def _blocks(dtype=np.float64, coo_at=None):
    host, blocks = {}, [[None] * len(SIZES_C) for _ in SIZES_R]
    for (i, j), base in LAYOUT.items():
        rng = np.random.default_rng(90 + 3 * i + j)
        m, n = SIZES_R[i], SIZES_C[j]
        rp, ci, v = random_csr(m, n, rng.integers(0, 14, m), seed=91 + i + 5 * j, base=base,
                               dtype=dtype)
        host[(i, j)] = (rp, ci, v, base)
        if (i, j) == coo_at:
            rows = np.repeat(np.arange(m, dtype=np.int32), np.diff(rp)) + base
            blocks[i][j] = J.coo_tensor(to_dev(rows), to_dev(ci), to_dev(v), (m, n), origin=base)
        else:
            blocks[i][j] = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(v), (m, n), origin=base)
    return host, J.BlockSparseMatrix(blocks)


def _dense(host, dtype=np.float64):
    D = np.zeros((sum(SIZES_R), sum(SIZES_C)), dtype)
    ro, co = np.cumsum([0] + SIZES_R), np.cumsum([0] + SIZES_C)
    for (i, j), (rp, ci, v, base) in host.items():
        for r in range(SIZES_R[i]):
            for k in range(rp[r] - base, rp[r + 1] - base):
                D[ro[i] + r, co[j] + ci[k] - base] += v[k]
    return D


def _oracle_y(host, x):
    rp, ci, v = O.bsm_assemble(SIZES_R, SIZES_C, host)
    return O.spmv(rp, ci, v, x)


def test_compiled_graph_bit_exact_and_replay():
    host, A = _blocks()
    m, n = A.shape
    x = np.random.default_rng(1).uniform(-1, 1, n)
    xd, yd = to_dev(x), torch.full((m,), np.nan, dtype=torch.float64, device=DEV)
    J.mul(yd, A, xd)                                  # assembles, runs, captures
    ref = _oracle_y(host, x)
    assert np.array_equal(yd.cpu().numpy(), ref)
    yd.fill_(np.nan)
    J.execute(J.BlockSpMVOp, A, xd, yd)               # replays the graph
    torch.cuda.synchronize()
    assert np.array_equal(yd.cpu().numpy(), ref)
    assert len(A._compiled.graphs) == 1
    x2 = np.random.default_rng(2).uniform(-1, 1, n)   # new buffers: a second graph
    y2 = torch.zeros(m, dtype=torch.float64, device=DEV)
    J.mul(y2, A, to_dev(x2))
    torch.cuda.synchronize()
    assert np.array_equal(y2.cpu().numpy(), _oracle_y(host, x2))
    assert len(A._compiled.graphs) == 2


def test_update_block_values_reaches_captured_graph():
    host, A = _blocks(np.float32)
    m, n = A.shape
    x = np.random.default_rng(3).uniform(-1, 1, n).astype(np.float32)
    xd, yd = to_dev(x), torch.zeros(m, dtype=torch.float32, device=DEV)
    J.mul(yd, A, xd)
    rp, ci, v, base = host[(2, 1)]
    nv = (v * -2.0 + 0.25).astype(np.float32)
    J.update_block_values(A, 3, 2, to_dev(nv))        # 1-based, as the reference
    host[(2, 1)] = (rp, ci, nv, base)
    J.mul(yd, A, xd)
    torch.cuda.synchronize()
    assert np.array_equal(yd.cpu().numpy(), _oracle_y(host, x))


def test_inside_callers_capture():
    host, A = _blocks()
    m, n = A.shape
    x = np.random.default_rng(4).uniform(-1, 1, n)
    xd, yd = to_dev(x), torch.zeros(m, dtype=torch.float64, device=DEV)
    J.mul(yd, A, xd)                                  # assemble before the capture
    yd.zero_()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        J.mul(yd, A, xd)
    g.replay()
    torch.cuda.synchronize()
    assert np.array_equal(yd.cpu().numpy(), _oracle_y(host, x))


def test_per_block_path_with_coo_block():
    host, A = _blocks(coo_at=(1, 1))
    assert not A.compilable()
    m, n = A.shape
    x = np.random.default_rng(5).uniform(-1, 1, n)
    yd = torch.full((m,), np.nan, dtype=torch.float64, device=DEV)
    J.mul(yd, A, to_dev(x))
    J.device_status()
    D = _dense(host)
    assert_within(yd.cpu().numpy(), D @ x, np.abs(D) @ np.abs(x), 1e-12)


def test_block_spmm():
    host, A = _blocks(np.float32)
    m, n = A.shape
    X = np.random.default_rng(6).uniform(-1, 1, (n, 16)).astype(np.float32)
    Y = torch.full((m, 16), np.nan, dtype=torch.float32, device=DEV)
    J.execute(J.BlockSpMMOp, A, to_dev(X), Y)
    J.device_status()
    D = _dense(host)
    assert_within(Y.cpu().numpy(), D @ X.astype(np.float64),
                  np.abs(D) @ np.abs(X.astype(np.float64)), 1e-5)


def test_block_banded_spmv():
    """BlockBandedMatrix y = M x (shared BlockSparseMatrix diagonal, a shared
    level-1 coupling pair, per-transition level-2 pairs): within tolerance of
    the reference's period-by-period product, and bit-exact with the oracle's
    SpMV of the same assembled CSR; a second call replays the graph."""
    T, bw, no = 6, 2, [300, 200]
    host, D = _blocks()                                # 2100 x 1400 BlockSparseMatrix
    nd, nc = D.shape
    dh_rp, dh_ci, dh_v = O.bsm_assemble(SIZES_R, SIZES_C, host)
    dh = (dh_rp, dh_ci, dh_v, 0)

    def pair(seed, rows):
        rng = np.random.default_rng(seed)
        out = []
        for s in (0, 1):
            rp, ci, v = random_csr(rows, nc, rng.integers(0, 9, rows), seed=seed + s)
            out.append(((rp, ci, v, 0), J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(v), (rows, nc),
                                                     origin=0)))
        return out
    (n1h, n1), (p1h, p1) = pair(600, no[0])
    lvl2h, lvl2 = [], []
    for t in range(T - 2):
        (ah, a), (bh, b) = pair(700 + 2 * t, no[1])
        lvl2h.append((ah, bh)), lvl2.append((a, b))
    M = J.BlockBandedMatrix(D, [(n1, p1), lvl2], T, bw, nd, no, nc)
    m, n = M.shape
    x = np.random.default_rng(8).uniform(-1, 1, n)
    xd, yd = to_dev(x), torch.full((m,), np.nan, dtype=torch.float64, device=DEV)
    J.mul(yd, M, xd)
    ref, bound = O.bbm_spmv_ref64([dh] * T, [[(n1h, p1h)] * (T - 1), lvl2h], T, bw, nd, no, nc, x)
    assert_within(yd.cpu().numpy(), ref, bound, 1e-12)
    c = M._compiled
    exact = O.spmv(c.csr.pos[1].cpu().numpy(), c.csr.crd[1].cpu().numpy(), c.val.cpu().numpy(), x)
    assert np.array_equal(yd.cpu().numpy(), exact)
    yd.fill_(np.nan)
    J.execute(J.BBMSpMVOp, M, xd, yd)
    torch.cuda.synchronize()
    assert np.array_equal(yd.cpu().numpy(), exact)


@pytest.mark.parametrize("diag_kind", ["csr", "bsm"])
def test_block_banded_periodic_kernel(diag_kind):
    """One diagonal block and one coupling pair shared over T periods (bw = 1)
    take jlb_bbm_periodic_spmv, which never stores the T-fold matrix:
    bit-exact with the oracle's restatement of JLUST's fused periodic kernel,
    within tolerance of the reference's period-by-period product."""
    from jlust_b200.block import _Periodic
    T, no = 24, 350
    if diag_kind == "csr":
        nd, nc, base = 900, 800, 1
        rng = np.random.default_rng(120)
        rp, ci, v = random_csr(nd, nc, rng.integers(0, 12, nd), seed=121, base=base)
        dh = (rp, ci, v, base)
        D = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(v), (nd, nc), origin=base)
    else:
        host, D = _blocks()
        nd, nc = D.shape
        base = 0
        dh = (*O.bsm_assemble(SIZES_R, SIZES_C, host), 0)
    pair_h, pair_d = [], []
    for s in (0, 1):
        rng = np.random.default_rng(130 + s)
        rp, ci, v = random_csr(no, nc, rng.integers(0, 7, no), seed=131 + s, base=base)
        pair_h.append((rp, ci, v, base))
        pair_d.append(J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(v), (no, nc), origin=base))
    M = J.BlockBandedMatrix(D, [tuple(pair_d)], T, 1, nd, [no], nc)
    m, n = M.shape
    x = np.random.default_rng(9).uniform(-1, 1, n)
    xd, yd = to_dev(x), torch.full((m,), np.nan, dtype=torch.float64, device=DEV)
    J.mul(yd, M, xd)
    J.device_status()
    assert isinstance(M._compiled, _Periodic)
    exact = O.bbm_periodic_spmv(T, nd, no, nc, dh[:3], pair_h[0][:3], pair_h[1][:3], x, base=base)
    assert np.array_equal(yd.cpu().numpy(), exact)
    ref, bound = O.bbm_spmv_ref64([dh] * T, [[tuple(pair_h)] * (T - 1)], T, 1, nd, [no], nc, x)
    assert_within(yd.cpu().numpy(), ref, bound, 1e-12)
    yd.fill_(np.nan)
    J.execute(J.BBMSpMVOp, M, xd, yd)                 # graph replay
    torch.cuda.synchronize()
    assert np.array_equal(yd.cpu().numpy(), exact)
