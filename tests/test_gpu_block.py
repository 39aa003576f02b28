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


def _patched_matrix(dtype=np.float64):
    """The LAYOUT blocks with the (0, 1) block replaced by a CSR block that
    is 2.5 times the identity (a selector) and a ShiftedDiag block (shift 50,
    value -0.75) added at (1, 0): the compile keeps two patches."""
    host, _ = _blocks(dtype)
    blocks = [[None] * len(SIZES_C) for _ in SIZES_R]
    for (i, j), (rp, ci, v, base) in host.items():
        blocks[i][j] = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(v), (SIZES_R[i], SIZES_C[j]),
                                    origin=base)
    m01 = SIZES_R[0]
    sel = (np.arange(m01 + 1, dtype=np.int32) + 1, np.arange(m01, dtype=np.int32) + 1,
           np.full(m01, 2.5, dtype), 1)
    host[(0, 1)] = sel
    blocks[0][1] = J.csr_tensor(to_dev(sel[0]), to_dev(sel[1]), to_dev(sel[2]),
                                (m01, SIZES_C[1]), origin=1)
    dt = torch.float64 if dtype == np.float64 else torch.float32
    blocks[1][0] = J.shifted_diag_tensor(dt, SIZES_R[1], SIZES_C[0], shift=50, val=-0.75,
                                         device=DEV)
    return host, {(1, 0): (50, -0.75)}, J.BlockSparseMatrix(blocks)


@pytest.mark.parametrize("dtype", [np.float64, np.float32])
def test_selector_patches_bit_exact(dtype):
    """A ShiftedDiag block and a CSR block that is 2.5 times the identity are
    kept out of the assembled CSR as selector patches: bit-exact with the
    oracle's restatement of the reference's patched kernel, within tolerance
    of fp64, also on graph replay and after update_block_values turns the
    selector block back into an ordinary one."""
    host, shifted, A = _patched_matrix(dtype)
    m, n = A.shape
    x = np.random.default_rng(11).uniform(-1, 1, n).astype(dtype)
    xd = to_dev(x)
    yd = torch.full((m,), np.nan, dtype=xd.dtype, device=DEV)
    J.mul(yd, A, xd)
    J.device_status()
    rp, ci, v, patches = O.bsm_compile(SIZES_R, SIZES_C, host, shifted)
    assert sorted(p[:3] for p in patches) == [(0, SIZES_R[0] - 1, SIZES_C[0]),
                                              (SIZES_R[0], SIZES_R[0] + SIZES_R[1] - 1, 50)]
    assert len(A._compiled.patches) == 2
    exact = O.csr_patched_spmv(rp, ci, v, patches, x)
    assert np.array_equal(yd.cpu().numpy(), exact)
    D = _dense({k: b for k, b in host.items()}, np.float64)
    r1, c0 = SIZES_R[0], 50
    D[r1 + np.arange(SIZES_R[1]), c0 + np.arange(SIZES_R[1])] += -0.75
    assert_within(yd.cpu().numpy(), D @ x.astype(np.float64),
                  np.abs(D) @ np.abs(x.astype(np.float64)), TOL_BLOCK[dtype])
    yd.fill_(np.nan)
    J.execute(J.BlockSpMVOp, A, xd, yd)                # graph replay
    torch.cuda.synchronize()
    assert np.array_equal(yd.cpu().numpy(), exact)
    # new values that are no longer constant: the block leaves the patches
    nv = np.linspace(1, 2, SIZES_R[0]).astype(dtype)
    J.update_block_values(A, 1, 2, to_dev(nv))
    host[(0, 1)] = (*host[(0, 1)][:2], nv, 1)
    J.mul(yd, A, xd)
    torch.cuda.synchronize()
    assert len(A._compiled.patches) == 1
    rp, ci, v, patches = O.bsm_compile(SIZES_R, SIZES_C, host, shifted)
    assert np.array_equal(yd.cpu().numpy(), O.csr_patched_spmv(rp, ci, v, patches, x))


TOL_BLOCK = {np.float64: 1e-12, np.float32: 1e-5}


@pytest.mark.parametrize("ab", [(1.0, 0.0), (-1.5, 0.5)])
def test_shifted_diag_standalone_spmv(ab):
    """y = alpha S x + beta y for a ShiftedDiag tensor alone: bit-exact with
    the oracle (one patch, no CSR entries)."""
    m, n, shift, val = 3000, 3400, 123, 1.25
    S = J.shifted_diag_tensor(torch.float64, m, n, shift=shift, val=val, device=DEV)
    rng = np.random.default_rng(12)
    x, y0 = rng.uniform(-1, 1, n), rng.uniform(-1, 1, m)
    y = to_dev(y0)
    J.execute(J.SpMVOp, S, to_dev(x), y, alpha=ab[0], beta=ab[1])
    J.device_status()
    ref = O.csr_patched_spmv(np.zeros(m + 1, np.int64), np.zeros(0, np.int64), np.zeros(0),
                             [(0, m - 1, shift, val)], x, y0, beta=ab[1], alpha=ab[0])
    assert np.array_equal(y.cpu().numpy(), ref)
    with pytest.raises(J.IncompatibleExtents):
        J.execute(J.SpMVOp, J.shifted_diag_tensor(torch.float64, m, n, shift=500, device=DEV),
                  to_dev(x), y)


@pytest.mark.parametrize("dtype", [np.float64, np.float32])
def test_block_banded_periodic_with_selectors(dtype):
    """The reference's periodic case with selectors: a BlockSparseMatrix
    diagonal holding a ShiftedDiag block and a CSR selector (kept as patches
    and added per period with the period's column offset) and a coupling pair
    of a ShiftedDiag neg and a CSR pos: bit-exact with the oracle's
    restatement of the fused periodic kernel, within tolerance of fp64."""
    from jlust_b200.block import _Periodic
    T, no = 12, 400
    host, shifted, D = _patched_matrix(dtype)
    nd, nc = D.shape
    rp, ci, v, patches = O.bsm_compile(SIZES_R, SIZES_C, host, shifted)
    rng = np.random.default_rng(140)
    prp, pci, pv = random_csr(no, nc, rng.integers(0, 7, no), seed=141, dtype=dtype)
    pos = J.csr_tensor(to_dev(prp), to_dev(pci), to_dev(pv), (no, nc), origin=0)
    dt = torch.float64 if dtype == np.float64 else torch.float32
    neg = J.shifted_diag_tensor(dt, no, nc, shift=17, val=-1.0, device=DEV)
    M = J.BlockBandedMatrix(D, [(neg, pos)], T, 1, nd, [no], nc)
    m, n = M.shape
    x = np.random.default_rng(10).uniform(-1, 1, n).astype(dtype)
    xd = to_dev(x)
    yd = torch.full((m,), np.nan, dtype=dt, device=DEV)
    J.mul(yd, M, xd)
    J.device_status()
    assert isinstance(M._compiled, _Periodic) and len(M._compiled.patches) == 2
    exact = O.bbm_periodic_spmv(T, nd, no, nc, (rp, ci, v), ("shifted", 17, -1.0),
                                (prp, pci, pv), x, patches=patches)
    assert np.array_equal(yd.cpu().numpy(), exact)
    # fp64 reference: the dense diagonal and coupling blocks period by period
    Dd = _dense(host)
    Dd[SIZES_R[0] + np.arange(SIZES_R[1]), 50 + np.arange(SIZES_R[1])] += -0.75
    Nd = np.zeros((no, nc))
    Nd[np.arange(no), 17 + np.arange(no)] = -1.0
    Pd = np.zeros((no, nc))
    for r in range(no):
        Pd[r, pci[prp[r]:prp[r + 1]]] += pv[prp[r]:prp[r + 1]]
    xs = x.astype(np.float64).reshape(T, nc)
    ref, bound = [], []
    for t in range(T):
        ref.append(Dd @ xs[t]), bound.append(np.abs(Dd) @ np.abs(xs[t]))
        if t < T - 1:
            ref.append(Nd @ xs[t] + Pd @ xs[t + 1])
            bound.append(np.abs(Nd) @ np.abs(xs[t]) + np.abs(Pd) @ np.abs(xs[t + 1]))
    assert_within(yd.cpu().numpy(), np.concatenate(ref), np.concatenate(bound), TOL_BLOCK[dtype])
    yd.fill_(np.nan)
    J.execute(J.BBMSpMVOp, M, xd, yd)                 # graph replay
    torch.cuda.synchronize()
    assert np.array_equal(yd.cpu().numpy(), exact)


def test_block_banded_assembled_with_shifted_diag():
    """A BlockBandedMatrix that is not periodic (per-transition pairs) with
    ShiftedDiag coupling blocks: the ShiftedDiag blocks become selector
    patches of the assembled CSR; within tolerance of fp64."""
    T, nd, no, nc = 4, 600, 250, 700
    rng = np.random.default_rng(150)
    rp, ci, v = random_csr(nd, nc, rng.integers(0, 10, nd), seed=151)
    D = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(v), (nd, nc), origin=0)
    pairs, dense_pairs = [], []
    for t in range(T - 1):
        prp, pci, pv = random_csr(no, nc, rng.integers(0, 6, no), seed=160 + t)
        pos = J.csr_tensor(to_dev(prp), to_dev(pci), to_dev(pv), (no, nc), origin=0)
        neg = J.shifted_diag_tensor(torch.float64, no, nc, shift=t * 10, val=0.5 + t, device=DEV)
        pairs.append((neg, pos))
        Nd, Pd = np.zeros((no, nc)), np.zeros((no, nc))
        Nd[np.arange(no), t * 10 + np.arange(no)] = 0.5 + t
        for r in range(no):
            Pd[r, pci[prp[r]:prp[r + 1]]] += pv[prp[r]:prp[r + 1]]
        dense_pairs.append((Nd, Pd))
    M = J.BlockBandedMatrix(D, [pairs], T, 1, nd, [no], nc)
    m, n = M.shape
    x = np.random.default_rng(13).uniform(-1, 1, n)
    yd = torch.full((m,), np.nan, dtype=torch.float64, device=DEV)
    J.mul(yd, M, to_dev(x))
    J.device_status()
    assert len(M._compiled.patches) == T - 1
    Dd = np.zeros((nd, nc))
    for r in range(nd):
        Dd[r, ci[rp[r]:rp[r + 1]]] += v[rp[r]:rp[r + 1]]
    xs = x.reshape(T, nc)
    ref, bound = [], []
    for t in range(T):
        ref.append(Dd @ xs[t]), bound.append(np.abs(Dd) @ np.abs(xs[t]))
        if t < T - 1:
            Nd, Pd = dense_pairs[t]
            ref.append(Nd @ xs[t] + Pd @ xs[t + 1])
            bound.append(np.abs(Nd) @ np.abs(xs[t]) + np.abs(Pd) @ np.abs(xs[t + 1]))
    assert_within(yd.cpu().numpy(), np.concatenate(ref), np.concatenate(bound), 1e-12)


# ---- the reference's own block-path tests (test/test_emitter_cuda.jl) ------
def _kat_bsm(g):
    nbr, nbc = g["grid"]
    grid = [[None] * nbc for _ in range(nbr)]
    for key, b in g["blocks"].items():
        i, j = map(int, key.split(","))
        grid[i][j] = J.csr_tensor(to_dev(np.array(b["rowptr"], np.int32)),
                                  to_dev(np.array(b["colind"], np.int32)),
                                  to_dev(np.array(b["val"])), (b["m"], b["n"]), origin=b["base"])
    return J.BlockSparseMatrix(grid)


@pytest.mark.parametrize("name", ["bsm_diagonal", "bsm_accumulate"])
def test_reference_bsm_kats(golden, name):
    """BlockSparseMatrix diagonal [7, 6, 5, 10] and accumulate [9, 10]
    (test/test_emitter_cuda.jl:297-322): mul! and a second product on the
    same buffers (graph replay) give the reference's vectors exactly."""
    g = golden[name]
    A = _kat_bsm(g)
    x = to_dev(np.array(g["x"]))
    y = torch.zeros(A.shape[0], dtype=torch.float64, device=DEV)
    for _ in range(2):
        J.mul(y, A, x)
        J.device_status()
        assert y.cpu().tolist() == g["y"]


def test_reference_shifted_diag_standalone():
    """shifted_diag_tensor SpMV (test/test_emitter_cuda.jl:330-345): shift 0,
    val 2.5 gives 2.5 x; an n x (n+3) tensor with shift 3, val -1.5 gives
    -1.5 x[3:]."""
    n = 1024
    x = torch.rand(n, dtype=torch.float64, device=DEV)
    y = torch.zeros(n, dtype=torch.float64, device=DEV)
    J.execute(J.SpMVOp, J.shifted_diag_tensor(torch.float64, n, n, shift=0, val=2.5, device=DEV),
              x, y)
    J.device_status()
    assert torch.equal(y, 2.5 * x)
    x2 = torch.rand(n + 3, dtype=torch.float64, device=DEV)
    y2 = torch.zeros(n, dtype=torch.float64, device=DEV)
    J.execute(J.SpMVOp, J.shifted_diag_tensor(torch.float64, n, n + 3, shift=3, val=-1.5,
                                               device=DEV), x2, y2)
    J.device_status()
    assert torch.equal(y2, -1.5 * x2[3:])


def _eye_csr(n, v):
    return J.csr_tensor(to_dev(np.arange(1, n + 2, dtype=np.int32)),
                        to_dev(np.arange(1, n + 1, dtype=np.int32)), to_dev(np.full(n, v)),
                        (n, n), origin=1)


def test_reference_bsm_shifted_diag_equivalence():
    """A CSR -I block and a ShiftedDiag(-I) block give the same product
    (test/test_emitter_cuda.jl:348-368), and [3I -I 2I] with two ShiftedDiag
    blocks gives 3 x1 - x2 + 2 x3 (:370-382)."""
    n = 16
    A = _eye_csr(n, 2.0)
    B_csr = J.BlockSparseMatrix([[A, _eye_csr(n, -1.0)]])
    B_sh = J.BlockSparseMatrix([[A, J.shifted_diag_tensor(torch.float64, n, n, val=-1.0,
                                                           device=DEV)]])
    x = torch.rand(2 * n, dtype=torch.float64, device=DEV)
    y1 = torch.zeros(n, dtype=torch.float64, device=DEV)
    y2 = torch.zeros(n, dtype=torch.float64, device=DEV)
    J.mul(y1, B_csr, x)
    J.mul(y2, B_sh, x)
    J.device_status()
    assert torch.equal(y1, y2)
    n = 8
    M = J.BlockSparseMatrix([[_eye_csr(n, 3.0),
                              J.shifted_diag_tensor(torch.float64, n, n, val=-1.0, device=DEV),
                              J.shifted_diag_tensor(torch.float64, n, n, val=2.0, device=DEV)]])
    x = torch.rand(3 * n, dtype=torch.float64, device=DEV)
    y = torch.zeros(n, dtype=torch.float64, device=DEV)
    J.mul(y, M, x)
    J.device_status()
    xh = x.cpu().numpy()
    want = 3.0 * xh[:n] - xh[n:2 * n] + 2.0 * xh[2 * n:]
    assert np.allclose(y.cpu().numpy(), want, rtol=1e-15, atol=1e-15)


def test_reference_bbm_periodic_shifted_diag_equivalence():
    """BlockBandedMatrix (bw = 1 form) whose BlockSparseMatrix diagonal holds
    a CSR -I block or a ShiftedDiag(-I) block, with a (-R, R) coupling pair
    (test/test_emitter_cuda.jl:384-418): identical products -- the CSR -I is
    recognised as a selector and both run as the same patch."""
    n, T = 16, 4
    A = _eye_csr(n, 3.0)
    bsm_csr = J.BlockSparseMatrix([[A, _eye_csr(n, -1.0)]])
    bsm_sh = J.BlockSparseMatrix([[A, J.shifted_diag_tensor(torch.float64, n, n, val=-1.0,
                                                             device=DEV)]])
    negR, R = _eye_csr(n, -1.0), _eye_csr(n, 1.0)
    M_csr = J.BlockBandedMatrix(bsm_csr, negR, R, T, n, n, 2 * n)
    M_sh = J.BlockBandedMatrix(bsm_sh, negR, R, T, n, n, 2 * n)
    n_total = T * n + (T - 1) * n
    assert M_csr.shape == (n_total, T * 2 * n)
    x = torch.rand(T * 2 * n, dtype=torch.float64, device=DEV)
    y1 = torch.zeros(n_total, dtype=torch.float64, device=DEV)
    y2 = torch.zeros(n_total, dtype=torch.float64, device=DEV)
    J.mul(y1, M_csr, x)
    J.mul(y2, M_sh, x)
    J.device_status()
    assert torch.equal(y1, y2)
