"""Parity at the benchmark configurations' full sizes (the inputs bench.py
times), against the CPU oracle on the same seeded inputs:

* cfg2: 20 iterations x <- A x on the 4096^2 Laplacian, bit-exact;
* cfg3: C = A B on the 4M-row power-law matrix, k = 64: rows of at most 256
  entries bit-exact, longer rows within 1e-5 of the fp64 restatement;
* cfg4: the 1M^2 SDDMM in the sampled-product mode (out = dot * S) and in the
  reference's additive mode (alpha * dot + beta * nz), within 1e-5;
* cfg5: the 65,536^2 BSR SpMM (1024 block rows), within 1e-5 of the fp64
  restatement of the block-SpMM loop (src/block_sparse.jl:177-188);
* CSR -> BSR of the whole cfg5 matrix, byte-exact: against the BSR the CSR
  was expanded from, and on the first 1/32 of the block rows against the
  oracle's composer (src/convert.jl:302-388).
"""
import numpy as np
import pytest
import torch

import jlust_b200 as J
from jlust_b200 import synth
from oracle import oracle as O
from _helpers import DEV, assert_within, bf16_dev, to_dev

pytestmark = pytest.mark.gpu


def _free():
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def test_cfg2_laplacian_20_iterations():
    g = 4096
    rp, ci, val, x = synth.config2(g=g)
    n = g * g
    A = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(val), (n, n), origin=0)
    xa, xb = to_dev(x), torch.empty(n, dtype=torch.float64, device=DEV)
    xr = x.copy()
    for _ in range(20):
        J.execute(J.SpMVOp, A, xa, xb)
        xa, xb = xb, xa
        xr = O.spmv(rp, ci, val, xr)
    J.device_status()
    assert np.array_equal(xa.cpu().numpy(), xr)
    del A, xa, xb
    _free()


def test_cfg3_spmm_full():
    rp, ci, val, B = synth.config3()
    m = rp.shape[0] - 1
    A = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(val), (m, m), origin=0)
    Cd = torch.zeros(m, B.shape[1], dtype=torch.float32, device=DEV)
    J.execute(J.SpMMOp, A, to_dev(B), Cd)
    J.device_status()
    got = Cd.cpu().numpy()
    del A, Cd
    _free()
    lens = np.diff(rp)
    short = lens <= 256
    assert np.array_equal(got[short], O.spmm(rp, ci, val, B)[short])
    longr = np.nonzero(~short)[0]
    assert longr.size > 0
    sub_rp = np.concatenate([[0], np.cumsum(lens[longr])]).astype(np.int32)
    idx = np.concatenate([np.arange(rp[r], rp[r + 1]) for r in longr])
    ref, bound = O.spmm_ref64(sub_rp, ci[idx], val[idx], B)
    assert_within(got[longr], ref, bound, 1e-5)


@pytest.mark.parametrize("mode", ["mul", "add"])
def test_cfg4_sddmm_full(mode):
    rp, ci, A, B, S = synth.config4()
    m = rp.shape[0] - 1
    Cs = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(S.copy()), (m, m), origin=0)
    Sd = to_dev(S)
    if mode == "mul":
        J.execute(J.SDDMMOp, to_dev(A), to_dev(B).t(), Cs, mode="mul", S=Sd)
        ref, bound = O.sddmm_ref64(rp, ci, A, B.T, S=S, mode=1)
    else:
        J.execute(J.SDDMMOp, to_dev(A), to_dev(B).t(), Cs, alpha=0.75, beta=0.5)
        ref, bound = O.sddmm_ref64(rp, ci, A, B.T, out_in=S, mode=0, alpha=0.75, beta=0.5)
    J.device_status()
    got = Cs.val.cpu().numpy()
    del Cs, Sd
    _free()
    assert_within(got, ref, bound, 1e-5)


def test_cfg5_bsr_full():
    bp, bc, bv, B = synth.config5()
    mb = bp.shape[0] - 1
    n = mb * 64
    A = J.bsr_tensor(to_dev(bp), to_dev(bc), bf16_dev(bv), (n, n), (64, 64), origin=0)
    Y = torch.zeros(n, B.shape[1], dtype=torch.float32, device=DEV)
    J.execute(J.BlockSpMMOp, A, bf16_dev(B), Y)
    J.device_status()
    got = Y.cpu().numpy()
    del A, Y
    _free()
    ref, bound = O.bsr_spmm_ref64(bp, bc, bv, B)
    assert_within(got, ref, bound, 1e-5)


def test_cfg5_csr_to_bsr_full():
    bp, bc, bv, _ = synth.config5(N=64)
    mb = bp.shape[0] - 1
    rp, ci, vals = synth.bsr_to_csr(bp, bc, bv, 64, mb)
    m = rp.shape[0] - 1
    A = J.csr_tensor(to_dev(rp), to_dev(ci), bf16_dev(vals), (m, m), origin=0)
    out = J.convert_format(A, J.Formats.BSRRight((64, 64)))
    J.device_status()
    gp = J.positions(out, 2).cpu().numpy()
    gc = J.coordinates(out, 2).cpu().numpy()
    gv = out.val.view(torch.int16).cpu().numpy().view(np.uint16)
    del A, out
    _free()
    assert np.array_equal(gp, bp) and np.array_equal(gc, bc)
    assert np.array_equal(gv, np.where((bv & 0x7FFF) == 0, np.uint16(0), bv))
    rows = (mb // 32) * 64
    op, oc, ov = O.csr_to_bsr(rows, m, rp[:rows + 1], ci, vals, 64, 64)
    nb = int(op[-1])
    assert np.array_equal(gp[:mb // 32 + 1], op)
    assert np.array_equal(gc[:nb], oc)
    assert np.array_equal(gv[:nb * 4096], ov)
