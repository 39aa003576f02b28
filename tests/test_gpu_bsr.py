"""BSR SpMM on tcgen05 tensor cores against the CPU oracle (fp64 reference,
inputs are exact bf16 so only the fp32 accumulation order differs), and the
SIMT kernel for other block sizes bit-exact against the fp32 oracle."""
import numpy as np
import pytest
import torch

import jlust_b200 as J
from jlust_b200 import synth
from oracle import oracle as O
from _helpers import DEV, assert_within, bf16_dev, to_dev

pytestmark = pytest.mark.gpu


def run(bp, bc, bv, B, bs, nbr_rows, nbr_cols, Y0=None, alpha=1.0, beta=0.0, base=0):
    A = J.bsr_tensor(to_dev(bp + base), to_dev(bc + base), bf16_dev(bv),
                     (nbr_rows * bs, nbr_cols * bs), (bs, bs), origin=base)
    N = B.shape[1]
    Y = torch.from_numpy(Y0.copy()).to(DEV) if Y0 is not None else \
        torch.full((nbr_rows * bs, N), float("nan"), dtype=torch.float32, device=DEV)
    J.execute(J.BlockSpMMOp, A, bf16_dev(B), Y, alpha=alpha, beta=beta)
    J.device_status()
    return Y.cpu().numpy()


@pytest.mark.parametrize("N", [128, 256, 384, 512])
def test_tensor_path(N):
    bp, bc, bv, B = synth.config5(seed=51, nbr=40, band=3, p_off=0.1, N=N)
    got = run(bp, bc, bv, B, 64, 40, 40)
    ref, bound = O.bsr_spmm_ref64(bp, bc, bv, B)
    assert_within(got, ref, bound, 1e-5)


def test_tensor_path_empty_rows_alpha_beta():
    rng = np.random.default_rng(52)
    nbr = 24
    present = rng.random((nbr, nbr)) < 0.15
    present[[0, 3, 6, 7, 17, 23]] = False                    # empty block rows (6, 7: a whole pair)
    bp = np.zeros(nbr + 1, np.int32)
    bp[1:] = np.cumsum(present.sum(axis=1))
    bc = np.nonzero(present)[1].astype(np.int32)
    bv = synth.f32_to_bf16_bits(rng.standard_normal(bc.shape[0] * 4096, dtype=np.float32))
    B = synth.f32_to_bf16_bits(rng.standard_normal((nbr * 64, 256), dtype=np.float32))
    Y0 = rng.standard_normal((nbr * 64, 256), dtype=np.float32)
    for base in (0, 1):
        got = run(bp, bc, bv, B, 64, nbr, nbr, Y0, alpha=0.5, beta=-2.0, base=base)
        ref, bound = O.bsr_spmm_ref64(bp, bc, bv, B, Y=Y0, alpha=0.5, beta=-2.0)
        assert_within(got, ref, bound, 1e-5)


def test_many_blocks_per_row():
    """Rows with more blocks than pipeline stages, and more rows than SMs."""
    bp, bc, bv, B = synth.config5(seed=53, nbr=320, band=20, p_off=0.05, N=256)
    got = run(bp, bc, bv, B, 64, 320, 320)
    ref, bound = O.bsr_spmm_ref64(bp, bc, bv, B)
    assert_within(got, ref, bound, 1e-5)


@pytest.mark.parametrize("bs,N", [(16, 40), (8, 128), (64, 96)])
def test_simt_path_bit_exact(bs, N):
    bp, bc, bv, B = synth.config5(seed=54, nbr=30, bs=bs, band=2, p_off=0.1, N=N)
    got = run(bp, bc, bv, B, bs, 30, 30, alpha=1.0)
    ref = O.bsr_spmm(bp, bc, bv, B, b1=bs, b2=bs)
    assert np.array_equal(got, ref)


def test_reduced_config5():
    """Config-5 structure (band +-8, 2% off-band, N = 256) at 1/4 of the block rows."""
    bp, bc, bv, B = synth.config5(nbr=256)
    got = run(bp, bc, bv, B, 64, 256, 256)
    ref, bound = O.bsr_spmm_ref64(bp, bc, bv, B)
    assert_within(got, ref, bound, 1e-5)
    f32 = O.bsr_spmm(bp, bc, bv, B)
    assert np.linalg.norm(got - f32) / np.linalg.norm(f32) < 1e-5


@pytest.mark.parametrize("nbr_rows,nbr_cols,N", [(41, 37, 64), (41, 37, 192), (33, 50, 320), (1, 5, 256), (41, 37, 256)])
def test_shapes_and_order(nbr_rows, nbr_cols, N):
    """Odd and rectangular block grids, N that the tensor path does not take
    (64, 192, 320: the SIMT kernel) and that it does (256), runs of empty
    block rows, and block columns stored out of order inside a row."""
    rng = np.random.default_rng(55 + N)
    present = rng.random((nbr_rows, nbr_cols)) < 0.2
    if nbr_rows > 6:
        present[[2, 3, 6]] = False                            # empty block rows
    bp = np.zeros(nbr_rows + 1, np.int32)
    bp[1:] = np.cumsum(present.sum(axis=1))
    bc = np.nonzero(present)[1].astype(np.int32)
    for r in range(0, nbr_rows, 5):                           # unsorted columns in some rows
        seg = bc[bp[r]:bp[r + 1]]
        bc[bp[r]:bp[r + 1]] = seg[::-1]
    bv = synth.f32_to_bf16_bits(rng.standard_normal(bc.shape[0] * 4096, dtype=np.float32))
    B = synth.f32_to_bf16_bits(rng.standard_normal((nbr_cols * 64, N), dtype=np.float32))
    Y0 = rng.standard_normal((nbr_rows * 64, N), dtype=np.float32)
    got = run(bp, bc, bv, B, 64, nbr_rows, nbr_cols, Y0, alpha=1.5, beta=0.25)
    ref, bound = O.bsr_spmm_ref64(bp, bc, bv, B, Y=Y0, alpha=1.5, beta=0.25)
    assert_within(got, ref, bound, 1e-5)
