"""SDDMM on the GPU against the CPU oracle: the fast (warp-per-row) path within
the fp32 tolerance, the generic path bit-exact (sequential K loop)."""
import numpy as np
import pytest
import torch

import jlust_b200 as J
from jlust_b200 import synth
from oracle import oracle as O
from _helpers import DEV, assert_within, random_csr, to_dev

pytestmark = pytest.mark.gpu


def test_kat(golden):
    g = golden["sddmm_csr_onebased"]
    Cg = g["C"]
    Cs = J.csr_tensor(to_dev(np.array(Cg["rowptr"], np.int32)), to_dev(np.array(Cg["colind"], np.int32)),
                      to_dev(np.array(Cg["val"], np.float32)), (3, 3), origin=1)
    A = to_dev(np.array(g["A"], np.float32))
    B = to_dev(np.array(g["B"], np.float32))
    J.execute(J.SDDMMOp, A, B, Cs, beta=0.0)
    J.device_status()
    assert Cs.val.cpu().tolist() == g["out"]


@pytest.mark.parametrize("K", [128, 64, 96, 256, 512])
@pytest.mark.parametrize("mode", ["add", "mul"])
def test_fast_path(K, mode):
    rng = np.random.default_rng(41)
    m, n = 2000, 1500
    rp, ci, _ = random_csr(m, n, rng.integers(0, 70, size=m), seed=42, dtype=np.float32)
    A = rng.standard_normal((m, K), dtype=np.float32)
    Bt = rng.standard_normal((n, K), dtype=np.float32)        # row-major n x K
    S = rng.random(ci.shape[0], dtype=np.float32)
    Cs = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(S.copy()), (m, n), origin=0)
    J.execute(J.SDDMMOp, to_dev(A), to_dev(Bt).t(), Cs, alpha=1.0, beta=0.0, mode=mode)
    J.device_status()
    got = Cs.val.cpu().numpy()
    ref, bound = O.sddmm_ref64(rp, ci, A, Bt.T, out_in=S, S=S, mode=0 if mode == "add" else 1)
    assert_within(got, ref, bound, 1e-5)


def test_beta_and_alpha():
    rng = np.random.default_rng(43)
    m, n, K = 500, 400, 128
    rp, ci, _ = random_csr(m, n, rng.integers(0, 33, size=m), seed=44, dtype=np.float32)
    A = rng.standard_normal((m, K), dtype=np.float32)
    Bt = rng.standard_normal((n, K), dtype=np.float32)
    v0 = rng.random(ci.shape[0], dtype=np.float32)
    Cs = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(v0.copy()), (m, n), origin=0)
    J.execute(J.SDDMMOp, to_dev(A), to_dev(Bt).t(), Cs, alpha=-0.5, beta=2.0)
    J.device_status()
    ref, bound = O.sddmm_ref64(rp, ci, A, Bt.T, out_in=v0, mode=0, alpha=-0.5, beta=2.0)
    assert_within(Cs.val.cpu().numpy(), ref, bound, 1e-5)


@pytest.mark.parametrize("base", [0, 1])
def test_generic_path_bit_exact(base):
    """Column-major A (Julia's layout) and row-major K x n B take the generic
    kernel, which sums k = 0..K-1 in order like the reference's leaf."""
    rng = np.random.default_rng(45)
    m, n, K = 300, 200, 37
    rp, ci, _ = random_csr(m, n, rng.integers(0, 20, size=m), seed=46, base=base, dtype=np.float32)
    A = np.asfortranarray(rng.standard_normal((m, K), dtype=np.float32))
    B = rng.standard_normal((K, n), dtype=np.float32)          # row-major K x n
    v0 = rng.random(ci.shape[0], dtype=np.float32)
    Ad = torch.from_numpy(np.ascontiguousarray(A.T)).to(DEV).t()
    Cs = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(v0.copy()), (m, n), origin=base)
    J.execute(J.SDDMMOp, Ad, to_dev(B), Cs, alpha=1.25, beta=0.5)
    J.device_status()
    ref = O.sddmm(rp, ci, A, B, v0, mode=0, alpha=1.25, beta=0.5, base=base)
    assert np.array_equal(Cs.val.cpu().numpy(), ref)


def test_reduced_config4():
    rp, ci, A, B, S = synth.config4(m=65_536)
    Cs = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(S.copy()), (65_536, 65_536), origin=0)
    J.execute(J.SDDMMOp, to_dev(A), to_dev(B).t(), Cs, mode="mul")
    J.device_status()
    ref, bound = O.sddmm_ref64(rp, ci, A, B.T, S=S, mode=1)
    assert_within(Cs.val.cpu().numpy(), ref, bound, 1e-5)


@pytest.mark.parametrize("K", [128, 64, 20])
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_column_major_a_fast_path(K, dtype):
    """JLUST's native layouts: A column-major m x K and B the column-major
    K x n operand; the warp-per-row kernel reads A(i, :) with strided scalar
    loads.  Within tolerance of the fp64 restatement, both modes, beta != 0."""
    rng = np.random.default_rng(47)
    m, n = 3000, 2000
    rp, ci, _ = random_csr(m, n, rng.integers(0, 45, size=m), seed=48, dtype=dtype)
    A = np.asfortranarray(rng.standard_normal((m, K)).astype(dtype))
    Bkn = np.asfortranarray(rng.standard_normal((K, n)).astype(dtype))
    v0 = rng.random(ci.shape[0]).astype(dtype)
    Ad = torch.from_numpy(np.ascontiguousarray(A.T)).to(DEV).t()
    Bd = torch.from_numpy(np.ascontiguousarray(Bkn.T)).to(DEV).t()
    tol = 1e-5 if dtype == np.float32 else 1e-12
    for mode in ("add", "mul"):
        Cs = J.csr_tensor(to_dev(rp), to_dev(ci), to_dev(v0.copy()), (m, n), origin=0)
        J.execute(J.SDDMMOp, Ad, Bd, Cs, alpha=0.5, beta=0.25, mode=mode)
        J.device_status()
        got = Cs.val.cpu().numpy()
        if dtype == np.float64:
            # the fp64 restatement in the reference's order; the warp's sum
            # differs from it by rounding only: per entry within 1e-12 of
            # the sum of the absolute terms
            ref = O.sddmm(rp, ci, A, Bkn, v0, S=v0, mode=0 if mode == "add" else 1, alpha=0.5,
                          beta=0.25)
            rows = np.repeat(np.arange(m), np.diff(rp))
            terms = np.einsum("pk,pk->p", np.abs(A[rows]), np.abs(Bkn[:, ci].T)) * 0.5
            if mode == "mul":
                terms = terms * np.abs(v0)
            assert_within(got, ref, terms + 0.25 * np.abs(v0), tol)
        else:
            ref, bound = O.sddmm_ref64(rp, ci, A, Bkn, out_in=v0, S=v0,
                                       mode=0 if mode == "add" else 1, alpha=0.5, beta=0.25)
            assert_within(got, ref, bound, tol)
