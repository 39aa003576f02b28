"""Host-side logic of the drop-in API: formats, level maps, capability table,
tensor constructors, dense layouts and the synthetic generators."""
import numpy as np
import pytest
import torch

import jlust_b200 as J
from jlust_b200 import synth
from jlust_b200.formats import level_extents
from jlust_b200.tensor import dense_layout

F = J.Formats


def _fmt(d):
    name = d["format"]
    return getattr(F, name)(tuple(d["block"])) if "block" in d else getattr(F, name)


def test_level_maps_match_reference(golden):
    g = golden["bsr_level_maps"]
    for c in g["dim2lvl"]:
        assert J.dim2lvl(_fmt(c), c["dims"]) == c["lvl"]
    for c in g["dim2lvl_as_size"]:
        assert J.dim2lvl(_fmt(c), c["dims"], as_size=True) == c["lvl"]
    for c in g["lvl2dim"]:
        assert J.lvl2dim(_fmt(c), c["lvl"]) == c["dims"]


def test_bsr_round_trip_and_extents():
    f = F.BSRRight((4, 4))
    for i in range(0, 17):
        for j in range(0, 23):
            assert J.lvl2dim(f, J.dim2lvl(f, [i, j])) == [i, j]
    assert level_extents(f, (10, 8)) == [3, 2, 4, 4]   # ceil(10/4) block rows
    assert F.BSRRight((4, 4)) == F.BSRRight((4, 4)) and F.BSRRight((4, 4)) != F.BSRRight((2, 2))


def test_supports_backend_table():
    be = J.B200Backend()
    d1, d2 = F.DensedRight(1), F.DensedRight(2)
    assert J.supports_backend(be, J.SpMVOp(F.CSR, d1, d1))
    for fmt in (F.DCSR, F.COO, F.CSC):
        assert J.supports_backend(be, J.SpMVOp(fmt, d1, d1))
    assert not J.supports_backend(be, J.SpMVOp(F.DCSC, d1, d1))
    assert not J.supports_backend(be, J.SpMVOp(d2, d1, d1))
    assert not J.supports_backend(be, J.SpMVOp(F.CSR, d1, F.CSR))
    assert J.supports_backend(be, J.SpMMOp(F.CSR, d2, d2))
    assert J.supports_backend(be, J.SpMMOp(F.BSRRight((64, 64)), d2, d2))
    assert not J.supports_backend(be, J.SpMMOp(d2, d2, d2))
    assert J.supports_backend(be, J.SDDMMOp(d2, d2, F.CSR))
    assert not J.supports_backend(be, J.SDDMMOp(F.CSR, d2, F.CSR))
    assert J.supports_backend(be, J.BlockSpMMOp(F.BSRRight((64, 64)), d2, d2))
    assert not J.supports_backend(be, J.SpSVOp(F.CSR, d1, d1))
    assert J.supports_backend(be, J.SpGEMMOp(F.CSR, F.CSR, F.CSR))
    assert not J.supports_backend(be, J.SpGEMMOp(F.CSC, F.CSC, F.CSC))
    assert not J.supports_backend(be, J.SpGEMMOp(F.CSR, F.CSC, F.CSR))


def test_constructors_validate_shapes():
    rp = torch.tensor([0, 2, 3], dtype=torch.int32)
    ci = torch.tensor([0, 1, 1], dtype=torch.int32)
    v = torch.ones(3)
    A = J.csr_tensor(rp, ci, v, (2, 2), origin=J.ZeroBased())
    assert J.positions(A, 2) is rp and J.coordinates(A, 2) is ci and J.nnz(A) == 3
    with pytest.raises(J.InvalidLevelAccess):
        J.positions(A, 1)
    with pytest.raises(J.IncompatibleExtents):
        J.csr_tensor(rp, ci, v, (3, 2))
    with pytest.raises(J.UnsupportedIndexType):
        J.csr_tensor(rp.long(), ci, v, (2, 2))


def test_no_cpu_fallback():
    A = J.csr_tensor(torch.tensor([0, 1], dtype=torch.int32), torch.tensor([0], dtype=torch.int32),
                     torch.ones(1, dtype=torch.float64), (1, 1), origin=0)
    with pytest.raises(J.DeviceMismatch):
        J.execute(J.SpMVOp, A, torch.ones(1, dtype=torch.float64), torch.zeros(1, dtype=torch.float64))
    with pytest.raises(J.UnsupportedFormat):
        J.execute(J.SpMVOp, A, torch.ones(1, dtype=torch.float64),
                  torch.zeros(1, dtype=torch.float64), input_fn=abs)


def test_dense_layouts():
    a = torch.zeros(5, 7)
    assert dense_layout(a) == (0, 7)
    assert dense_layout(a.t()) == (1, 7)
    assert dense_layout(torch.zeros(10, 8)[:, :4]) == (0, 8)
    assert dense_layout(torch.zeros(10, 8)[::2]) == (0, 16)
    assert dense_layout(torch.zeros(4, 4, 4)) is None


def test_bf16_rounding_is_rne():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e-39, 65504.0], np.float32)
    bits = synth.f32_to_bf16_bits(x)
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(bits, ref)
    assert np.array_equal(synth.bf16_bits_to_f32(bits), torch.from_numpy(x).to(torch.bfloat16).float().numpy())


def test_laplacian_shape():
    rp, ci, v = synth.laplacian_2d(64)
    n = 64 * 64
    assert rp[-1] == 5 * n - 4 * 64 == ci.shape[0]
    assert np.all(np.diff(rp) >= 3) and np.all(np.diff(rp) <= 5)
    row = np.repeat(np.arange(n), np.diff(rp))
    assert np.all(v[ci == row] == 4.0) and np.all(v[ci != row] == -1.0)
    # columns strictly increasing inside each row
    d = np.diff(ci)
    starts = rp[1:-1]
    d[starts - 1] = 1
    assert np.all(d > 0)


def test_uniform_rows_distinct_sorted():
    rp, ci, _ = synth.uniform_rows(1000, 50, 10, seed=1)
    rows = ci.reshape(1000, 10)
    assert np.all(np.diff(rows, axis=1) > 0)
    assert rows.min() >= 0 and rows.max() < 50


def test_power_law_degrees():
    rp, ci, _ = synth.power_law(200_000, 1 << 22, 2.0, 4096, seed=2)
    deg = np.diff(rp)
    assert deg.min() >= 1 and deg.max() <= 4096
    assert 4.5 < deg.mean() < 6.5            # truncated Zipf(2) mean is about 5.4
    assert abs((deg == 1).mean() - 0.6079) < 0.01


def test_block_banded_pattern():
    bp, bc, _ = synth.block_banded(64, 8, 0.02, seed=4)
    for I in range(64):
        js = bc[bp[I]:bp[I + 1]]
        assert np.all(np.diff(js) > 0)
        assert set(range(max(0, I - 8), min(64, I + 9))) <= set(js.tolist())


def test_spgemm_handle_validation():
    """The SpGEMM handle's checks run before any device work: transposed
    operands and beta != 0 are refused as in the reference's prepare
    (KA spgemm.jl:313-323), and inner extents must agree."""
    z = torch.zeros(0, dtype=torch.int32)
    A = J.csr_tensor(torch.zeros(5, dtype=torch.int32), z, torch.zeros(0, dtype=torch.float64),
                     (4, 3), origin=0)
    be = J.B200Backend()
    with pytest.raises(J.UnsupportedFormat):
        J.prepare(be, J.SpGEMMOp, A, A, transa="T")
    with pytest.raises(J.UnsupportedFormat):
        J.prepare(be, J.SpGEMMOp, A, A, beta=1.0)
    with pytest.raises(J.IncompatibleExtents):
        J.prepare(be, J.SpGEMMOp, A, A)


def test_conversion_and_selector_host_checks():
    """Host-side refusals that come before any device work: conversions the
    backend does not run, and a ShiftedDiag tensor whose shifted diagonal
    leaves its columns."""
    bsr = J.bsr_tensor(torch.zeros(3, dtype=torch.int32), torch.zeros(0, dtype=torch.int32),
                       torch.zeros(0, dtype=torch.float32), (4, 4), (2, 2), origin=0)
    with pytest.raises(J.UnsupportedFormat):
        J.convert_format(bsr, J.Formats.CSC)
    csr = J.csr_tensor(torch.zeros(4, dtype=torch.int32), torch.zeros(0, dtype=torch.int32),
                       torch.zeros(0, dtype=torch.float64), (3, 3), origin=0)
    with pytest.raises(J.UnsupportedFormat):
        J.convert_format(csr, J.Formats.DCSR)
    S = J.shifted_diag_tensor(torch.float64, 4, 5, shift=2)
    with pytest.raises(J.IncompatibleExtents):
        J.execute(J.SpMVOp, S, torch.zeros(5, dtype=torch.float64), torch.zeros(4, dtype=torch.float64),
                  backend=J.B200Backend())
    d1 = J.Formats.DensedRight(1)
    assert J.supports_backend(J.B200Backend(), J.SpMVOp(S.format, d1, d1))
