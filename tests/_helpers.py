"""Shared helpers of the GPU parity tests."""
import numpy as np
import torch

DEV = "cuda:0"


def to_dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(DEV)


def bf16_dev(bits):
    """uint16 bf16 bit patterns -> torch.bfloat16 on the device."""
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(DEV)


def assert_within(got, ref64, bound, tol):
    """Per element |got - ref| <= tol * bound (bound = sum of |terms|), plus the
    normwise relative error of the reference's benchmarks
    (benchmark/bench_suitesparse.jl:263-264) <= tol."""
    got = np.asarray(got, dtype=np.float64)
    err = np.abs(got - ref64)
    lim = tol * np.asarray(bound) + 1e-300
    bad = np.nonzero(err > lim)[0] if err.ndim == 1 else np.argwhere(err > lim)
    assert bad.size == 0, f"{bad.shape[0]} elements out of tolerance, first {bad[:3]}: " \
                          f"got {got.flat[0]} ..."
    nr = np.linalg.norm(ref64)
    if nr > 0:
        assert np.linalg.norm(got - ref64) / nr <= tol


def random_csr(m, n, lengths, seed, base=0, dtype=np.float64, zero_frac=0.0):
    """CSR with the given row lengths (array of m ints), distinct sorted columns."""
    rng = np.random.default_rng(seed)
    lengths = np.minimum(np.asarray(lengths, np.int64), n)
    cols = [np.sort(rng.choice(n, size=int(L), replace=False)) if L else np.zeros(0, np.int64)
            for L in lengths]
    rowptr = np.zeros(m + 1, np.int64)
    np.cumsum(lengths, out=rowptr[1:])
    colind = np.concatenate(cols).astype(np.int32) if m else np.zeros(0, np.int32)
    val = rng.uniform(-1, 1, size=colind.shape[0]).astype(dtype)
    if zero_frac:
        val[rng.random(val.shape[0]) < zero_frac] = 0
    return (rowptr + base).astype(np.int32), (colind + base).astype(np.int32), val
