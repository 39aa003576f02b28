"""Seeded synthetic inputs with the shapes, sizes and value distributions of
the benchmark configurations (the reference benchmarks on downloaded
SuiteSparse / power-grid cases that are not available here; these generators
stand in for them).  All randomness comes from numpy's PCG64 generator
(`numpy.random.default_rng(seed)`), so "seed s" means that generator seeded
with s.  Every function returns host numpy arrays; CSR outputs are canonical
(row pointer from 0, columns strictly increasing within a row).
"""
from __future__ import annotations

import numpy as np


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 (round to nearest even) and return the bits as
    uint16.  NaN inputs become a quiet NaN."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32)
    t = u >> np.uint32(16)              # in-place steps: no full-size temporaries
    t &= np.uint32(1)
    t += np.uint32(0x7FFF)
    t += u
    t >>= np.uint32(16)
    out = t.astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.uint16(0x7FC0)
    return out


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def _rowptr_from_counts(counts: np.ndarray) -> np.ndarray:
    rp = np.zeros(counts.shape[0] + 1, dtype=np.int64)
    np.cumsum(counts, out=rp[1:])
    if rp[-1] > np.iinfo(np.int32).max:
        raise OverflowError("nnz exceeds Int32 positions")
    return rp.astype(np.int32)


def csr_from_rows_cols(m: int, n: int, rows: np.ndarray, cols: np.ndarray):
    """Canonical CSR pattern (rowptr, colind) of (row, col) pairs, duplicates removed."""
    key = np.sort(rows.astype(np.int64) * np.int64(n) + cols.astype(np.int64))
    # sorted unique keys (np.unique's result; a sort and a mask are faster)
    keep = np.ones(key.shape[0], dtype=bool)
    np.not_equal(key[1:], key[:-1], out=keep[1:])
    key = key[keep]
    r = (key // n).astype(np.int64)
    colind = (key % n).astype(np.int32)
    counts = np.bincount(r, minlength=m)
    return _rowptr_from_counts(counts), colind


def uniform_rows(m: int, n: int, k: int, seed: int):
    """Exactly k distinct uniformly random columns per row, sorted (configs 1 and 4)."""
    rng = np.random.default_rng(seed)
    k = min(k, n)
    extra = max(4, k // 2)
    cols = np.empty((m, k), dtype=np.int32)
    todo = np.arange(m)
    while todo.size:
        cand = np.sort(rng.integers(0, n, size=(todo.size, k + extra), dtype=np.int64), axis=1)
        dup = np.zeros_like(cand, dtype=bool)
        dup[:, 1:] = cand[:, 1:] == cand[:, :-1]
        nuniq = (~dup).sum(axis=1)
        ok = nuniq >= k
        if ok.any():
            c = cand[ok]
            d = dup[ok]
            # first k unique entries of each row, in sorted order
            order = np.argsort(d, axis=1, kind="stable")[:, :k]
            cols[todo[ok]] = np.sort(np.take_along_axis(c, order, axis=1), axis=1).astype(np.int32)
        todo = todo[~ok]
    rowptr = np.arange(0, (m + 1) * k, k, dtype=np.int64).astype(np.int32)
    return rowptr, cols.reshape(-1), rng


def config1(seed: int = 0, n: int = 100_000, k: int = 10):
    """CSR SpMV fp64: n x n, k distinct uniform columns per row, values and x U[-1,1]."""
    rowptr, colind, rng = uniform_rows(n, n, k, seed)
    val = rng.uniform(-1.0, 1.0, size=colind.shape[0])
    x = rng.uniform(-1.0, 1.0, size=n)
    return rowptr, colind, val, x


def laplacian_rows(g: int, r0: int = 0, r1: int | None = None):
    """Rows [r0, r1) of the 5-point Laplacian of a g x g grid in natural
    ordering: 4 on the diagonal, -1 for each grid neighbour, columns ascending
    in every row.  The row pointer starts at 0; columns are global."""
    r1 = g * g if r1 is None else r1
    r = np.arange(r0, r1, dtype=np.int64)
    i, j = r // g, r % g
    cand = np.stack([r - g, r - 1, r, r + 1, r + g], axis=1)
    mask = np.stack([i > 0, j > 0, np.ones(r.shape[0], bool), j < g - 1, i < g - 1], axis=1)
    vals = np.broadcast_to(np.array([-1.0, -1.0, 4.0, -1.0, -1.0]), (r.shape[0], 5))
    colind = cand[mask].astype(np.int32)
    val = vals[mask].astype(np.float64)
    rowptr = _rowptr_from_counts(mask.sum(axis=1))
    return rowptr, colind, val


def laplacian_2d(g: int):
    """The whole 5-point Laplacian of a g x g grid (see laplacian_rows)."""
    return laplacian_rows(g)


def config2(seed: int = 1, g: int = 4096):
    """Laplacian SpMV fp64 on a g x g grid, x U[-1,1]."""
    rowptr, colind, val = laplacian_2d(g)
    x = np.random.default_rng(seed).uniform(-1.0, 1.0, size=g * g)
    return rowptr, colind, val, x


def zipf_degrees(m: int, alpha: float, kmax: int, rng) -> np.ndarray:
    """Out-degrees with P(k) proportional to k^-alpha on [1, kmax] (inverse CDF)."""
    k = np.arange(1, kmax + 1, dtype=np.float64)
    cdf = np.cumsum(k ** -alpha)
    cdf /= cdf[-1]
    return (np.searchsorted(cdf, rng.random(m), side="right") + 1).astype(np.int64)


def power_law(m: int, n: int, alpha: float, kmax: int, seed: int):
    """Power-law CSR pattern: Zipf(alpha) out-degree truncated to [1, kmax],
    uniform random columns, duplicates within a row merged."""
    rng = np.random.default_rng(seed)
    deg = zipf_degrees(m, alpha, kmax, rng)
    rows = np.repeat(np.arange(m, dtype=np.int64), deg)
    cols = rng.integers(0, n, size=rows.shape[0], dtype=np.int64)
    rowptr, colind = csr_from_rows_cols(m, n, rows, cols)
    return rowptr, colind, rng


def config3(seed: int = 2, m: int = 4_194_304, k: int = 64, alpha: float = 2.0, kmax: int = 4096):
    """CSR SpMM fp32: power-law A (values U[0,1]) and row-major B m x k U[-1,1]."""
    rowptr, colind, rng = power_law(m, m, alpha, kmax, seed)
    val = rng.random(colind.shape[0], dtype=np.float32)
    # U[-1, 1) generated in fp32 directly (no fp64 temporary of m x k)
    B = rng.random(size=(m, k), dtype=np.float32)
    B *= np.float32(2.0)
    B -= np.float32(1.0)
    return rowptr, colind, val, B


def config4(seed: int = 3, m: int = 1_048_576, K: int = 128, k: int = 32):
    """SDDMM fp32: k uniform columns per row, A and B (m x K) N(0,1), S U[0,1]."""
    rowptr, colind, rng = uniform_rows(m, m, k, seed)
    A = rng.standard_normal(size=(m, K), dtype=np.float32)
    B = rng.standard_normal(size=(m, K), dtype=np.float32)
    S = rng.random(colind.shape[0], dtype=np.float32)
    return rowptr, colind, A, B, S


def block_banded(nbr: int, band: int, p_off: float, seed: int):
    """Block pattern of an nbr x nbr block grid: (I, J) present when |I-J| <= band
    or, off the band, with probability p_off.  Returns (browptr, bcolind, rng)."""
    rng = np.random.default_rng(seed)
    I = np.arange(nbr)[:, None]
    J = np.arange(nbr)[None, :]
    present = (np.abs(I - J) <= band) | (rng.random((nbr, nbr)) < p_off)
    browptr = _rowptr_from_counts(present.sum(axis=1))
    bcolind = np.nonzero(present)[1].astype(np.int32)
    return browptr, bcolind, rng


def config5(seed: int = 4, nbr: int = 1024, bs: int = 64, band: int = 8, p_off: float = 0.02,
            N: int = 256, std: float = 0.02):
    """BSR SpMM: block-banded 64x64 blocks with N(0, std) bf16 values, B N(0,1) bf16."""
    browptr, bcolind, rng = block_banded(nbr, band, p_off, seed)
    nnzb = bcolind.shape[0]
    bval = f32_to_bf16_bits(rng.standard_normal(size=nnzb * bs * bs, dtype=np.float32) * np.float32(std))
    B = f32_to_bf16_bits(rng.standard_normal(size=(nbr * bs, N), dtype=np.float32))
    return browptr, bcolind, bval, B


def bsr_to_csr(browptr, bcolind, bval, bs: int, nbr_rows: int, drop_zeros: bool = True):
    """Expand a BSRRight matrix (row-major tiles, block columns ascending in
    each block row) to CSR with the same values, the CSR input of the
    conversion benchmark.  Row r of block row I holds row r of each of I's
    tiles in block-column order, so the CSR comes out canonical with no sort.
    Explicit zeros (either sign) are dropped when drop_zeros."""
    browptr = np.asarray(browptr, np.int64)
    nnzb = bcolind.shape[0]
    tiles = np.asarray(bval).reshape(nnzb, bs, bs)
    cols_all = bcolind.astype(np.int64)[:, None] * bs + np.arange(bs)[None, :]   # nnzb x bs
    val_parts, col_parts, counts = [], [], np.zeros(nbr_rows * bs, np.int64)
    for I in range(nbr_rows):
        q0, q1 = int(browptr[I]), int(browptr[I + 1])
        if q1 == q0:
            continue
        v = tiles[q0:q1].transpose(1, 0, 2).reshape(bs, -1)          # rows x (blocks * bs)
        c = np.broadcast_to(cols_all[q0:q1].reshape(1, -1), v.shape)
        keep = None
        if drop_zeros:
            keep = ((v.view(np.uint16) & 0x7FFF) != 0) if v.dtype == np.uint16 else v != 0
            if keep.all():
                keep = None
        if keep is not None:
            counts[I * bs:(I + 1) * bs] = keep.sum(axis=1)
            val_parts.append(v[keep])
            col_parts.append(c[keep])
        else:
            counts[I * bs:(I + 1) * bs] = v.shape[1]
            val_parts.append(v.reshape(-1))
            col_parts.append(c.reshape(-1))
    vals = np.concatenate(val_parts) if val_parts else np.zeros(0, tiles.dtype)
    cols = np.concatenate(col_parts) if col_parts else np.zeros(0, np.int64)
    return _rowptr_from_counts(counts), cols.astype(np.int32), vals
