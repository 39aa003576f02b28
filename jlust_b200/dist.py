"""Row-partitioned SpMV across GPUs (one process per GPU, torch.distributed).

The reference has no distributed layer; this is the B200 design for its
iterative SpMV workload (x <- A x on a 2-D Laplacian).  Rank r owns rows
[r*R, (r+1)*R) of A and the same slice of x.  Its local x buffer is
[lower halo (h) | own rows (R) | upper halo (h)], where h is the half
bandwidth (the grid width for a 5-point Laplacian), and the local CSR's column
indices are shifted into that buffer.  Each iteration exchanges only the
halos: the first h own entries go to rank r-1 (its upper halo), the last h to
rank r+1 (its lower halo) -- 2*h*8 bytes per neighbour instead of the whole of
x.  The interior rows, which read no halo entry, run while the exchange is in
flight; the 2*h boundary rows run after it.

Every row's sum is formed exactly as on one GPU (same entries, same order),
so the partitioned iteration is bit-identical to the single-GPU one.

`allgather` exchange mode replaces the halo exchange by an all-gather of the
whole x for comparison.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist


def partition_rows(n: int, world: int, rank: int, align: int = 1):
    """Contiguous, equal row ranges (rounded to `align` rows)."""
    per = -(-n // world)
    per = -(-per // align) * align
    r0 = min(rank * per, n)
    r1 = min(r0 + per, n)
    return r0, r1


def local_csr(rowptr: np.ndarray, colind: np.ndarray, val: np.ndarray, r0: int, r1: int, h: int):
    """Rows [r0, r1) of a global CSR with columns shifted into the local halo
    buffer (column c -> c - (r0 - h)).  Requires every column of those rows to
    lie in [r0 - h, r1 + h)."""
    p0, p1 = int(rowptr[r0]), int(rowptr[r1])
    lrp = (rowptr[r0:r1 + 1].astype(np.int64) - p0).astype(np.int32)
    lci = colind[p0:p1].astype(np.int64) - (r0 - h)
    if lci.size and (lci.min() < 0 or lci.max() >= (r1 - r0) + 2 * h):
        raise ValueError("local_csr: a column falls outside the halo window")
    return lrp, lci.astype(np.int32), val[p0:p1]


def interior_rows(lrp: np.ndarray, lci: np.ndarray, R: int, h: int):
    """[first, last) local rows that read only own entries [h, h + R)."""
    lo, hi = 0, R
    while lo < R:
        cols = lci[lrp[lo]:lrp[lo + 1]]
        if cols.size and cols.min() < h:
            lo += 1
        else:
            break
    while hi > lo:
        cols = lci[lrp[hi - 1]:lrp[hi]]
        if cols.size and cols.max() >= h + R:
            hi -= 1
        else:
            break
    return lo, hi


class HaloSpMV:
    """Distributed x <- A x with halo exchange.

    `spmv(row_lo, row_hi, x_buf, y_buf)` computes local rows [row_lo, row_hi)
    of A times the halo buffer x_buf into y_buf[h + row_lo : h + row_hi]; it is
    the B200 kernel on GPUs and any CPU stand-in on gloo.
    """

    def __init__(self, R: int, h: int, spmv, device, dtype=torch.float64, mode: str = "halo",
                 interior=None, group=None):
        self.R, self.h = R, h
        self.spmv = spmv
        self.mode = mode
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.bufs = [torch.zeros(R + 2 * h, dtype=dtype, device=device) for _ in range(2)]
        self.cur = 0
        self.interior = interior if interior is not None else (0, R)
        if mode == "allgather":
            self.gather = torch.zeros(R * self.world, dtype=dtype, device=device)

    @property
    def x(self) -> torch.Tensor:
        return self.bufs[self.cur]

    def own(self, buf=None) -> torch.Tensor:
        b = self.x if buf is None else buf
        return b[self.h:self.h + self.R]

    def _exchange(self, buf):
        h, R = self.h, self.R
        ops = []
        if self.rank > 0:
            ops.append(dist.P2POp(dist.isend, buf[h:2 * h], self.rank - 1, self.group))
            ops.append(dist.P2POp(dist.irecv, buf[0:h], self.rank - 1, self.group))
        if self.rank < self.world - 1:
            ops.append(dist.P2POp(dist.isend, buf[R:R + h], self.rank + 1, self.group))
            ops.append(dist.P2POp(dist.irecv, buf[R + h:R + 2 * h], self.rank + 1, self.group))
        return dist.batch_isend_irecv(ops) if ops else []

    def _allgather(self, buf):
        h, R = self.h, self.R
        dist.all_gather_into_tensor(self.gather, buf[h:h + R].contiguous(), group=self.group)
        g0 = self.rank * R - h
        lo, hi = max(g0, 0), min(g0 + R + 2 * h, self.gather.numel())
        buf[lo - g0:hi - g0].copy_(self.gather[lo:hi])

    def step(self):
        """One iteration x <- A x; returns the new x buffer."""
        x, y = self.bufs[self.cur], self.bufs[1 - self.cur]
        if self.world == 1:
            self.spmv(0, self.R, x, y)
        elif self.mode == "allgather":
            self._allgather(x)
            self.spmv(0, self.R, x, y)
        else:
            reqs = self._exchange(x)
            i0, i1 = self.interior
            if i1 > i0:
                self.spmv(i0, i1, x, y)
            for r in reqs:
                r.wait()
            if i0 > 0:
                self.spmv(0, i0, x, y)
            if i1 < self.R:
                self.spmv(i1, self.R, x, y)
        self.cur = 1 - self.cur
        return self.bufs[self.cur]
