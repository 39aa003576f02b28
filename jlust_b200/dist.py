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
whole x for comparison.  P2PHaloSpMV fuses the exchange into the SpMV kernel
over NVLink peer memory (one launch per step, no collective library).
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


def partition_by_nnz(rowptr: np.ndarray, world: int, rank: int):
    """Contiguous row range of `rank` with about (m + nnz) / world rows plus
    entries: each row counts once plus its entries, so power-law rows and
    empty rows both balance.  Returns (r0, r1)."""
    rowptr = np.asarray(rowptr, dtype=np.int64)
    m = rowptr.shape[0] - 1
    base = int(rowptr[0])
    work = (rowptr - base) + np.arange(m + 1)
    total = int(work[-1])

    def cut(k):
        return int(np.searchsorted(work, total * k / world, side="left"))

    r0 = 0 if rank == 0 else min(cut(rank), m)
    r1 = m if rank == world - 1 else min(cut(rank + 1), m)
    return r0, max(r0, r1)


def exclusive_scan(counts: torch.Tensor, base: int = 0, scan=None, group=None) -> torch.Tensor:
    """Exclusive scan of counts split across ranks in rank order (rank r holds
    a contiguous slice): returns this rank's part of the global position
    buffer, out[0] = base + (counts of lower ranks), out[i+1] = out[i] +
    counts[i] -- len(counts) + 1 entries, so rank r's last entry equals rank
    r+1's first.  Each rank scans its slice locally (`scan`, default the
    library's jlb_exclusive_scan_i32 on the slice's GPU; any callable with the
    same contract on CPU ranks), then one all-gather of the slice totals gives
    the offsets.  The result is int32 like every position buffer; a global
    total past Int32 raises OverflowError on every rank."""
    if scan is None:
        from .convert import exclusive_scan as scan
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    # the shard total as an int64 sum (not the scan's last entry, which would
    # wrap); every rank takes the all-gather, also one whose shard alone
    # overflows, so that all ranks raise together
    mine = int(counts.sum(dtype=torch.int64).item())
    local = scan(counts, 0) if base + mine <= 2**31 - 1 else None
    total = torch.tensor([mine], dtype=torch.int64)
    if counts.is_cuda and world > 1 and dist.get_backend(group) == "nccl":
        total = total.to(counts.device)
    totals = [torch.zeros_like(total) for _ in range(world)]
    if world > 1:
        dist.all_gather(totals, total, group=group)
    else:
        totals = [total]
    totals = [int(t.item()) for t in totals]
    if local is None or base + sum(totals) > 2**31 - 1:
        raise OverflowError("exclusive_scan: global total exceeds Int32 positions")
    offset = base + sum(totals[:rank])
    return local + offset if offset else local


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


class P2PHaloSpMV:
    """Distributed x <- A x with the halo exchange fused into the SpMV kernel
    (jlb_halo_spmv_steps): each step is one launch per GPU that computes the
    local rows, stores the boundary results straight into the neighbours'
    halo buffers over NVLink (CUDA IPC peer pointers) and publishes them with
    a system-scope release flag; the neighbour's boundary rows wait for it.
    No host synchronisation and no collective library on the data path.

    rowptr / colind / val are the local CSR on this rank's GPU (columns in
    halo-buffer coordinates); interior = (lo, hi) local rows reading no halo.
    """

    def __init__(self, R: int, h: int, rowptr, colind, val, interior, device, group=None,
                 timeout_s: float = 2.0):
        import ctypes as C

        from . import _lib
        self.C, self._lib = C, _lib
        self.R, self.h = R, h
        self.rowptr, self.colind, self.val = rowptr, colind, val
        self.dtype = {torch.float64: _lib.F64, torch.float32: _lib.F32}[val.dtype]
        self.interior = interior
        self.device = torch.device(device)
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.timeout_ns = int(timeout_s * 1e9)
        self.bufs = [torch.zeros(R + 2 * h, dtype=val.dtype, device=self.device) for _ in range(2)]
        self.flags = torch.zeros(4, dtype=torch.int32, device=self.device)
        self.step_no = 0
        self._opened = []
        self._bases = {}
        self.lower = self.upper = None   # (bufs ptrs [2], flags ptr) of neighbours
        if self.world > 1:
            mine = [self._handle(t) for t in (*self.bufs, self.flags)]
            allh = [None] * self.world
            dist.all_gather_object(allh, mine, group=group)
            torch.cuda.synchronize(self.device)
            if self.rank > 0:
                self.lower = self._open(allh[self.rank - 1])
            if self.rank < self.world - 1:
                self.upper = self._open(allh[self.rank + 1])
            dist.barrier(group=group)

    def _handle(self, t):
        C = self.C
        hbuf = (C.c_char * 64)()
        off = C.c_uint64()
        self._lib.call("jlb_ipc_handle", C.c_void_p(t.data_ptr()), hbuf, C.byref(off))
        return bytes(hbuf), off.value

    def _open(self, handles):
        # Several tensors may share one allocation, hence one handle: map each
        # allocation once.
        C = self.C
        ptrs = []
        for hb, off in handles:
            if hb not in self._bases:
                base = C.c_void_p()
                self._lib.call("jlb_ipc_open", C.c_char_p(hb), C.byref(base))
                self._bases[hb] = base.value
                self._opened.append(base.value)
            ptrs.append(self._bases[hb] + off)
        return ptrs[:2], ptrs[2]

    @property
    def x(self) -> torch.Tensor:
        return self.bufs[self.step_no % 2]

    def own(self, buf=None) -> torch.Tensor:
        b = self.x if buf is None else buf
        return b[self.h:self.h + self.R]

    def _arrays(self):
        C = self.C
        P2 = C.c_void_p * 2
        self._xb = P2(*(b.data_ptr() for b in self.bufs))
        self._lb = P2(*self.lower[0]) if self.lower else None
        self._ub = P2(*self.upper[0]) if self.upper else None

    def steps(self, k: int = 1):
        """Run k iterations (k launches, one ABI call); returns the current x buffer."""
        C = self.C
        if not hasattr(self, "_xb"):
            self._arrays()
        st = C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        self._lib.call("jlb_halo_spmv_steps", st, self.dtype, 0, self.R, self.h, self.interior[0],
                       self.interior[1], C.c_void_p(self.rowptr.data_ptr()),
                       C.c_void_p(self.colind.data_ptr()), C.c_void_p(self.val.data_ptr()),
                       self._xb, self._lb, self._ub, C.c_void_p(self.flags.data_ptr()),
                       C.c_void_p(self.lower[1] + 4) if self.lower else C.c_void_p(0),
                       C.c_void_p(self.upper[1]) if self.upper else C.c_void_p(0),
                       self.step_no, k, self.timeout_ns)
        self.step_no += k
        return self.bufs[self.step_no % 2]

    def step(self):
        return self.steps(1)

    def close(self):
        """Unmap the neighbours' buffers; call on every rank, between steps."""
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        for base in self._opened:
            self._lib.call("jlb_ipc_close", self.C.c_void_p(base))
        self._opened = []
        self._bases = {}
        self.lower = self.upper = None
        if hasattr(self, "_xb"):
            del self._xb
