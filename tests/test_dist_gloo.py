"""Row-partitioned Laplacian iteration with halo exchange (jlust_b200/dist.py)
on two CPU ranks over gloo; the local SpMV is the oracle, so the check is
that partitioning and exchange reproduce the single-process iteration bit
for bit, in both exchange modes."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

G = 48          # grid width: n = 2304 rows, halo = 48
ITERS = 6


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, out_dir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from jlust_b200 import dist as D
    from jlust_b200 import synth
    from oracle import oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n = G * G
        r0, r1 = D.partition_rows(n, world, rank, align=G)
        R = r1 - r0
        rp, ci, val = synth.laplacian_rows(G, r0, r1)
        lci = (ci.astype(np.int64) - (r0 - G)).astype(np.int32)
        x0 = np.random.default_rng(1).uniform(-1, 1, n)

        def spmv(lo, hi, x, y):
            y[G + lo:G + hi] = torch.from_numpy(O.spmv(rp[lo:hi + 1], lci, val, x.numpy()))

        interior = D.interior_rows(rp, lci, R, G)
        h = D.HaloSpMV(R, G, spmv, "cpu", mode=mode, interior=interior)
        buf = np.zeros(R + 2 * G)
        lo, hi = max(r0 - G, 0), min(r1 + G, n)
        buf[lo - (r0 - G):hi - (r0 - G)] = x0[lo:hi]
        h.bufs[0].copy_(torch.from_numpy(buf))
        for _ in range(ITERS):
            h.step()
        np.save(os.path.join(out_dir, f"x{rank}.npy"), h.own().numpy())
        np.save(os.path.join(out_dir, f"interior{rank}.npy"), np.array(interior))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["halo", "allgather"])
def test_two_rank_laplacian_matches_single(tmp_path, mode):
    from jlust_b200 import synth
    from oracle import oracle as O
    O.build()
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), mode, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    got = np.concatenate([np.load(tmp_path / f"x{r}.npy") for r in range(world)])
    rp, ci, val = synth.laplacian_2d(G)
    x = np.random.default_rng(1).uniform(-1, 1, G * G)
    for _ in range(ITERS):
        x = O.spmv(rp, ci, val, x)
    assert np.array_equal(got, x)
    # interior rows exclude exactly the first and last grid line of each rank
    for r in range(world):
        i0, i1 = np.load(tmp_path / f"interior{r}.npy")
        assert (i0, i1) == ((G if r > 0 else 0), (G * G // world - G if r < world - 1 else G * G // world))


def test_partition_rows():
    from jlust_b200 import dist as D
    n, g = 4096 * 4096, 4096
    spans = [D.partition_rows(n, 8, r, align=g) for r in range(8)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    assert all(b == c for (_, b), (c, _) in zip(spans, spans[1:]))
    assert all((b - a) % g == 0 for a, b in spans)


def test_partition_by_nnz_balances_power_law():
    from jlust_b200 import dist as D
    from jlust_b200 import synth
    rp, _, _ = synth.power_law(100_000, 100_000, 2.0, 4096, seed=3)
    for world in (2, 4, 8):
        spans = [D.partition_by_nnz(rp, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == 100_000
        assert all(b == c for (_, b), (c, _) in zip(spans, spans[1:]))
        work = [(rp[b] - rp[a]) + (b - a) for a, b in spans]
        assert max(work) - min(work) <= 4096 + 2          # at most one long row apart


def _scan_worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from jlust_b200 import dist as D
    from oracle import oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        counts = np.random.default_rng(7).integers(0, 50, size=1001).astype(np.int32)
        lo, hi = D.partition_rows(counts.shape[0], world, rank)
        part = torch.from_numpy(counts[lo:hi].copy())

        def cpu_scan(c, base):   # the oracle's scan stands in for the GPU's on gloo ranks
            return torch.from_numpy(O.exclusive_scan(c.numpy(), base).astype(np.int32))

        out = D.exclusive_scan(part, base=1, scan=cpu_scan)
        np.save(os.path.join(out_dir, f"scan{rank}.npy"), out.numpy())
        # rank 0's slice overflows by itself, the others only together
        big = torch.full((4,), 2**29 if rank == 0 else 2**28, dtype=torch.int32)
        try:
            D.exclusive_scan(big, scan=cpu_scan)
            np.save(os.path.join(out_dir, f"ovf{rank}.npy"), np.array([0]))
        except OverflowError:
            np.save(os.path.join(out_dir, f"ovf{rank}.npy"), np.array([1]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_distributed_scan_matches_global(tmp_path, world):
    """Local scans + all-gather of shard totals reproduce the global exclusive
    scan bit for bit (origin 1, an uneven split); a global total past Int32
    raises on every rank."""
    from oracle import oracle as O
    mp.spawn(_scan_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    counts = np.random.default_rng(7).integers(0, 50, size=1001).astype(np.int32)
    ref = O.exclusive_scan(counts, 1)
    from jlust_b200 import dist as D
    for r in range(world):
        lo, hi = D.partition_rows(counts.shape[0], world, r)
        got = np.load(tmp_path / f"scan{r}.npy")
        assert np.array_equal(got, ref[lo:hi + 1])
        assert np.load(tmp_path / f"ovf{r}.npy")[0] == 1
