"""Child process of tests/test_gpu_halo.py (run under torch.distributed.run on
2+ GPUs): the fused NVLink halo iteration against the single-GPU iteration,
then a rank that leaves between steps so its neighbour's next step times out."""
import ctypes as C
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import jlust_b200 as J  # noqa: E402
from jlust_b200 import _lib, synth  # noqa: E402
from jlust_b200 import dist as D  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    g, iters = 512, 12
    n = g * g
    r0, r1 = D.partition_rows(n, world, rank, align=g)
    R = r1 - r0
    rp, ci, val = synth.laplacian_rows(g, r0, r1)
    lci = (ci.astype(np.int64) - (r0 - g)).astype(np.int32)
    d = [torch.from_numpy(a).to(dev) for a in (rp, lci, val)]
    h = D.P2PHaloSpMV(R, g, d[0], d[1], d[2], D.interior_rows(rp, lci, R, g), dev,
                      timeout_s=0.25)
    x0 = np.random.default_rng(1).uniform(-1, 1, n)
    buf = np.zeros(R + 2 * g)
    lo, hi = max(r0 - g, 0), min(r1 + g, n)
    buf[lo - (r0 - g):hi - (r0 - g)] = x0[lo:hi]
    h.bufs[0].copy_(torch.from_numpy(buf))
    dist.barrier()
    for _ in range(iters):
        h.step()
    J.device_status()
    own = h.own().contiguous()
    parts = [torch.empty_like(own) for _ in range(world)]
    dist.all_gather(parts, own)
    ok = True
    if rank == 0:
        frp, fci, fval = synth.laplacian_2d(g)
        A = J.csr_tensor(torch.from_numpy(frp).to(dev), torch.from_numpy(fci).to(dev),
                         torch.from_numpy(fval).to(dev), (n, n), origin=0)
        xa = torch.from_numpy(x0).to(dev)
        xb = torch.empty_like(xa)
        for _ in range(iters):
            J.execute(J.SpMVOp, A, xa, xb)
            xa, xb = xb, xa
        ok = torch.equal(torch.cat(parts), xa)
        print(f"BITEXACT {ok}", flush=True)
    # Failure detection: the last rank leaves (between steps, nothing in
    # flight); rank world-2 waits for its publication, times out, and reports.
    dist.barrier()
    timed_out = False
    if rank == world - 2:
        h.step()     # step `iters` uses the last rank's final publication
        h.step()     # step `iters`+1 waits for a publication that never comes
        try:
            J.device_status()
        except J.DeviceTimeout:
            timed_out = True
        # the context is still usable
        y = torch.zeros(R, dtype=torch.float64, device=dev)
        J.execute(J.SpMVOp, J.csr_tensor(d[0], d[1], d[2], (R, R + 2 * g), origin=0),
                  h.bufs[0], y)
        J.device_status()
        print(f"TIMEOUT {timed_out}", flush=True)
    h.close()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
