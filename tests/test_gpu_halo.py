"""The SpMV step fused with its NVLink halo exchange (jlb_halo_spmv_step)."""
import ctypes as C
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import jlust_b200 as J
from jlust_b200 import _lib, synth
from jlust_b200 import dist as D
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _local(g, r0, r1):
    rp, ci, val = synth.laplacian_rows(g, r0, r1)
    lci = (ci.astype(np.int64) - (r0 - g)).astype(np.int32)
    return rp, lci, val


@pytest.mark.parametrize("split", [False, True])
def test_single_rank_iteration_bit_exact(split):
    """One rank (no neighbours): interior-only, or with the boundary blocks
    exercised by declaring the first and last grid lines as boundary rows."""
    g = 256
    n = g * g
    rp, lci, val = _local(g, 0, n)
    d = [torch.from_numpy(a).to(DEV) for a in (rp, lci, val)]
    interior = (g, n - g) if split else (0, n)
    h = D.P2PHaloSpMV(n, g, d[0], d[1], d[2], interior, DEV)
    x = np.random.default_rng(5).uniform(-1, 1, n)
    h.bufs[0][g:g + n].copy_(torch.from_numpy(x))
    frp, fci, fval = synth.laplacian_2d(g)
    for _ in range(7):
        h.step()
        x = O.spmv(frp, fci, fval, x)
    J.device_status()
    assert np.array_equal(h.own().cpu().numpy(), x)


def test_bounded_wait_times_out():
    """A boundary block waits for a neighbour flag that nothing sets: after the
    limit the launch ends, jlb_device_status reports DeviceTimeout and the
    context stays usable."""
    g = 64
    R = 4 * g
    rp, lci, val = _local(g, g, g + R)            # a middle slab: reads both halos
    d = [torch.from_numpy(a).to(DEV) for a in (rp, lci, val)]
    bufs = [torch.zeros(R + 2 * g, dtype=torch.float64, device=DEV) for _ in range(2)]
    flags = torch.zeros(4, dtype=torch.int32, device=DEV)
    fake_peer = torch.zeros(R + 2 * g, dtype=torch.float64, device=DEV)   # stands in for a peer
    fake_flag = torch.zeros(4, dtype=torch.int32, device=DEV)
    st = C.c_void_p(torch.cuda.current_stream(0).cuda_stream)
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    i0, i1 = D.interior_rows(rp, lci, R, g)
    P2 = C.c_void_p * 2
    xb = P2(bufs[0].data_ptr(), bufs[1].data_ptr())
    lb = P2(fake_peer.data_ptr(), fake_peer.data_ptr())
    _lib.call("jlb_halo_spmv_steps", st, _lib.F64, 0, R, g, i0, i1, p(d[0]), p(d[1]), p(d[2]),
              xb, lb, None, p(flags), p(fake_flag), C.c_void_p(0), 1, 1,
              int(20e6))     # step 1 needs the lower neighbour's flag >= 1; limit 20 ms
    with pytest.raises(J.DeviceTimeout):
        J.device_status()
    y = torch.zeros(R, dtype=torch.float64, device=DEV)
    J.execute(J.SpMVOp, J.csr_tensor(d[0], d[1], d[2], (R, R + 2 * g), origin=0), bufs[0], y)
    J.device_status()


def test_argument_checks():
    L = _lib.load()
    P2 = C.c_void_p * 2
    xb = P2(16, 32)
    # a neighbour buffer without its flag
    st = L.jlb_halo_spmv_steps(None, _lib.F64, 0, 200, 64, 64, 136, None, None, None, xb,
                               P2(16, 32), None, None, None, None, 0, 1, 1000)
    assert st == 8
    # rows feeding the lower neighbour declared interior
    st = L.jlb_halo_spmv_steps(None, _lib.F64, 0, 200, 64, 0, 136, None, None, None, xb,
                               P2(16, 32), None, None, C.c_void_p(16), None, 0, 1, 1000)
    assert st == 8


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_ranks_bit_exact_and_failure_detection():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", "29533",
           os.path.join(root, "tests", "dist_p2p_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-3000:]
    assert "BITEXACT True" in out
    assert "TIMEOUT True" in out
