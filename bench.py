#!/usr/bin/env python
"""Benchmark of the JLUST hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|cusparse]
                    [--workload laplacian|spmv1|spmm|sddmm|bsr|convert|scan|coo2csr|
                                spmv_powerlaw|spmv_medium]
                    [--extra auto|none]

Default workload (the configuration the headline metric is quoted on): CSR
SpMV fp64 on the 5-point Laplacian of a 4096 x 4096 grid, x <- A x, one step
per iteration, rows partitioned across the N ranks with a halo exchange
(strong scaling: the matrix is the same for every N).  Inputs are larger than
L2 (1.34 GB per iteration), so no flush is needed between iterations.

Prints ONE JSON line on rank 0.  `value` is whole-job GFLOP/s (2 flops per
stored entry) from CUDA events on the launch stream, max over ranks; `e2e` is
the same metric through the public API with the step's input copied from
pinned host memory and its result copied back inside the timed region;
`roofline` relates the dominant kernel's algorithmic bytes per launch to the
measured HBM copy bandwidth; `cpu_baseline` times the CPU restatement of the
reference's path on this host's cores (all of them, and one); `parity` checks
the last timed step's output against that restatement.

With the default workload the line also carries `workloads`: the other
configurations measured the same way in the same process (cfg3 SpMM, cfg4
SDDMM, cfg5 BSR SpMM, the CSR -> BSR conversion of the cfg5 matrix and the
cfg2 row-pointer scan on one GPU; the sharded cfg3/cfg4/cfg5 on N GPUs).
`--extra none` leaves them out.

`--impl reference` times the CPU restatement of the reference's path (the
reference is Julia; no Julia toolchain exists here) on the same workloads
with every host thread (rank 0; other ranks exit).  `--impl cusparse` times
cuSPARSE (the reference's default GPU library for SpMM and SDDMM) through
torch.sparse on cfg2, cfg3 and cfg4, as a comparison point only.
"""
from __future__ import annotations

import argparse
import datetime
import gc
import json
import os
import re
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

METRIC = "SpMV/SpMM GFLOP/s and effective HBM GB/s (% roofline) at 1/2/4/8 B200"
DATA = "synthetic (numpy PCG64, seeds of the configs)"


def parse_args(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference", "cusparse"], default="ours")
    p.add_argument("--workload", default="laplacian", choices=sorted(WORKLOADS))
    p.add_argument("--extra", choices=["auto", "none"], default="auto",
                   help="auto: with the default workload, also measure the other configurations "
                        "(the `workloads` object); none: the headline workload only")
    p.add_argument("--extra-steps", type=int, default=20,
                   help="timed steps of each extra workload (at most --steps)")
    p.add_argument("--exchange", choices=["p2p", "halo", "allgather"], default="p2p",
                   help="p2p: halo fused into the SpMV kernel over NVLink (default); "
                        "halo: NCCL send/recv; allgather: NCCL all-gather of x")
    p.add_argument("--grid", type=int, default=4096, help="Laplacian grid width")
    p.add_argument("--l2-persist", type=int, default=1,
                   help="Laplacian: persisting L2 window over the local CSR: 1 = where the "
                        "set-aside holds half of it, 2 = always, 0 = never")
    p.add_argument("--cpu-budget", type=float, default=5.0,
                   help="seconds of CPU work per CPU-baseline leg (all cores, one core)")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--no-parity", action="store_true")
    return p.parse_args(argv)


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def profile_traffic(name: str):
    """dram bytes per launch recorded from an ncu capture in profiles/<name>.md."""
    path = os.path.join(ROOT, "profiles", name + ".md")
    if not os.path.exists(path):
        return None
    m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", open(path).read())
    return float(m.group(1)) if m else None


# --------------------------------------------------------------- clocks ----
_REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
            0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x1: "gpu_idle",
            0x2: "applications_clocks_setting", 0x10: "sync_boost", 0x100: "display_clock"}


class ClockSampler:
    """Samples SM clock, power and clock-event reasons through NVML from a
    background thread while the timed region runs."""

    def __init__(self, torch_device, period_s=0.005):
        self.period = period_s
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self.h = None
        self.err = None
        try:
            import pynvml as N
            import torch
            N.nvmlInit()
            pr = torch.cuda.get_device_properties(torch_device)
            bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
            try:
                self.h = N.nvmlDeviceGetHandleByPciBusId(bus.encode())
            except Exception:
                self.h = N.nvmlDeviceGetHandleByPciBusId(bus)
            self.N = N
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM)
        except Exception as e:  # NVML missing: report no clocks rather than fail
            self.h = None
            self.err = repr(e)
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        N = self.N
        while not self._stop.is_set():
            try:
                self.samples.append(N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM))
                bits = N.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for b, name in _REASONS.items():
                    if bits & b and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def start(self):
        if self.h is not None and self._t is None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __enter__(self):
        return self.start()

    def __exit__(self, *a):
        if self._t is not None:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": 0, "error": self.err}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------------------ distributed --
class Ctx:
    def __init__(self, args):
        import torch
        self.torch = torch
        self.rank = env_int("RANK", 0)
        self.world = env_int("WORLD_SIZE", 1)
        self.local = env_int("LOCAL_RANK", 0)
        self.args = args
        self.dist = None
        if args.impl in ("ours", "cusparse"):
            torch.cuda.set_device(self.local)
            self.device = torch.device("cuda", self.local)
            if self.world > 1:
                import torch.distributed as dist
                dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                        device_id=self.device)
                self.dist = dist

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()
        self.torch.cuda.synchronize(self.device)

    def max_over_ranks(self, v: float) -> float:
        if self.dist is None:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device=self.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(self, v: float) -> float:
        if self.dist is None:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device=self.device)
        self.dist.all_reduce(t)
        return float(t.item())

    def close(self):
        if self.dist is not None:
            self.dist.barrier()
            self.dist.destroy_process_group()


def timed(ctx, fn, steps, stream, finish=None):
    """Runs fn() `steps` times between a barrier+sync and CUDA events on
    `stream` (`finish()`, if given, joins other streams into `stream` before
    the end event); returns (max-over-ranks seconds, clock summary)."""
    torch = ctx.torch
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    # NVML set-up and the sampling thread start before the barrier, so every
    # rank enters the timed region together.
    clk = ClockSampler(ctx.device).start()
    ctx.barrier()
    with clk:
        start.record(stream)
        for _ in range(steps):
            fn()
        if finish is not None:
            finish()
        end.record(stream)
        torch.cuda.synchronize(ctx.device)
    secs = start.elapsed_time(end) / 1e3
    ctx.barrier()
    return ctx.max_over_ranks(secs), clk.summary()


# ----------------------------------------------------------------- parity --
def tol_check(got, ref, bound, tol):
    """Per element |got - ref| / bound (bound = sum of |terms|, from the fp64
    restatement) and the normwise relative error (bench_suitesparse.jl:
    263-264 form); both must be <= tol."""
    got = np.asarray(got, dtype=np.float64).reshape(-1)
    ref = np.asarray(ref, dtype=np.float64).reshape(-1)
    bound = np.asarray(bound, dtype=np.float64).reshape(-1)
    if got.size == 0:
        return 0.0, 0.0
    per = float(np.max(np.abs(got - ref) / (bound + 1e-300)))
    nr = float(np.linalg.norm(ref))
    norm = float(np.linalg.norm(got - ref) / nr) if nr > 0 else 0.0
    return per, norm


def exact_check(got, ref):
    """Mismatching elements, comparing bits (NaNs match NaNs)."""
    got, ref = np.asarray(got).reshape(-1), np.asarray(ref).reshape(-1)
    if got.shape != ref.shape:
        return max(got.size, ref.size)
    if got.dtype.kind == "f":
        bad = (got != ref) & ~(np.isnan(got) & np.isnan(ref))
        return int(np.count_nonzero(bad))
    return int(np.count_nonzero(got != ref))


def exact_result(mismatches, checked):
    return {"kind": "bit-exact", "mismatches": int(mismatches), "max_rel": 0.0 if not mismatches
            else None, "pass": mismatches == 0, "checked": checked}


def tol_result(per, norm, tol, checked, **extra):
    return {"kind": "tol", "tol": tol, "max_rel": per, "normwise": norm,
            "pass": bool(per <= tol and norm <= tol), "checked": checked, **extra}


# ------------------------------------------------------------- workloads --
class Laplacian:
    """Config 2: x <- A x on the 5-point Laplacian of a g x g grid, fp64."""

    key, kernel, dtype, unit = "cfg2_laplacian", "spmv_rows", "f64", "GFLOP/s"
    profile = "laplacian"
    bound = "hbm"

    def __init__(self, ctx, host_only=False):
        from jlust_b200 import synth
        self.ctx = ctx
        g = ctx.args.grid
        self.g, self.n = g, g * g
        self.nnz_total = 5 * self.n - 4 * g
        self.x0 = np.random.default_rng(1).uniform(-1.0, 1.0, size=self.n)
        self.synth = synth
        if host_only:
            return
        import ctypes as C

        import torch

        import jlust_b200 as J
        from jlust_b200 import _lib
        from jlust_b200 import dist as D

        self.J, self.C, self._lib = J, C, _lib
        r0, r1 = D.partition_rows(self.n, ctx.world, ctx.rank, align=g)
        self.r0, self.r1, self.R = r0, r1, r1 - r0
        rp, ci, val = synth.laplacian_rows(g, r0, r1)
        lci = (ci.astype(np.int64) - (r0 - g)).astype(np.int32)
        self.nnz_local = int(rp[-1])
        dev = ctx.device
        # the local CSR in one allocation (row pointer | columns | values, 256-byte
        # aligned parts) so that one L2 access-policy window covers it
        parts = [rp, lci, val]
        offs, tot = [], 0
        for a in parts:
            offs.append(tot)
            tot += -(-a.nbytes // 256) * 256
        self.csr_buf = torch.empty(tot, dtype=torch.uint8, device=dev)
        views = []
        for a, o in zip(parts, offs):
            v = self.csr_buf[o:o + a.nbytes].view(getattr(torch, str(a.dtype)))
            v.copy_(torch.from_numpy(a))
            views.append(v)
        self.rowptr, self.colind, self.val = views
        self.persisted = 0
        if ctx.args.l2_persist:
            # kept only where the set-aside holds at least half of the local CSR
            # (8 ranks at 4096^2); on larger shards it would only shrink L2
            self.persisted = J.l2_persist(self.csr_buf, tot, device=dev)
            if ctx.args.l2_persist == 1 and 2 * self.persisted < tot:
                self.persisted = J.l2_persist(0, 0, device=dev)
        self.csr_bytes = tot
        self.A = J.csr_tensor(self.rowptr, self.colind, self.val, (self.R, self.R + 2 * g), origin=0)
        interior = D.interior_rows(rp, lci, self.R, g) if ctx.world > 1 else (0, self.R)
        self.p2p = ctx.world > 1 and ctx.args.exchange == "p2p"
        if self.p2p:
            self.halo = D.P2PHaloSpMV(self.R, g, self.rowptr, self.colind, self.val, interior, dev)
            self.launches_per_step = 1
            self.kernel = "halo_step"
        else:
            self.halo = D.HaloSpMV(self.R, g, self._spmv_rows, dev, mode=ctx.args.exchange,
                                   interior=interior)
            self.launches_per_step = sum(
                1 for a, b in ((0, interior[0]), interior, (interior[1], self.R)) if b > a
            ) if ctx.world > 1 and ctx.args.exchange == "halo" else 1
        self.reset()

    def reset(self):
        """x = x0 on every rank; all ranks call it together, between steps."""
        import torch
        g, r0, r1 = self.g, self.r0, self.r1
        buf = np.zeros(self.R + 2 * g)
        lo, hi = max(r0 - g, 0), min(r1 + g, self.n)
        buf[lo - (r0 - g):hi - (r0 - g)] = self.x0[lo:hi]
        self.ctx.barrier()
        if self.p2p:
            self.halo.step_no = 0
            self.halo.flags.zero_()
        else:
            self.halo.cur = 0
        self.halo.bufs[0].copy_(torch.from_numpy(buf))
        self.halo.bufs[1].zero_()
        self.ctx.barrier()

    def close(self):
        if self.p2p:
            self.halo.close()
        if self.persisted:
            self.J.l2_persist(0, 0, device=self.ctx.device)

    def _spmv_rows(self, lo, hi, x, y):
        """Rows [lo, hi) through the C ABI (row-range view of the local CSR)."""
        C = self.C
        st = C.c_void_p(self.ctx.torch.cuda.current_stream(self.ctx.device).cuda_stream)
        self._lib.call("jlb_csr_spmv", st, self._lib.F64, 0, hi - lo, self.R + 2 * self.g,
                       self.nnz_local, C.c_void_p(self.rowptr.data_ptr() + 4 * lo),
                       C.c_void_p(self.colind.data_ptr()), C.c_void_p(self.val.data_ptr()),
                       C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr() + 8 * (self.g + lo)),
                       1.0, 0.0)

    def step(self):
        self.halo.step()

    def run_steps(self, k):
        if self.p2p:
            self.halo.steps(k)
        else:
            for _ in range(k):
                self.halo.step()

    # algorithmic work, whole job, per step (bench_suitesparse.jl:170-172 form)
    def flops(self):
        return 2.0 * self.nnz_total

    def bytes(self):
        return 12.0 * self.nnz_total + 4.0 * (self.n + 1) + 8.0 * (2 * self.n)

    def config(self):
        c = {"workload": f"cfg2: CSR SpMV fp64, 2D 5-point Laplacian {self.g}x{self.g} "
                         f"(n={self.n}, nnz={self.nnz_total}), x <- A x per step",
             "n": self.n, "nnz": self.nnz_total}
        if not hasattr(self, "halo"):
            return c
        c.update({"partition": f"rows/{self.ctx.world}",
                  "exchange": "none" if self.ctx.world == 1 else
                  ("halo fused into the SpMV kernel over NVLink peer memory" if self.p2p
                   else self.ctx.args.exchange),
                  "l2": (f"per-rank CSR {self.csr_bytes} B under a persisting L2 window "
                         f"({self.persisted} B set-aside), x and y not; no flush"
                         if self.persisted else "inputs larger than L2, no flush")})
        return c

    # parity: after K steps from reset() the own rows hold A^K x0
    def snapshot(self, k):
        self.snap = (k, self.halo.own().cpu().numpy().copy())

    def parity(self):
        from oracle import oracle as O
        k, got = self.snap
        rp, ci, val = self.synth.laplacian_2d(self.g)
        x = self.x0.copy()
        for _ in range(k):
            x = O.spmv(rp, ci, val, x)
        bad = exact_check(got, x[self.r0:self.r1])
        bad = int(self.ctx.sum_over_ranks(bad))
        return exact_result(bad, f"x after the {k} timed steps (A^{k} x0, all {self.n} rows over "
                                 f"{self.ctx.world} rank(s)) against the oracle's {k} iterations")

    # end to end through the public API: x from pinned host memory, y back to it
    def e2e_setup(self):
        import torch
        self.hx = [torch.from_numpy(self.x0[self.r0:self.r1].copy()).pin_memory(),
                   torch.empty(self.R, dtype=torch.float64).pin_memory()]
        self.hcur = 0
        self.h2d = 8 * self.n
        self.d2h = 8 * self.n
        if self.ctx.world == 1:
            # one GPU: the step runs in row chunks on three streams, so that x's
            # chunks go in, row chunks compute and y's chunks come back at once
            # (PCIe is full duplex); every step still copies all of x in and
            # all of y out, and step t+1's x is step t's y read back
            nch = 16
            b = [self.R * c // nch for c in range(nch + 1)]
            self.chunks = list(zip(b[:-1], b[1:]))
            self.views = [self.J.csr_tensor(self.rowptr[lo:hi + 1], self.colind, self.val,
                                            (hi - lo, self.R + 2 * self.g), origin=0)
                          for lo, hi in self.chunks]
            self.s_in = torch.cuda.Stream(self.ctx.device)
            self.s_out = torch.cuda.Stream(self.ctx.device)
            ev = lambda: [torch.cuda.Event() for _ in range(nch)]  # noqa: E731
            self.ev_in, self.ev_done, self.ev_out = ev(), ev(), ev()
            for e in self.ev_out:
                e.record(self.s_out)

    def e2e_finish(self):
        if self.ctx.world == 1:
            self.ctx.torch.cuda.current_stream(self.ctx.device).wait_stream(self.s_out)

    def e2e_step(self):
        J, h, g, R = self.J, self.halo, self.g, self.R
        if self.ctx.world == 1:
            torch = self.ctx.torch
            main = torch.cuda.current_stream(self.ctx.device)
            x, y = h.bufs[h.cur], h.bufs[1 - h.cur]
            hin, hout = self.hx[self.hcur], self.hx[1 - self.hcur]
            with torch.cuda.stream(self.s_in):
                for k, (lo, hi) in enumerate(self.chunks):
                    # chunk k of hin was last step's y chunk k: wait for its copy out
                    self.s_in.wait_event(self.ev_out[k])
                    x[g + lo:g + hi].copy_(hin[lo:hi], non_blocking=True)
                    self.ev_in[k].record(self.s_in)
            nch = len(self.chunks)
            for k, (lo, hi) in enumerate(self.chunks):
                main.wait_event(self.ev_in[k])
                if k + 1 < nch:
                    main.wait_event(self.ev_in[k + 1])   # rows near the chunk's end read the next
                J.execute(J.SpMVOp, self.views[k], x, y[g + lo:g + hi])
                self.ev_done[k].record(main)
            with torch.cuda.stream(self.s_out):
                for k, (lo, hi) in enumerate(self.chunks):
                    self.s_out.wait_event(self.ev_done[k])
                    hout[lo:hi].copy_(y[g + lo:g + hi], non_blocking=True)
                    self.ev_out[k].record(self.s_out)
            h.cur = 1 - h.cur
            self.hcur = 1 - self.hcur
            return
        if self.p2p:
            t = h.step_no
            h.bufs[t % 2][g:g + R].copy_(self.hx[self.hcur], non_blocking=True)
            y = h.step()
            self.hx[1 - self.hcur].copy_(y[g:g + R], non_blocking=True)
            self.hcur = 1 - self.hcur
            return
        x, y = h.bufs[h.cur], h.bufs[1 - h.cur]
        x[g:g + R].copy_(self.hx[self.hcur], non_blocking=True)
        if self.ctx.world > 1:
            if h.mode == "allgather":
                h._allgather(x)
            else:
                for r in h._exchange(x):
                    r.wait()
        J.execute(J.SpMVOp, self.A, x, y[g:g + R])
        self.hx[1 - self.hcur].copy_(y[g:g + R], non_blocking=True)
        h.cur = 1 - h.cur
        self.hcur = 1 - self.hcur

    # CPU restatement of the reference's path: whole iterations x <- A x while
    # they fit the sample, else a prefix of the rows of one iteration
    def cpu_work(self, frac):
        from oracle import oracle as O
        if not hasattr(self, "crp"):
            self.crp, self.cci, self.cval = self.synth.laplacian_2d(self.g)
        if frac >= 1.0:
            state = {"x": self.x0.copy()}

            def fn():
                state["x"] = O.spmv(self.crp, self.cci, self.cval, state["x"])
            return fn, 2.0 * self.nnz_total, (f"full iterations x <- A x of the {self.g}^2 "
                                              "Laplacian (fp64, oracle row order)")
        rows = max(self.g, int(self.n * frac) // self.g * self.g)
        rp = self.crp[:rows + 1]

        def fn():  # noqa: F811
            O.spmv(rp, self.cci, self.cval, self.x0)
        return fn, 2.0 * int(rp[-1]), f"rows [0, {rows}) of one iteration ({rows / self.n:.4f})"


class Single:
    """Base of the workloads other than the Laplacian.  Subclasses set
    `host()` (the seeded host inputs), `setup()` (this rank's device data) and
    the work model."""

    flush_l2 = False
    launches_per_step = 1
    bound = "hbm"
    unit = "GFLOP/s"
    shardable = False

    def __init__(self, ctx, host_only=False):
        from jlust_b200 import synth
        self.ctx, self.synth = ctx, synth
        self.rank, self.world = ctx.rank, ctx.world
        if not host_only and ctx.world > 1 and not self.shardable:
            raise SystemExit(f"workload {self.profile} runs on one GPU")
        self.host()
        if host_only:
            return
        import torch

        import jlust_b200 as J
        self.J, self.torch = J, torch
        self.dev = ctx.device
        self.setup()

    def shard(self, rowptr):
        """This rank's rows (balanced by rows + entries) and the rebased CSR
        pointer of that slice."""
        from jlust_b200 import dist as D
        r0, r1 = D.partition_by_nnz(rowptr, self.world, self.rank)
        return r0, r1, (rowptr[r0:r1 + 1].astype(np.int64) - int(rowptr[r0])).astype(np.int32)

    def d(self, a):
        return self.torch.from_numpy(np.ascontiguousarray(a)).to(self.dev)

    def bf(self, bits):
        return self.torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(self.dev).view(
            self.torch.bfloat16)

    def reset(self):
        pass

    def close(self):
        pass

    def snapshot(self, k):
        """Host copy of the last timed step's output (checked by parity())."""
        self.snap = [t.cpu().numpy().copy() for t in self.e2e_out()]

    def e2e_setup(self):
        self.e2e_inputs = [t.cpu().pin_memory() for t in self.e2e_in()]
        self.e2e_outputs = [self.torch.empty_like(t, device="cpu").pin_memory() for t in self.e2e_out()]
        self.h2d = self.world * sum(t.numel() * t.element_size() for t in self.e2e_inputs)
        self.d2h = self.world * sum(t.numel() * t.element_size() for t in self.e2e_outputs)

    def e2e_step(self):
        for hd, dv in zip(self.e2e_inputs, self.e2e_in()):
            dv.copy_(hd, non_blocking=True)
        self.api_call()
        for hd, dv in zip(self.e2e_outputs, self.e2e_out()):
            hd.copy_(dv, non_blocking=True)

    def step(self):
        self.api_call()


class SpMV1(Single):
    """Config 1: CSR SpMV fp64, n = 100,000, 10 uniform columns per row."""

    key, kernel, dtype, flush_l2, profile = "cfg1_spmv", "spmv_rows", "f64", True, "spmv1"

    def host(self):
        self.h = self.synth.config1()
        rp = self.h[0]
        self.nnz, self.m = int(rp[-1]), rp.shape[0] - 1

    def setup(self):
        rp, ci, val, x = self.h
        self.A = self.J.csr_tensor(self.d(rp), self.d(ci), self.d(val), (self.m, self.m), origin=0)
        self.x, self.y = self.d(x), self.torch.zeros(self.m, dtype=self.torch.float64, device=self.dev)

    def api_call(self):
        self.J.execute(self.J.SpMVOp, self.A, self.x, self.y)

    def e2e_in(self):
        return [self.x]

    def e2e_out(self):
        return [self.y]

    def flops(self):
        return 2.0 * self.nnz

    def bytes(self):
        return 12.0 * self.nnz + 4.0 * (self.m + 1) + 16.0 * self.m

    def config(self):
        return {"workload": f"cfg1: CSR SpMV fp64, n={self.m}, 10 nnz/row (nnz={self.nnz}), y = A x",
                "l2": "256 MB buffer written between timed launches (inputs 14 MB < L2)"}

    def parity(self):
        from oracle import oracle as O
        rp, ci, val, x = self.h
        return exact_result(exact_check(self.snap[0], O.spmv(rp, ci, val, x)), "all rows of y")

    def cpu_work(self, frac):
        from oracle import oracle as O
        rp, ci, val, x = self.h
        rows = max(1, min(self.m, int(self.m * frac)))
        rps = rp[:rows + 1]
        return (lambda: O.spmv(rps, ci, val, x)), 2.0 * int(rps[-1]), \
            f"rows [0, {rows}) of y = A x (fp64, oracle row order)"


class SpMVRows(SpMV1):
    """CSR SpMV fp64 on other row-length distributions (the choice of the
    vector-per-row variants): `powerlaw` is the cfg3 pattern (Zipf(2) on
    [1, 4096], 4M rows) with fp64 values; `medium` has 4M/8 rows of 40-200
    uniform entries."""

    flush_l2 = False

    def host(self):
        rng_seed = 12
        if self.profile == "spmv_powerlaw":
            rp, ci, _ = self.synth.power_law(4_194_304, 4_194_304, 2.0, 4096, seed=2)
        else:
            m = 524_288
            rng = np.random.default_rng(rng_seed)
            lens = rng.integers(40, 201, size=m)
            rows = np.repeat(np.arange(m, dtype=np.int64), lens)
            cols = rng.integers(0, m, size=rows.shape[0], dtype=np.int64)
            rp, ci = self.synth.csr_from_rows_cols(m, m, rows, cols)
        rng = np.random.default_rng(rng_seed + 1)
        m = rp.shape[0] - 1
        val = rng.uniform(-1.0, 1.0, size=ci.shape[0])
        x = rng.uniform(-1.0, 1.0, size=m)
        self.h = (rp, ci, val, x)
        self.nnz, self.m = int(rp[-1]), m

    def config(self):
        what = ("power-law (the cfg3 pattern, Zipf 2.0 on [1,4096])" if self.profile == "spmv_powerlaw"
                else "medium rows (40-200 uniform entries)")
        return {"workload": f"CSR SpMV fp64, {what}, n={self.m}, nnz={self.nnz}, y = A x",
                "l2": "inputs larger than L2"}


class SpMVPowerLaw(SpMVRows):
    key, profile = "spmv_powerlaw", "spmv_powerlaw"


class SpMVMedium(SpMVRows):
    key, profile = "spmv_medium", "spmv_medium"


class SpMM(Single):
    """Config 3: CSR SpMM fp32, power-law A (4M x 4M), B 4M x 64 row-major."""

    key, kernel, dtype, shardable, profile = "cfg3_spmm", "spmm_stream", "f32", True, "spmm"
    launches_per_step = 2   # spmm_stream + spmm_long_rows

    col_major = False

    def host(self):
        self.h = _HOST.pop("cfg3", None) or self.synth.config3()
        _HOST["cfg3"] = self.h          # kept for the column-major run that follows
        rp, _, _, B = self.h
        self.nnz, self.m, self.k = int(rp[-1]), rp.shape[0] - 1, B.shape[1]

    def setup(self):
        rp, ci, val, B = self.h
        # rows sharded by rows + entries; B replicated on every rank (copied once, untimed)
        r0, r1, lrp = self.shard(rp)
        self.rows = (r0, r1)
        p0, p1 = int(rp[r0]), int(rp[r1])
        self.A = self.J.csr_tensor(self.d(lrp), self.d(ci[p0:p1]), self.d(val[p0:p1]),
                                   (r1 - r0, self.m), origin=0)
        if self.col_major:
            # Julia's native layout: B and C column-major (transposed views
            # of row-major k x n and k x m device arrays)
            self.B = self.d(B).t().contiguous().t()
            self.C = self.torch.zeros(self.k, r1 - r0, dtype=self.torch.float32,
                                      device=self.dev).t()
        else:
            self.B = self.d(B)
            self.C = self.torch.zeros(r1 - r0, self.k, dtype=self.torch.float32, device=self.dev)

    def api_call(self):
        self.J.execute(self.J.SpMMOp, self.A, self.B, self.C)

    def e2e_in(self):
        return [self.B]

    def e2e_out(self):
        return [self.C]

    def flops(self):
        return 2.0 * self.nnz * self.k

    def bytes(self):  # gather model: one B row per stored entry, C written once
        return 8.0 * self.nnz + 4.0 * (self.m + 1) + 4.0 * self.k * (self.nnz + self.m)

    def config(self):
        return {"workload": f"cfg3: CSR SpMM fp32, power-law {self.m}x{self.m} (Zipf 2.0 on "
                            f"[1,4096], nnz={self.nnz}, mean {self.nnz / self.m:.2f}/row), "
                            f"B {self.m}x{self.k} row-major",
                "bytes_model": "gather (8 nnz + 4 (m+1) + 256 nnz + 256 m)",
                "compulsory_bytes": 8.0 * self.nnz + 4.0 * (self.m + 1) + 8.0 * self.k * self.m,
                "partition": f"rows/{self.world} (balanced by rows + entries), B replicated",
                "l2": "inputs larger than L2"}

    def parity(self):
        """Rows of at most 256 entries bit-exact against the fp32 restatement;
        longer rows (summed in segments) within 1e-5 of the fp64 one."""
        from oracle import oracle as O
        rp, ci, val, B = self.h
        r0, r1 = self.rows
        p0, p1 = int(rp[r0]), int(rp[r1])
        lrp = (rp[r0:r1 + 1].astype(np.int64) - p0).astype(np.int32)
        got = self.snap[0]
        lens = np.diff(lrp)
        short = lens <= 256
        want = O.spmm(lrp, ci[p0:p1], val[p0:p1], B)
        bad = exact_check(got[short], want[short])
        longr = np.nonzero(~short)[0]
        sub_rp = np.concatenate([[0], np.cumsum(lens[longr])]).astype(np.int32)
        idx = np.concatenate([np.arange(lrp[r], lrp[r + 1]) for r in longr]) + p0 \
            if longr.size else np.zeros(0, np.int64)
        ref, bound = O.spmm_ref64(sub_rp, ci[idx], val[idx], B)
        per, norm = tol_check(got[longr], ref, bound, 1e-5)
        per = self.ctx.max_over_ranks(per)
        norm = self.ctx.max_over_ranks(norm)
        bad = int(self.ctx.sum_over_ranks(bad))
        r = tol_result(per, norm, 1e-5, f"all {self.m} rows of C")
        r["bit_exact_rows_le_256"] = {"mismatches": bad, "pass": bad == 0}
        r["pass"] = r["pass"] and bad == 0
        return r

    def cpu_work(self, frac):
        from oracle import oracle as O
        rp, ci, val, B = self.h
        if self.col_major and not hasattr(self, "hBf"):
            self.hBf = np.asfortranarray(B)
        Bx = self.hBf if self.col_major else B
        rows = max(1, min(self.m, int(self.m * frac)))
        rps = rp[:rows + 1]
        return (lambda: O.spmm(rps, ci, val, Bx, c_order=1 if self.col_major else 0)), \
            2.0 * int(rps[-1]) * self.k, \
            f"rows [0, {rows}) of C = A B (fp32, Tiled per-(row,col) order)"


class SpMMCol(SpMM):
    """Config 3 with JLUST's native column-major B and C (the layout the
    Julia binding passes): B is transposed into a workspace inside the call."""

    key, profile, col_major = "cfg3_spmm_colmajor", "spmm_col", True
    launches_per_step = 4   # transpose B, spmm_stream, spmm_long_rows, transpose C

    def host(self):
        self.h = _HOST.pop("cfg3", None) or self.synth.config3()
        rp, _, _, B = self.h
        self.nnz, self.m, self.k = int(rp[-1]), rp.shape[0] - 1, B.shape[1]

    def config(self):
        c = super().config()
        c["workload"] = c["workload"].replace("row-major", "column-major, C column-major "
                                              "(Julia's layout; B transposed in the call)")
        return c


class SDDMM(Single):
    """Config 4: SDDMM fp32, 1M x 1M pattern with 32 entries per row, K = 128."""

    key, kernel, dtype, shardable, profile = "cfg4_sddmm", "sddmm_fast", "f32", True, "sddmm"

    col_major = False

    def host(self):
        self.h = _HOST.pop("cfg4", None) or self.synth.config4()
        if not self.col_major:
            _HOST["cfg4"] = self.h      # kept for the column-major run that follows
        rp, _, A, _, _ = self.h
        self.nnz, self.m, self.K = int(rp[-1]), rp.shape[0] - 1, A.shape[1]

    def setup(self):
        rp, ci, A, B, S = self.h
        r0, r1, lrp = self.shard(rp)
        self.rows = (r0, r1)
        p0, p1 = int(rp[r0]), int(rp[r1])
        self.S = self.d(S[p0:p1])
        self.Cs = self.J.csr_tensor(self.d(lrp), self.d(ci[p0:p1]), self.S.clone(),
                                    (r1 - r0, self.m), origin=0)
        self.A, self.Bt = self.d(A[r0:r1]), self.d(B)
        if self.col_major:
            # Julia's native layout: A column-major m x K (B's K x n operand
            # is column-major already: each B(:, j) contiguous)
            self.A = self.A.t().contiguous().t()

    def api_call(self):
        J = self.J
        J.execute(J.SDDMMOp, self.A, self.Bt.t(), self.Cs, mode="mul", S=self.S)

    def e2e_in(self):
        return [self.A, self.Bt]

    def e2e_out(self):
        return [self.Cs.val]

    def flops(self):
        return 2.0 * self.nnz * self.K

    def gather_bytes(self):  # A rows once, one B row per entry
        return 4.0 * self.K * (self.m + self.nnz) + 4.0 * self.nnz + 4.0 * (self.m + 1) + 8.0 * self.nnz

    def bytes(self):
        # the bytes that bound the kernel: its DRAM traffic (ncu); a fifth of
        # the gathered B rows hit L2, so the gather model overstates the bytes
        t = profile_traffic("sddmm_fast_sddmm")
        return t if t is not None else self.gather_bytes()

    def config(self):
        return {"workload": f"cfg4: SDDMM fp32, pattern {self.m}x{self.m} with 32 uniform "
                            f"entries/row (nnz={self.nnz}), A, B {self.m}x{self.K} N(0,1), "
                            "out = dot(A_i, B_j) * S_ij",
                "bytes_model": "DRAM bytes per launch measured by ncu (profiles/sddmm_fast_sddmm.md)",
                "gather_bytes": self.gather_bytes(),
                "partition": f"pattern rows/{self.world}, A rows sharded, B replicated",
                "l2": "inputs larger than L2"}

    def parity(self):
        from oracle import oracle as O
        rp, ci, A, B, S = self.h
        r0, r1 = self.rows
        p0, p1 = int(rp[r0]), int(rp[r1])
        lrp = (rp[r0:r1 + 1].astype(np.int64) - p0).astype(np.int32)
        ref, bound = O.sddmm_ref64(lrp, ci[p0:p1], A[r0:r1], B.T, S=S[p0:p1], mode=1)
        per, norm = tol_check(self.snap[0], ref, bound, 1e-5)
        return tol_result(self.ctx.max_over_ranks(per), self.ctx.max_over_ranks(norm), 1e-5,
                          f"all {self.nnz} sampled entries")

    def cpu_work(self, frac):
        from oracle import oracle as O
        rp, ci, A, B, S = self.h
        rows = max(1, min(self.m, int(self.m * frac)))
        rps = rp[:rows + 1]
        Ss = S[:int(rps[-1])]
        Ax = np.asfortranarray(A[:rows]) if self.col_major else A
        return (lambda: O.sddmm(rps, ci, Ax, B.T, Ss, S=Ss, mode=1)), 2.0 * int(rps[-1]) * self.K, \
            f"pattern rows [0, {rows}) (fp32, sequential K loop)"


class SDDMMCol(SDDMM):
    """Config 4 with JLUST's native column-major A (m x K) and K x n B."""

    key, profile, col_major = "cfg4_sddmm_colmajor", "sddmm_col", True

    def config(self):
        c = super().config()
        c["workload"] += "; A column-major (Julia's layout), B the column-major K x n operand"
        return c


class BSR(Single):
    """Config 5: BSR SpMM bf16 -> fp32, 65,536^2 with 64x64 blocks, band +-8 + 2%."""

    key, kernel, dtype, bound, shardable, profile = ("cfg5_bsr", "bsr_spmm_tc",
                                                     "bf16 in, f32 accumulate", "tensor", True, "bsr")

    def host(self):
        self.h = self.synth.config5()
        bp, bc, _, B = self.h
        self.nnzb, self.mb, self.N = bc.shape[0], bp.shape[0] - 1, B.shape[1]

    def setup(self):
        bp, bc, bv, B = self.h
        n = self.mb * 64
        I0, I1, lbp = self.shard(bp)
        self.brows = (I0, I1)
        q0, q1 = int(bp[I0]), int(bp[I1])
        self.A = self.J.bsr_tensor(self.d(lbp), self.d(bc[q0:q1]), self.bf(bv[q0 * 4096:q1 * 4096]),
                                   ((I1 - I0) * 64, n), (64, 64), origin=0)
        self.B = self.bf(B)
        self.C = self.torch.zeros((I1 - I0) * 64, self.N, dtype=self.torch.float32, device=self.dev)

    def api_call(self):
        self.J.execute(self.J.BlockSpMMOp, self.A, self.B, self.C)

    def e2e_in(self):
        return [self.B]

    def e2e_out(self):
        return [self.C]

    def flops(self):
        return 2.0 * self.nnzb * 64 * 64 * self.N

    def bytes(self):
        n = self.mb * 64
        return 8192.0 * self.nnzb + 2.0 * n * self.N + 4.0 * n * self.N + 4.0 * (self.nnzb + self.mb + 1)

    def config(self):
        return {"workload": f"cfg5: BSR SpMM bf16 (fp32 accumulate), {self.mb * 64}^2 with 64x64 "
                            f"blocks, band +-8 + 2% off-band (nnzb={self.nnzb}), B "
                            f"{self.mb * 64}x{self.N} bf16 row-major",
                "partition": f"block rows/{self.world} (balanced by rows + blocks), B replicated",
                "l2": "A values (311 MB) larger than L2; B (33.5 MB) L2-resident by design",
                "parity_note": "BSR values are pinned by no reference vector (the reference has "
                               "no working BSR SpMM); the check is against the fp64 restatement "
                               "of its block-SpMM loop"}

    def parity(self):
        from oracle import oracle as O
        bp, bc, bv, B = self.h
        I0, I1 = self.brows
        q0 = int(bp[I0])
        lbp = (bp[I0:I1 + 1].astype(np.int64) - q0).astype(np.int32)
        ref, bound = O.bsr_spmm_ref64(lbp, bc[q0:], bv[q0 * 4096:], B)
        per, norm = tol_check(self.snap[0], ref, bound, 1e-5)
        return tol_result(self.ctx.max_over_ranks(per), self.ctx.max_over_ranks(norm), 1e-5,
                          f"all {self.mb * 64} x {self.N} entries of C against the fp64 "
                          "restatement (no reference vector pins BSR values)")

    def cpu_work(self, frac):
        from oracle import oracle as O
        bp, bc, bv, B = self.h
        rows = max(1, min(self.mb, int(self.mb * frac)))
        bps = bp[:rows + 1]
        return (lambda: O.bsr_spmm(bps, bc, bv, B)), 2.0 * int(bps[-1]) * 64 * 64 * self.N, \
            f"block rows [0, {rows}) (fp32, fused-loop order)"


class Convert(Single):
    """CSR -> BSRRight((64, 64)) of the config-5 matrix (bf16 values)."""

    key, kernel, dtype, profile, unit = ("csr2bsr", "count_csr", "bf16 values, int32 indices",
                                         "convert", "Gentries/s")
    # count, three scan launches, then the three tile-row fill kernels and the
    # entry-by-entry one (for block rows that are not ascending)
    launches_per_step = 8

    def host(self):
        bp, bc, bv, _ = self.synth.config5(N=64)
        self.src = (bp, bc, bv)
        rp, ci, vals = self.synth.bsr_to_csr(bp, bc, bv, 64, bp.shape[0] - 1)
        self.h = (rp, ci, vals)
        self.m = rp.shape[0] - 1
        self.nnz = int(rp[-1])
        self.nnzb, self.mb = bc.shape[0], bp.shape[0] - 1

    def setup(self):
        rp, ci, vals = self.h
        self.A = self.J.csr_tensor(self.d(rp), self.d(ci), self.bf(vals), (self.m, self.m), origin=0)

    def api_call(self):
        self.out = self.J.convert_format(self.A, self.J.Formats.BSRRight((64, 64)))

    def e2e_setup(self):
        torch = self.torch
        self.hv = self.A.val.cpu().pin_memory()
        self.hout = torch.empty(self.nnzb * 4096, dtype=torch.bfloat16).pin_memory()
        self.h2d = self.hv.numel() * 2
        self.d2h = self.hout.numel() * 2

    def e2e_step(self):
        self.A.val.copy_(self.hv, non_blocking=True)
        self.api_call()
        self.hout.copy_(self.out.val, non_blocking=True)

    def snapshot(self, k):
        J = self.J
        self.snap = (J.positions(self.out, 2).cpu().numpy(), J.coordinates(self.out, 2).cpu().numpy(),
                     self.out.val.view(self.torch.int16).cpu().numpy().view(np.uint16))

    def flops(self):  # reported as entries converted per second
        return float(self.nnz)

    def bytes(self):
        return (4.0 * (self.m + 1) + 6.0 * self.nnz) + (8192.0 * self.nnzb + 4.0 * self.nnzb +
                                                         4.0 * (self.mb + 1))

    def config(self):
        return {"workload": f"CSR -> BSR 64x64 of the cfg5 matrix ({self.m}^2, nnz={self.nnz}, "
                            f"nnzb={self.nnzb}), count + fill (host sync between)",
                "value_unit_note": "value = G stored entries converted per second"}

    def parity(self):
        """Byte-exact twice: the whole output against the BSR the CSR was
        expanded from (an explicit zero comes back as +0 padding), and the
        first 1/32 of the block rows against the oracle's composer."""
        from oracle import oracle as O
        bp, bc, bv = self.src
        gp, gc, gv = self.snap
        want_v = np.where((bv & 0x7FFF) == 0, np.uint16(0), bv)
        bad = exact_check(gp, bp) + exact_check(gc, bc) + exact_check(gv, want_v)
        rp, ci, vals = self.h
        rows = (self.mb // 32) * 64
        op, oc, ov = O.csr_to_bsr(rows, self.m, rp[:rows + 1], ci, vals, 64, 64)
        nb = int(op[-1])
        bad_o = exact_check(gp[:rows // 64 + 1], op) + exact_check(gc[:nb], oc) + \
            exact_check(gv[:nb * 4096], ov)
        return exact_result(bad + bad_o, f"block row pointer, block columns and all {self.nnzb} "
                                         "tiles against the source BSR; block rows [0, "
                                         f"{rows // 64}) also against the oracle composer")

    def cpu_work(self, frac):
        from oracle import oracle as O
        rp, ci, vals = self.h
        rows = max(64, int(self.m * frac) // 64 * 64)
        return (lambda: O.csr_to_bsr(rows, self.m, rp[:rows + 1], ci, vals, 64, 64)), \
            float(rp[rows]), f"rows [0, {rows}) (the composer is single-threaded)"


class Scan(Single):
    """The cfg2 row-pointer scan: exclusive scan of the Laplacian's 16.8 M
    row lengths (int32) into its row pointer, through the C-ABI with buffers
    allocated once."""

    key, kernel, dtype, flush_l2, profile, unit = ("scan", "scan_tiles_final", "int32", True,
                                                   "scan", "Gcounts/s")
    launches_per_step = 3

    def host(self):
        rp, _, _ = self.synth.laplacian_2d(4096)
        self.h = np.diff(rp).astype(np.int32)
        self.n = self.h.shape[0]

    def setup(self):
        import ctypes as C

        from jlust_b200 import _lib
        from jlust_b200.backend import _stream
        self.counts = self.d(self.h)
        self.out = self.torch.empty(self.n + 1, dtype=self.torch.int32, device=self.dev)
        self.wsb = _lib.load().jlb_scan_workspace_size(self.n)
        self.ws = self.torch.empty(self.wsb, dtype=self.torch.uint8, device=self.dev)
        self._lib, self._st = _lib, _stream(self.torch.device(self.dev))
        self._p = lambda t: C.c_void_p(t.data_ptr())

    def api_call(self):
        p = self._p
        self._lib.call("jlb_exclusive_scan_i32", self._st, self.n, p(self.counts), p(self.out), 0,
                       p(self.ws), self.wsb)

    def e2e_setup(self):
        self.hc = self.counts.cpu().pin_memory()
        self.hout = self.torch.empty(self.n + 1, dtype=self.torch.int32).pin_memory()
        self.h2d, self.d2h = 4 * self.n, 4 * (self.n + 1)

    def e2e_step(self):
        self.counts.copy_(self.hc, non_blocking=True)
        out = self.J.exclusive_scan(self.counts)          # the public call (allocates)
        self.hout.copy_(out, non_blocking=True)

    def snapshot(self, k):
        self.snap = [self.out.cpu().numpy()]

    def flops(self):  # reported as counts scanned per second
        return float(self.n)

    def bytes(self):
        return 4.0 * self.n + 4.0 * (self.n + 1)

    def config(self):
        return {"workload": f"cfg2 row-pointer scan: exclusive scan of {self.n} int32 row "
                            "lengths of the 4096^2 Laplacian",
                "l2": "256 MB buffer written between timed launches (67 MB of counts < L2)",
                "value_unit_note": "value = G counts scanned per second"}

    def parity(self):
        want = np.concatenate([[0], np.cumsum(self.h, dtype=np.int64)]).astype(np.int32)
        return exact_result(exact_check(self.snap[0], want), f"all {self.n + 1} row pointers")

    def cpu_work(self, frac):
        from oracle import oracle as O
        k = max(1, min(self.n, int(self.n * frac)))
        c = self.h[:k]
        return (lambda: O.exclusive_scan(c)), float(k), \
            f"counts [0, {k}) (single-threaded C loop)"


class CooToCsr(Single):
    """COO -> CSR of the cfg2 Laplacian (its 83.9 M fp64 entries given as
    row-ordered COO) through convert_format: count, host read of nnz, fill."""

    key, kernel, dtype, profile, unit = ("coo2csr", "coo_keep_tiles", "f64 values, int32 indices",
                                         "coo2csr", "Gentries/s")
    launches_per_step = 8          # keep, scan of tile counts (3), of row counts (3), emit

    def host(self):
        rp, ci, val, _ = self.synth.config2(g=4096)
        self.m = rp.shape[0] - 1
        self.nnz = int(rp[-1])
        rows = np.repeat(np.arange(self.m, dtype=np.int32), np.diff(rp))
        self.h = (rows, ci, val)
        self.csr = (rp, ci, val)

    def setup(self):
        rows, ci, val = self.h
        self.A = self.J.coo_tensor(self.d(rows), self.d(ci), self.d(val), (self.m, self.m), origin=0)

    def api_call(self):
        self.out = self.J.convert_format(self.A, self.J.Formats.CSR)

    def e2e_setup(self):
        torch = self.torch
        self.hv = self.A.val.cpu().pin_memory()
        self.hout = torch.empty(self.nnz, dtype=torch.float64).pin_memory()
        self.h2d = self.hv.numel() * 8
        self.d2h = self.hout.numel() * 8

    def e2e_step(self):
        self.A.val.copy_(self.hv, non_blocking=True)
        self.api_call()
        self.hout.copy_(self.out.val, non_blocking=True)

    def snapshot(self, k):
        J = self.J
        self.snap = (J.positions(self.out, 2).cpu().numpy(), J.coordinates(self.out, 2).cpu().numpy(),
                     self.out.val.cpu().numpy())

    def flops(self):  # reported as entries converted per second
        return float(self.nnz)

    def bytes(self):  # read rows, cols, values; write colind, values, row pointer
        return 16.0 * self.nnz + 12.0 * self.nnz + 4.0 * (self.m + 1)

    def config(self):
        return {"workload": f"COO -> CSR of the cfg2 Laplacian ({self.m} rows, nnz={self.nnz}, "
                            "fp64), count + host read + fill",
                "value_unit_note": "value = G entries converted per second"}

    def parity(self):
        rp, ci, val = self.csr
        bad = sum(exact_check(g, w) for g, w in zip(self.snap, (rp, ci, val)))
        return exact_result(bad, "row pointer, columns and values against the CSR the COO was "
                                 "expanded from (the composer keeps a row-ordered source's order)")

    def cpu_work(self, frac):
        from oracle import oracle as O
        rows, ci, val = self.h
        k = max(1, min(self.nnz, int(self.nnz * frac)))
        return (lambda: O.coo_to_csr(self.m, self.m, rows[:k], ci[:k], val[:k])), float(k), \
            f"entries [0, {k}) (vectorised numpy composer)"


WORKLOADS = {"laplacian": Laplacian, "spmv1": SpMV1, "spmm": SpMM, "sddmm": SDDMM, "bsr": BSR,
             "convert": Convert, "scan": Scan, "coo2csr": CooToCsr,
             "spmv_powerlaw": SpMVPowerLaw, "spmv_medium": SpMVMedium, "spmm_col": SpMMCol,
             "sddmm_col": SDDMMCol}

# measured beside the headline (one GPU: all; N GPUs: the sharded ones)
EXTRA = ["spmm", "spmm_col", "sddmm", "sddmm_col", "bsr", "convert", "scan"]

# host inputs shared by consecutive workloads of one configuration
_HOST = {}


# ------------------------------------------------------------------- arms --
def timed_flushed(ctx, fn, steps, stream):
    """Like timed(), for inputs smaller than L2: a 256 MB buffer is written
    before every launch and only the launches are timed (CUDA events around
    each one on `stream`, summed)."""
    torch = ctx.torch
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=ctx.device)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    clk = ClockSampler(ctx.device).start()
    ctx.barrier()
    with clk:
        for a, b in evs:
            flush.zero_()
            a.record(stream)
            fn()
            b.record(stream)
        torch.cuda.synchronize(ctx.device)
    secs = sum(a.elapsed_time(b) for a, b in evs) / 1e3
    ctx.barrier()
    return ctx.max_over_ranks(secs), clk.summary()


def cpu_time(step, work_per_step, min_steps=2, max_steps=20, budget_s=20.0):
    """Times `step` on the host: one untimed call, then up to max_steps calls
    or budget_s seconds.  Returns (G units/s, steps timed)."""
    step()
    t0 = time.perf_counter()
    k = 0
    while k < min_steps or (k < max_steps and time.perf_counter() - t0 < budget_s):
        step()
        k += 1
    dt = time.perf_counter() - t0
    return work_per_step * k / dt / 1e9, k


def sample_frac(W, step_s, frac0=1.0 / 256):
    """The fraction of the workload whose CPU step takes about step_s seconds
    (a power of two, at most 1): one calibration call at frac0."""
    fn, _, _ = W.cpu_work(frac0)
    t0 = time.perf_counter()
    fn()
    t = max(time.perf_counter() - t0, 1e-4)
    frac = frac0 * step_s / t
    if frac >= 1.0:
        return 1.0
    return max(frac0, 2.0 ** np.floor(np.log2(frac)))


_THREADS = []


def host_threads():
    """The oracle's thread count at start-up (every host thread OpenMP may
    use), read once: set_threads changes what max_threads reports."""
    if not _THREADS:
        from oracle import oracle as O
        _THREADS.append(O.max_threads())
    return _THREADS[0]


def cpu_leg(W, threads, budget_s):
    """The CPU restatement of the reference's path on `threads` host threads,
    over a sample of W sized to the budget."""
    from oracle import oracle as O
    all_threads = host_threads()
    O.set_threads(threads)
    try:
        frac = sample_frac(W, budget_s / 4)
        fn, work, desc = W.cpu_work(frac)
        v, k = cpu_time(fn, work, min_steps=2, max_steps=20, budget_s=budget_s)
    finally:
        O.set_threads(all_threads)
    return round(v, 4), k, desc


def cpu_baseline(W, budget_s):
    cores = host_threads()
    v, k, desc = cpu_leg(W, cores, budget_s)
    v1, k1, desc1 = cpu_leg(W, 1, budget_s) if cores > 1 else (v, k, desc)
    single = getattr(W, "profile", "") in ("convert", "scan")
    return {"value": v, "unit": W.unit, "cores": 1 if single else cores, "kind": "port",
            "sample": f"{k} steps, {desc}",
            "single_thread": {"value": v1, "cores": 1, "sample": f"{k1} steps, {desc1}"},
            "impl": "C restatement of JLUST's CPU path (oracle/oracle.c)"
                    + (", sequential by construction" if single else ", OpenMP over rows")}


def free_gpu(ctx):
    gc.collect()
    ctx.torch.cuda.synchronize(ctx.device)
    ctx.torch.cuda.empty_cache()


def measure(ctx, W, K, warmup, args):
    """Times W on the GPU(s) and returns its record: value, roofline, e2e,
    cpu_baseline (rank 0, one GPU), parity, launches and clocks."""
    torch = ctx.torch
    import jlust_b200 as J
    stream = torch.cuda.current_stream(ctx.device)
    for _ in range(warmup):
        W.step()
    J.device_status()
    W.reset()
    if getattr(W, "flush_l2", False):
        secs, clocks = timed_flushed(ctx, W.step, K, stream)
    elif hasattr(W, "run_steps"):
        # K launches enqueued by one ABI call (no per-step host overhead)
        secs, clocks = timed(ctx, lambda: W.run_steps(K), 1, stream)
    else:
        secs, clocks = timed(ctx, W.step, K, stream)
    J.device_status()
    W.snapshot(K)
    value = W.flops() * K / secs / 1e9
    eff_gbs = W.bytes() * K / secs / 1e9
    pk = peaks()
    per_launch_s = secs / K
    prof = f"spmv_rows_{W.profile}" if W.kernel == "halo_step" else f"{W.kernel}_{W.profile}"
    traffic = profile_traffic(prof)
    if traffic is not None and ctx.world > 1:
        traffic /= ctx.world        # the capture is of the 1-GPU launch; rows split evenly
    if getattr(W, "bound", "hbm") == "tensor":
        # per GPU, like the HBM roofline: the job's work / N over the step time
        achieved = (W.flops() / ctx.world) / per_launch_s / 1e12
        hbm = (W.bytes() / ctx.world) / per_launch_s / 1e9
        roof = {"bound": "tensor", "kernel": W.kernel, "achieved": round(achieved, 2),
                "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": round(achieved / pk["bf16_tflops"], 4), "traffic": traffic,
                "peak_source": pk["source"] + " (bf16_tflops, cuBLAS burst)",
                "hbm_achieved_gbs": round(hbm, 1), "hbm_frac": round(hbm / pk["hbm_gbs"], 4)}
    else:
        achieved = (W.bytes() / ctx.world) / per_launch_s / 1e9
        roof = {"bound": "hbm", "kernel": W.kernel, "achieved": round(achieved, 1),
                "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                "traffic": traffic, "peak_source": pk["source"] + " (hbm_gbs, copy burst)",
                "algorithmic_bytes_per_launch": W.bytes() / ctx.world}
        if hasattr(W, "gather_bytes"):
            g = (W.gather_bytes() / ctx.world) / per_launch_s / 1e9
            roof["gather_model"] = {"achieved": round(g, 1), "frac": round(g / pk["hbm_gbs"], 4),
                                    "note": "gather model (every B row fetched from DRAM); "
                                            "overstates the bytes, an aside only"}
    if ctx.world > 1:
        roof["note"] = ("per GPU: the job's work / N over the step time (max over ranks)"
                        + (", halo exchange included" if W.profile == "laplacian" else ""))

    parity = None
    if not args.no_parity:
        from oracle import oracle as O
        all_threads = host_threads()
        if ctx.world > 1:
            O.set_threads(max(1, all_threads // ctx.world))
        parity = W.parity()
        O.set_threads(all_threads)

    e2e = None
    if not args.no_e2e:
        W.reset()
        W.e2e_setup()
        for _ in range(2):
            W.e2e_step()
        if hasattr(W, "e2e_finish"):
            W.e2e_finish()
        J.device_status()
        torch.cuda.synchronize(ctx.device)
        e_secs, _ = timed(ctx, W.e2e_step, K, stream, getattr(W, "e2e_finish", None))
        J.device_status()
        e2e = {"value": round(W.flops() * K / e_secs / 1e9, 3), "unit": W.unit,
               "h2d_bytes_per_step": W.h2d, "d2h_bytes_per_step": W.d2h,
               "ms_per_step": round(e_secs * 1e3 / K, 4), "api": "jlust_b200.execute / convert_format"}

    cpu = None
    if ctx.rank == 0 and ctx.world == 1 and not args.no_cpu:
        cpu = cpu_baseline(W, args.cpu_budget)

    launches = int(ctx.sum_over_ranks(W.launches_per_step * K))
    return {"value": round(value, 3), "unit": W.unit, "ms_per_step": round(secs * 1e3 / K, 5),
            "steps": K, "warmup": warmup, "dtype": W.dtype, "config": W.config(),
            "effective_gbs": round(eff_gbs, 1), "roofline": roof, "parity": parity,
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches, "clocks": clocks}


def run_ours(args):
    ctx = Ctx(args)
    W = WORKLOADS[args.workload](ctx)
    r = measure(ctx, W, args.steps, args.warmup, args)
    W.close()
    del W
    line = {"metric": METRIC, "value": r["value"], "unit": r["unit"], "n_gpus": ctx.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": r["dtype"], "data": DATA}
    line.update({k: r[k] for k in ("config", "effective_gbs", "roofline", "cpu_baseline", "e2e",
                                   "parity", "gpu_launches", "clocks")})
    if args.workload == "laplacian" and args.extra == "auto":
        free_gpu(ctx)
        K2, W2 = max(1, min(args.steps, args.extra_steps)), max(3, min(args.warmup, 5))
        extra = {}
        for name in EXTRA:
            cls = WORKLOADS[name]
            if ctx.world > 1 and not cls.shardable:
                continue
            w = cls(ctx)
            extra[cls.key] = measure(ctx, w, K2, W2, args)
            w.close()
            del w
            free_gpu(ctx)
        line["workloads"] = extra
    if ctx.rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()


def run_reference(args):
    """The reference's path on the host cores: the CPU restatement (the
    reference is Julia; no Julia toolchain exists on this box), every host
    thread, each step a bounded sample of the workload, on the same
    workloads as run_ours with the same metric and units."""
    if env_int("RANK", 0) != 0:
        return
    ctx = Ctx(args)
    threads = host_threads()
    K, warm = args.steps, args.warmup

    def one(W, step_s):
        frac = sample_frac(W, step_s)
        fn, work, desc = W.cpu_work(frac)
        for _ in range(warm):
            fn()
        t0 = time.perf_counter()
        for _ in range(K):
            fn()
        dt = time.perf_counter() - t0
        v = work * K / dt / 1e9
        single = getattr(W, "profile", "") in ("convert", "scan")
        return {"value": round(v, 4), "unit": W.unit, "ms_per_step": round(dt * 1e3 / K, 4),
                "steps": K, "warmup": warm, "dtype": W.dtype, "config": W.config(),
                "cpu_baseline": {"value": round(v, 4), "unit": W.unit,
                                 "cores": 1 if single else threads, "kind": "port",
                                 "sample": f"{K} steps, {desc}; C restatement of JLUST's CPU "
                                           "path (oracle/oracle.c)"},
                "e2e": {"value": round(v, 4), "unit": W.unit, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}

    W = WORKLOADS[args.workload](ctx, host_only=True)
    # the headline: full iterations while K of them fit in ~3 minutes
    r = one(W, 180.0 / max(K, 1))
    line = {"metric": METRIC, "value": r["value"], "unit": r["unit"], "n_gpus": args.gpus,
            "steps": K, "warmup": warm, "ms_per_step": r["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": r["dtype"], "data": DATA, "impl": "reference", "config": r["config"],
            "cpu_baseline": r["cpu_baseline"], "e2e": r["e2e"]}
    if args.workload == "laplacian" and args.extra == "auto":
        K2 = max(1, min(args.steps, args.extra_steps))
        K, warm = K2, max(3, min(args.warmup, 5))
        extra = {}
        for name in EXTRA:
            cls = WORKLOADS[name]
            if args.gpus > 1 and not cls.shardable:
                continue
            w = cls(ctx, host_only=True)
            extra[cls.key] = one(w, 0.5)
            del w
            gc.collect()
        line["workloads"] = extra
    print(json.dumps(line), flush=True)


class _CuSparse:
    """The cuSPARSE generic API through ctypes (libcusparse of the CUDA
    toolkit), for the comparison arm only."""

    INDEX_32I, BASE_ZERO, NON_TRANSPOSE, ORDER_COL, ORDER_ROW = 2, 0, 0, 1, 2
    R_32F, R_64F = 0, 1

    def __init__(self, stream):
        import ctypes as C
        self.C = C
        for name in ("libcusparse.so.12", "/usr/local/cuda/lib64/libcusparse.so.12"):
            try:
                self.L = C.CDLL(name)
                break
            except OSError:
                continue
        self.h = C.c_void_p()
        self.ok(self.L.cusparseCreate(C.byref(self.h)), "cusparseCreate")
        self.ok(self.L.cusparseSetStream(self.h, C.c_void_p(stream)), "cusparseSetStream")

    def ok(self, st, what):
        if st != 0:
            raise RuntimeError(f"{what} failed with cuSPARSE status {st}")

    def csr(self, m, n, nnz, rp, ci, val, dt):
        C = self.C
        d = C.c_void_p()
        self.ok(self.L.cusparseCreateCsr(C.byref(d), C.c_int64(m), C.c_int64(n), C.c_int64(nnz),
                                         C.c_void_p(rp), C.c_void_p(ci), C.c_void_p(val),
                                         self.INDEX_32I, self.INDEX_32I, self.BASE_ZERO, dt),
                "cusparseCreateCsr")
        return d

    def vec(self, size, ptr, dt):
        C = self.C
        d = C.c_void_p()
        self.ok(self.L.cusparseCreateDnVec(C.byref(d), C.c_int64(size), C.c_void_p(ptr), dt),
                "cusparseCreateDnVec")
        return d

    def mat(self, rows, cols, ld, ptr, dt, order):
        C = self.C
        d = C.c_void_p()
        self.ok(self.L.cusparseCreateDnMat(C.byref(d), C.c_int64(rows), C.c_int64(cols),
                                           C.c_int64(ld), C.c_void_p(ptr), dt, order),
                "cusparseCreateDnMat")
        return d

    def scalars(self, dt):
        C = self.C
        t = C.c_double if dt == self.R_64F else C.c_float
        self._one, self._zero = t(1.0), t(0.0)
        return C.byref(self._one), C.byref(self._zero)


def run_cusparse(args):
    """cuSPARSE (the reference's default GPU library for SpMM and SDDMM,
    ext/CUDAExt/CUDAExt.jl:234-239, and its CUSPARSEBackend SpMV) through its
    generic API on cfg2 (cusparseSpMV), cfg3 (cusparseSpMM, row-major B and
    C) and cfg4 (cusparseSDDMM, the additive form with beta = 0: cuSPARSE has
    no sampled-times-S mode), timed with CUDA events after a warm-up, as a
    comparison point.  Not part of the product."""
    if env_int("RANK", 0) != 0:
        return
    import ctypes as C
    ctx = Ctx(args)
    torch = ctx.torch
    dev = ctx.device
    stream = torch.cuda.current_stream(dev)
    cs = _CuSparse(stream.cuda_stream)
    K, warm = args.steps, args.warmup

    def d(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    def time_it(fn, flops, byts=None):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize(dev)
        secs, clocks = timed(ctx, lambda: [fn() for _ in range(K)], 1, stream)
        r = {"value": round(flops * K / secs / 1e9, 3), "unit": "GFLOP/s",
             "ms_per_step": round(secs * 1e3 / K, 5), "clocks": clocks}
        if byts:
            r["effective_gbs"] = round(byts * K / secs / 1e9, 1)
        return r

    def buffer(size_fn, *a):
        sz = C.c_size_t(0)
        cs.ok(size_fn(cs.h, *a, C.byref(sz)), "bufferSize")
        return torch.empty(max(int(sz.value), 1), dtype=torch.uint8, device=dev)

    from jlust_b200 import synth
    out = {}
    # cfg2: SpMV fp64
    rp, ci, val, x = synth.config2(g=args.grid)
    n, nnz = rp.shape[0] - 1, int(rp[-1])
    tr, tc, tv, tx = d(rp), d(ci), d(val), d(x)
    ty = torch.zeros(n, dtype=torch.float64, device=dev)
    A = cs.csr(n, n, nnz, tr.data_ptr(), tc.data_ptr(), tv.data_ptr(), cs.R_64F)
    vx, vy = cs.vec(n, tx.data_ptr(), cs.R_64F), cs.vec(n, ty.data_ptr(), cs.R_64F)
    one, zero = cs.scalars(cs.R_64F)
    buf = buffer(cs.L.cusparseSpMV_bufferSize, 0, one, A, vx, zero, vy, cs.R_64F, 0)
    r = time_it(lambda: cs.ok(cs.L.cusparseSpMV(cs.h, 0, one, A, vx, zero, vy, cs.R_64F, 0,
                                                C.c_void_p(buf.data_ptr())), "cusparseSpMV"),
                2.0 * nnz, 12.0 * nnz + 4.0 * (n + 1) + 16.0 * n)
    r["config"] = f"cfg2 Laplacian {args.grid}^2 fp64, y = A x (cusparseSpMV, CUSPARSE_SPMV_ALG_DEFAULT)"
    out["cfg2_laplacian"] = r
    del tr, tc, tv, tx, ty, buf
    free_gpu(ctx)
    # cfg3: SpMM fp32, row-major B and C
    rp, ci, val, B = synth.config3()
    m, nnz, k = rp.shape[0] - 1, int(rp[-1]), B.shape[1]
    tr, tc, tv, tB = d(rp), d(ci), d(val), d(B)
    tC = torch.zeros(m, k, dtype=torch.float32, device=dev)
    A = cs.csr(m, m, nnz, tr.data_ptr(), tc.data_ptr(), tv.data_ptr(), cs.R_32F)
    mB = cs.mat(m, k, k, tB.data_ptr(), cs.R_32F, cs.ORDER_ROW)
    mC = cs.mat(m, k, k, tC.data_ptr(), cs.R_32F, cs.ORDER_ROW)
    one, zero = cs.scalars(cs.R_32F)
    buf = buffer(cs.L.cusparseSpMM_bufferSize, 0, 0, one, A, mB, zero, mC, cs.R_32F, 0)
    r = time_it(lambda: cs.ok(cs.L.cusparseSpMM(cs.h, 0, 0, one, A, mB, zero, mC, cs.R_32F, 0,
                                                C.c_void_p(buf.data_ptr())), "cusparseSpMM"),
                2.0 * nnz * k, 8.0 * nnz + 4.0 * (m + 1) + 4.0 * k * (nnz + m))
    r["config"] = ("cfg3 power-law 4M^2 fp32, C = A B, B 4M x 64 and C row-major "
                   "(cusparseSpMM, CUSPARSE_SPMM_ALG_DEFAULT)")
    out["cfg3_spmm"] = r
    del tr, tc, tv, tB, tC, buf, B
    free_gpu(ctx)
    # cfg4: SDDMM fp32; B (n x K row-major) is the column-major K x n operand
    rp, ci, Am, Bm, S = synth.config4()
    m, nnz, Kd = rp.shape[0] - 1, int(rp[-1]), Am.shape[1]
    tr, tc, tS, tA, tB = d(rp), d(ci), d(S), d(Am), d(Bm)
    P = cs.csr(m, m, nnz, tr.data_ptr(), tc.data_ptr(), tS.data_ptr(), cs.R_32F)
    mA = cs.mat(m, Kd, Kd, tA.data_ptr(), cs.R_32F, cs.ORDER_ROW)
    mB = cs.mat(Kd, m, Kd, tB.data_ptr(), cs.R_32F, cs.ORDER_COL)
    one, zero = cs.scalars(cs.R_32F)
    buf = buffer(cs.L.cusparseSDDMM_bufferSize, 0, 0, one, mA, mB, zero, P, cs.R_32F, 0)
    cs.ok(cs.L.cusparseSDDMM_preprocess(cs.h, 0, 0, one, mA, mB, zero, P, cs.R_32F, 0,
                                        C.c_void_p(buf.data_ptr())), "cusparseSDDMM_preprocess")
    r = time_it(lambda: cs.ok(cs.L.cusparseSDDMM(cs.h, 0, 0, one, mA, mB, zero, P, cs.R_32F, 0,
                                                 C.c_void_p(buf.data_ptr())), "cusparseSDDMM"),
                2.0 * nnz * Kd)
    r["config"] = ("cfg4 pattern 1M^2 32/row fp32, K = 128, out = A B^T at the pattern "
                   "(cusparseSDDMM, beta = 0, after cusparseSDDMM_preprocess)")
    out["cfg4_sddmm"] = r
    print(json.dumps({"impl": "cusparse", "metric": METRIC, "n_gpus": 1, "steps": K,
                      "warmup": warm, "data": DATA, "library": "cuSPARSE (CUDA toolkit, generic API)",
                      "workloads": out}), flush=True)


def main(argv=None):
    args = parse_args(argv)
    if args.impl == "reference":
        run_reference(args)
    elif args.impl == "cusparse":
        run_cusparse(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
