"""The allocation-free scan entry point (jlb_exclusive_scan_i32_noalloc).

Some callers cannot call cudaMalloc at the point where they need a scan --
code that must not re-enter a memory pool, such as Julia finalizers and
callbacks while CUDA.jl's allocator is busy, or a device whose memory is all
handed to another allocator.  This entry point keeps its scratch in a static
device array inside the library instead of a caller workspace.  The test calls
it through the C ABI twice in a row and compares each result with the
workspace-based jlb_exclusive_scan_i32 on the same counts (integer results:
bit-exact).  This file sorts last so that a run stopping at the first failure
has already run every other test; it also passes alone in a fresh process,
where its first call performs the per-device scratch lookup.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from jlust_b200 import _lib, errors

pytestmark = pytest.mark.gpu



def _header_limit() -> int:
    """JLB_SCAN_NOALLOC_MAX_N as the public header states it."""
    import os
    import re
    h = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                     "jlust_b200.h")
    return int(re.search(r"#define JLB_SCAN_NOALLOC_MAX_N (\d+)", open(h).read()).group(1))


MAX_N = _header_limit()


def _stream():
    return C.c_void_p(torch.cuda.current_stream(0).cuda_stream)


def _scan_with_workspace(counts: torch.Tensor, base: int) -> torch.Tensor:
    L = _lib.load()
    n = counts.numel()
    out = torch.empty(n + 1, dtype=torch.int32, device="cuda:0")
    wsb = L.jlb_scan_workspace_size(n)
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda:0")
    _lib.check(L.jlb_exclusive_scan_i32(_stream(), n, C.c_void_p(counts.data_ptr()),
                                        C.c_void_p(out.data_ptr()), base,
                                        C.c_void_p(ws.data_ptr()), wsb))
    return out


def _scan_noalloc(counts: torch.Tensor, base: int) -> torch.Tensor:
    L = _lib.load()
    n = counts.numel()
    out = torch.full((n + 1,), -1, dtype=torch.int32, device="cuda:0")
    ptr = C.c_void_p(counts.data_ptr()) if n else C.c_void_p(0)
    _lib.check(L.jlb_exclusive_scan_i32_noalloc(_stream(), n, ptr, C.c_void_p(out.data_ptr()),
                                                base))
    return out


def test_noalloc_scan_matches_workspace_scan_twice():
    torch.cuda.set_device(0)
    rng = np.random.default_rng(71)
    # first call: many tiles; second call: fewer tiles, so stale partial sums
    # from the first call sit in the shared scratch beyond what it reads
    for n, base in ((3_000_001, 1), (70_000, 0)):
        counts = torch.from_numpy(rng.integers(0, 500, size=n).astype(np.int32)).to("cuda:0")
        got = _scan_noalloc(counts, base)
        want = _scan_with_workspace(counts, base)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
        ref = np.concatenate([[base], base + np.cumsum(counts.cpu().numpy(), dtype=np.int64)])
        assert np.array_equal(got.cpu().numpy(), ref.astype(np.int32))
    _lib.check(_lib.load().jlb_device_status(_stream()))


def test_noalloc_scan_limits():
    L = _lib.load()
    out = torch.empty(1, dtype=torch.int32, device="cuda:0")
    st = L.jlb_exclusive_scan_i32_noalloc(_stream(), MAX_N + 1, C.c_void_p(out.data_ptr()),
                                          C.c_void_p(out.data_ptr()), 0)
    assert st == 8 and "static scratch limit" in _lib.last_error()
    with pytest.raises(errors.InvalidArgument):
        _lib.check(st)
    # n = 0 writes just the origin
    got = _scan_noalloc(torch.empty(0, dtype=torch.int32, device="cuda:0"), 1)
    assert got.cpu().tolist() == [1]


def test_noalloc_scan_empty_inside_capture():
    """n = 0 writes out[0] with a kernel on the caller's stream (no host copy,
    no synchronisation), so a call made while a stream is being captured
    records into the graph; the replay writes the origin."""
    _scan_noalloc(torch.empty(0, dtype=torch.int32, device="cuda:0"), 0)   # per-device set-up
    out = torch.full((1,), -1, dtype=torch.int32, device="cuda:0")
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        _lib.check(_lib.load().jlb_exclusive_scan_i32_noalloc(
            _stream(), 0, C.c_void_p(0), C.c_void_p(out.data_ptr()), 1))
    assert out.cpu().tolist() == [-1]       # captured, not run
    g.replay()
    torch.cuda.synchronize()
    assert out.cpu().tolist() == [1]
