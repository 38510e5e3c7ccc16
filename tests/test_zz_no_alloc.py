"""The allocation-free APF format selection (nimf_cf_autoselect_dev_noalloc)
against the allocating nimf_cf_autoselect, through the C ABI.

The entry point keeps its reduction scratch in a fixed device array, so each
pair of calls below must give exactly the format the allocating entry point
chooses for the same data, call after call.  Collected last so it also runs
after everything else has used the library.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _cases():
    rng = np.random.default_rng(11)
    wide = (rng.standard_normal(300_001) * np.exp2(rng.integers(-20, 12, 300_001))).astype(np.float32)
    wide[::13] = 0.0
    w = rng.standard_normal(100_001).astype(np.float32)
    g = (rng.standard_normal(50_001) * 1e-6).astype(np.float32)
    g[::7] = 0.0
    return [
        ("wide", wide, None),
        ("with_grad", w, g),
        ("ragged", rng.standard_normal(1_237).astype(np.float32), rng.standard_normal(3).astype(np.float32)),
        ("nonfinite", np.array([0.0, np.inf, np.nan, -0.0], np.float32), None),
        ("empty", np.zeros(0, np.float32), None),
    ]


def _alloc_select(nimf, x, g):
    e, m = ctypes.c_int(), ctypes.c_int()
    gp = None if g is None else g.ctypes.data_as(ctypes.c_void_p)
    nimf.check(nimf.lib().nimf_cf_autoselect(
        x.ctypes.data_as(ctypes.c_void_p), x.size, gp, 0 if g is None else g.size,
        nimf.APF_DEFAULT_REL_ERROR_TOL, nimf.APF_EXP_MARGIN_BITS, ctypes.byref(e), ctypes.byref(m)))
    return e.value, m.value


def _noalloc_select(nimf, xd, n, gd, ng, stream):
    e, m = ctypes.c_int(-1), ctypes.c_int(-1)
    rc = nimf.lib().nimf_cf_autoselect_dev_noalloc(
        ctypes.c_void_p(xd), n, ctypes.c_void_p(gd) if gd else None, ng,
        nimf.APF_DEFAULT_REL_ERROR_TOL, nimf.APF_EXP_MARGIN_BITS, ctypes.byref(e), ctypes.byref(m),
        ctypes.c_void_p(stream))
    nimf.check(rc)
    return e.value, m.value


def test_noalloc_autoselect_matches_allocating_entry(nimf_gpu):
    import torch
    stream = torch.cuda.current_stream().cuda_stream
    for name, x, g in _cases():
        want = _alloc_select(nimf_gpu, x, g)
        xd = torch.from_numpy(x).cuda()
        gd = None if g is None else torch.from_numpy(g).cuda()
        torch.cuda.synchronize()
        args = (xd.data_ptr() if x.size else 0, x.size,
                0 if gd is None else gd.data_ptr(), 0 if g is None else g.size, stream)
        first = _noalloc_select(nimf_gpu, *args)
        second = _noalloc_select(nimf_gpu, *args)
        assert first == want, name
        assert second == want, name


def _alloc_count(nimf):
    n = ctypes.c_int64()
    nimf.check(nimf.lib().nimf_alloc_count(ctypes.byref(n)))
    return n.value


def test_noalloc_makes_no_device_allocation(nimf_gpu):
    """The library's own allocation counter and torch's allocator both stay
    put across calls (device-wide free memory is not compared: other
    processes on the GPU move it)."""
    import torch
    x = torch.randn(1 << 20, device="cuda")
    g = torch.randn(1 << 16, device="cuda") * 1e-5
    stream = torch.cuda.current_stream().cuda_stream
    args = (x.data_ptr(), x.numel(), g.data_ptr(), g.numel(), stream)
    n0 = _alloc_count(nimf_gpu)
    t0 = torch.cuda.memory_allocated()
    first = _noalloc_select(nimf_gpu, *args)     # the first call on the device does its set-up
    for _ in range(3):
        assert _noalloc_select(nimf_gpu, *args) == first
    assert _alloc_count(nimf_gpu) == n0
    assert torch.cuda.memory_allocated() == t0
    assert first == _alloc_select(nimf_gpu, x.cpu().numpy(), g.cpu().numpy())


def test_noalloc_refuses_a_capturing_stream(nimf_gpu):
    """It reads its reductions back to the host and synchronises, so on a
    stream that is being captured it answers NIMF_ERR_STATE and leaves the
    capture intact."""
    import torch
    x = torch.randn(4096, device="cuda")
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    e, m = ctypes.c_int(-1), ctypes.c_int(-1)
    with torch.cuda.stream(side):
        graph.capture_begin()
        try:
            x.mul_(1.0)
            rc = nimf_gpu.lib().nimf_cf_autoselect_dev_noalloc(
                ctypes.c_void_p(x.data_ptr()), x.numel(), None, 0, 1e-3, 1,
                ctypes.byref(e), ctypes.byref(m), ctypes.c_void_p(side.cuda_stream))
        finally:
            graph.capture_end()
    assert rc == -7 and b"captured" in nimf_gpu.lib().nimf_last_error()
    assert (e.value, m.value) == (-1, -1)
    graph.replay()                               # the capture is still valid
    torch.cuda.synchronize()


def test_noalloc_rejects_oversize_and_bad_arguments(nimf_gpu):
    import torch
    x = torch.ones(16, device="cuda")
    lib = nimf_gpu.lib()
    e, m = ctypes.c_int(), ctypes.c_int()
    # length checks run before any device access
    rc = lib.nimf_cf_autoselect_dev_noalloc(ctypes.c_void_p(x.data_ptr()), 1 << 31, None, 0,
                                            1e-3, 2, ctypes.byref(e), ctypes.byref(m), None)
    assert rc == -2 and b"2147483647" in lib.nimf_last_error()
    rc = lib.nimf_cf_autoselect_dev_noalloc(None, 16, None, 0, 1e-3, 2,
                                            ctypes.byref(e), ctypes.byref(m), None)
    assert rc == -1
    rc = lib.nimf_cf_autoselect_dev_noalloc(ctypes.c_void_p(x.data_ptr()), 16, None, 0, 1e-3, 2,
                                            None, ctypes.byref(m), None)
    assert rc == -1
