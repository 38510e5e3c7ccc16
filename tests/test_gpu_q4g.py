"""int4 asymmetric per-group path on the GPU, through the C ABI, against the
CPU oracle.

Bar: dequantised weights bit-exact with quant.nim's LUT formula; GEMV
outputs within  max|y - y_ref| / max|y_ref| <= 1e-3  (fp32 accumulate) of the
reference path cpuDequantMatmulQ4Fallback + cpuMatmul (gpubackend.nim:628-653).
"""
import ctypes
import glob
import os

import numpy as np
import pytest

import pyoracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOL = 1e-3


def rel_err(y, ref):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def quantized(n, k, gs, seed=0, std=0.02):
    w = (np.random.default_rng(seed).standard_normal((n, k)) * std).astype(np.float32)
    if gs > 0:
        p, s, z = O.quantize_int4_asym_per_group(w, gs)
        ngr = (k + gs - 1) // gs
    else:  # one group per row (gpubackend.nim:645 with groupSize <= 0)
        p, s, z = O.quantize_int4_asym_per_group(w, k)
        ngr = 1
    return p, s, z, ngr


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "q4g_*.npz"))),
                         ids=lambda p: os.path.basename(p))
def test_dequant_bit_exact_on_reference_fixtures(nimf_gpu, path):
    d = np.load(path)
    n, k = d["w"].shape
    gs = int(d["group_size"])
    w = nimf_gpu.Weight.q4g(d["packed"], d["scales"], d["zeros"], n, k, gs)
    try:
        got = w.dequant()
    finally:
        w.free()
    ref = O.dequantize_int4_asym(d["packed"], d["scales"], d["zeros"], n, k, gs)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


SHAPES = [(33, 4096, 128), (16, 200, 64), (50, 1000, 256), (7, 129, 128), (9, 96, 32),
          (5, 40, 40), (3, 64, 0), (17, 4096, 128), (1, 128, 128)]


@pytest.mark.parametrize("n,k,gs", SHAPES)
def test_dequant_bit_exact_random(nimf_gpu, n, k, gs):
    p, s, z, ngr = quantized(n, k, gs, seed=n + k)
    w = nimf_gpu.Weight.q4g(p, s, z, n, k, gs, ngr)
    got = w.dequant()
    w.free()
    ref = O.dequantize_int4_asym(p, s, z, n, k, gs if gs > 0 else k)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 7, 8, 9, 16])
@pytest.mark.parametrize("n,k,gs", [(64, 4096, 128), (37, 1000, 128), (48, 512, 64),
                                    (21, 768, 256), (9, 96, 32), (5, 130, 0), (4096, 11008, 128)])
def test_gemv_matches_reference_path(nimf_gpu, m, n, k, gs):
    if n * k > 10_000_000 and m not in (1, 8):
        pytest.skip("large shape checked at M=1 and 8 only")
    p, s, z, ngr = quantized(n, k, gs, seed=7)
    x = np.random.default_rng(1).standard_normal((m, k)).astype(np.float32)
    w = nimf_gpu.Weight.q4g(p, s, z, n, k, gs, ngr)
    y = w.matmul(x, m)
    w.free()
    ref = O.dequant_matmul_q4(x, p, s, z, m, k, n, gs, ngr)
    assert rel_err(y, ref) <= TOL


@pytest.mark.parametrize("n", [4096, 11008, 12288])
@pytest.mark.parametrize("m", [1, 4, 8])
def test_decode_gemv_config_shapes(nimf_gpu, n, m):
    """int4-g128 decode GEMV shapes: K=4096, N in {4096, 11008, 12288}, M in {1,4,8}."""
    k, gs = 4096, 128
    p, s, z, ngr = quantized(n, k, gs, seed=0)
    x = np.random.default_rng(1).standard_normal((m, k)).astype(np.float32)
    w = nimf_gpu.Weight.q4g(p, s, z, n, k, gs)
    y = w.matmul(x, m)
    y2 = w.matmul(x, m)
    w.free()
    assert np.array_equal(y.view(np.uint32), y2.view(np.uint32))   # deterministic
    ref = O.dequant_matmul_q4(x, p, s, z, m, k, n, gs, ngr)
    assert rel_err(y, ref) <= TOL


def test_beMatmulQ4_dropin(nimf_gpu):
    """Same call as backend.nim:93-110, host arrays in, seq[float32] out."""
    n, k, gs, m = 96, 512, 128, 3
    p, s, z, ngr = quantized(n, k, gs, seed=3)
    a = np.random.default_rng(2).standard_normal(m * k).astype(np.float32)
    ctx = nimf_gpu.newBackend()
    y1 = nimf_gpu.beMatmulQ4(ctx, a, p, s, z, m, k, n, gs, ngr)
    y2 = nimf_gpu.beMatmulQ4(ctx, a, p, s, z, m, k, n, gs, ngr)   # served from the device cache
    assert y1.shape == (m * n,)
    assert np.array_equal(y1, y2)
    ref = O.dequant_matmul_q4(a, p, s, z, m, k, n, gs, ngr).ravel()
    assert rel_err(y1, ref) <= TOL
    nimf_gpu.check(nimf_gpu.lib().nimf_weight_cache_clear())


def test_beMatmulQ4_cache_sees_changed_scales(nimf_gpu):
    """Scales and zeros changed in place behind the same pointers (and the
    packed bytes too) give fresh results, not the cached device copy."""
    n, k, gs, m = 64, 512, 128, 2
    p, s, z, ngr = quantized(n, k, gs, seed=5)
    a = np.random.default_rng(6).standard_normal(m * k).astype(np.float32)
    ctx = nimf_gpu.newBackend()
    L = nimf_gpu.lib()
    nimf_gpu.check(L.nimf_weight_cache_clear())
    y1 = nimf_gpu.beMatmulQ4(ctx, a, p, s, z, m, k, n, gs, ngr)
    s *= np.float32(2.0)                       # in place: same address
    y2 = nimf_gpu.beMatmulQ4(ctx, a, p, s, z, m, k, n, gs, ngr)
    ref2 = O.dequant_matmul_q4(a, p, s, z, m, k, n, gs, ngr).ravel()
    assert rel_err(y2, ref2) <= TOL
    assert rel_err(y2, 2 * y1) <= 1e-5
    z[:] = z[::-1]
    p[: p.size // 2] ^= 0x5A
    y3 = nimf_gpu.beMatmulQ4(ctx, a, p, s, z, m, k, n, gs, ngr)
    assert rel_err(y3, O.dequant_matmul_q4(a, p, s, z, m, k, n, gs, ngr).ravel()) <= TOL
    cnt = ctypes.c_int64()
    nimf_gpu.check(L.nimf_q4_cache_size(ctypes.byref(cnt)))
    assert cnt.value == 1                      # the stale copies were dropped
    nimf_gpu.check(L.nimf_weight_cache_clear())


def test_beMatmulQ4_cache_sees_a_new_weight_at_a_reused_address(nimf_gpu):
    """A weight freed and replaced by another of the same shape in the same
    host buffers (as a GC'd seq whose memory is reused) is registered afresh,
    in every fingerprint mode that reads the contents."""
    n, k, gs, m = 48, 1024, 128, 1
    L = nimf_gpu.lib()
    ctx = nimf_gpu.newBackend()
    a = np.random.default_rng(7).standard_normal(m * k).astype(np.float32)
    p, s, z, ngr = quantized(n, k, gs, seed=8)
    p2, s2, z2, _ = quantized(n, k, gs, seed=9)
    try:
        for mode in (0, 1):                    # FULL, SAMPLED
            nimf_gpu.check(L.nimf_q4_cache_set_check(mode))
            nimf_gpu.check(L.nimf_weight_cache_clear())
            bp, bs, bz = p.copy(), s.copy(), z.copy()
            nimf_gpu.beMatmulQ4(ctx, a, bp, bs, bz, m, k, n, gs, ngr)
            bp[:], bs[:], bz[:] = p2, s2, z2       # the "new" weight, same addresses
            y = nimf_gpu.beMatmulQ4(ctx, a, bp, bs, bz, m, k, n, gs, ngr)
            assert rel_err(y, O.dequant_matmul_q4(a, p2, s2, z2, m, k, n, gs, ngr).ravel()) <= TOL
        # NONE trusts the pointers: the caller clears the cache on replacement
        nimf_gpu.check(L.nimf_q4_cache_set_check(2))
        nimf_gpu.check(L.nimf_weight_cache_clear())
        bp, bs, bz = p.copy(), s.copy(), z.copy()
        y0 = nimf_gpu.beMatmulQ4(ctx, a, bp, bs, bz, m, k, n, gs, ngr)
        bs *= np.float32(3.0)
        assert np.array_equal(nimf_gpu.beMatmulQ4(ctx, a, bp, bs, bz, m, k, n, gs, ngr), y0)
        nimf_gpu.check(L.nimf_weight_cache_clear())
        y = nimf_gpu.beMatmulQ4(ctx, a, bp, bs, bz, m, k, n, gs, ngr)
        assert rel_err(y, 3 * y0) <= 1e-5
        assert L.nimf_q4_cache_set_check(7) == -1
    finally:
        nimf_gpu.check(L.nimf_q4_cache_set_check(0))
        nimf_gpu.check(L.nimf_weight_cache_clear())


def test_row_shards_concatenate_to_full(nimf_gpu):
    n, k, gs, m = 200, 1024, 128, 2
    p, s, z, ngr = quantized(n, k, gs, seed=4)
    x = np.random.default_rng(3).standard_normal((m, k)).astype(np.float32)
    full = nimf_gpu.Weight.q4g(p, s, z, n, k, gs)
    yf = full.matmul(x, m)
    parts = []
    for r0, r1 in [(0, 50), (50, 128), (128, 200)]:
        w = nimf_gpu.Weight.q4g(p, s, z, n, k, gs, rows=(r0, r1))
        assert w.rows == r1 - r0
        parts.append(w.matmul(x, m))
        assert np.array_equal(w.dequant(), full.dequant()[r0:r1])
        w.free()
    full.free()
    assert rel_err(np.concatenate(parts, axis=1), yf) <= 1e-6


def test_device_pointer_entry(nimf_gpu):
    import torch
    n, k, gs, m = 256, 2048, 128, 4
    p, s, z, ngr = quantized(n, k, gs, seed=5)
    w = nimf_gpu.Weight.q4g(p, s, z, n, k, gs)
    x = torch.randn(m, k, device="cuda", dtype=torch.float32)
    y = torch.empty(m, n, device="cuda", dtype=torch.float32)
    st = torch.cuda.current_stream()
    w.matmul_dev(x.data_ptr(), m, y.data_ptr(), st.cuda_stream)
    st.synchronize()
    ref = O.dequant_matmul_q4(x.cpu().numpy(), p, s, z, m, k, n, gs, ngr)
    w.free()
    assert rel_err(y.cpu().numpy(), ref) <= TOL


def test_full_size_properties(nimf_gpu):
    """K=4096, N=12288: odd symmetry is exact, linearity holds to tolerance."""
    n, k, gs = 12288, 4096, 128
    p, s, z, ngr = quantized(n, k, gs, seed=0)
    w = nimf_gpu.Weight.q4g(p, s, z, n, k, gs)
    rng = np.random.default_rng(9)
    x1 = rng.standard_normal((1, k)).astype(np.float32)
    x2 = rng.standard_normal((1, k)).astype(np.float32)
    y1, y2 = w.matmul(x1, 1), w.matmul(x2, 1)
    yn = w.matmul(-x1, 1)
    assert np.array_equal((-y1).view(np.uint32), yn.view(np.uint32))
    y12 = w.matmul(x1 + x2, 1)
    assert rel_err(y12, y1 + y2) <= TOL
    y3 = w.matmul(4.0 * x1, 1)
    assert np.array_equal(y3.view(np.uint32), (4.0 * y1).astype(np.float32).view(np.uint32))
    w.free()


def test_edge_cases(nimf_gpu):
    n, k, gs = 20, 256, 128
    p, s, z, ngr = quantized(n, k, gs, seed=6)
    w = nimf_gpu.Weight.q4g(p, s, z, n, k, gs)
    assert w.matmul(np.zeros((0, k), np.float32), 0).shape == (0, n)
    x = np.zeros((1, k), np.float32)
    assert np.all(w.matmul(x, 1) == 0.0)
    x = np.full((2, k), 1e4, np.float32)
    ref = O.dequant_matmul_q4(x, p, s, z, 2, k, n, gs, ngr)
    assert rel_err(w.matmul(x, 2), ref) <= TOL
    w.free()
    # constant groups (scale 1.0, zero 0.0 in the reference quantiser)
    wc = np.zeros((16, 256), np.float32)
    wc[3] = 0.25
    p, s, z = O.quantize_int4_asym_per_group(wc, 128)
    w = nimf_gpu.Weight.q4g(p, s, z, 16, 256, 128)
    ref_w = O.dequantize_int4_asym(p, s, z, 16, 256, 128)
    assert np.array_equal(w.dequant().view(np.uint32), ref_w.view(np.uint32))
    w.free()


def test_bad_arguments_raise(nimf_gpu):
    p, s, z, ngr = quantized(16, 256, 128)
    with pytest.raises(nimf_gpu.CatchableError, match="SHAPE"):
        nimf_gpu.Weight.q4g(p, s, z, 16, 256, 128, nGroupsPerRow=1)
    with pytest.raises(nimf_gpu.CatchableError, match="SHAPE"):
        nimf_gpu.Weight.q4g(p, s, z, 16, 256, 128, rows=(4, 20))
    w = nimf_gpu.Weight.q4g(p, s, z, 16, 256, 128)
    with pytest.raises(nimf_gpu.CatchableError):
        w.matmul(np.zeros(255, np.float32), 1)
    w.free()
    with pytest.raises(nimf_gpu.CatchableError, match="STATE"):
        w.handle = 999999
        w.matmul(np.zeros(256, np.float32), 1)


@pytest.mark.parametrize("m", [1, 4, 8])
def test_grouped_gemv_matches_individual(nimf_gpu, m):
    """Fused projections sharing x (q/k/v shapes 4096x4096, 4096x1024 x2 and a
    4096x11008 gate/up pair) in one grouped launch."""
    k, gs = 4096, 128
    shapes = [4096, 1024, 1024, 11008, 11008]
    ws, qs = [], []
    for i, n in enumerate(shapes):
        p, s, z, ngr = quantized(n, k, gs, seed=20 + i)
        qs.append((p, s, z, ngr, n))
        ws.append(nimf_gpu.Weight.q4g(p, s, z, n, k, gs))
    x = np.random.default_rng(3).standard_normal((m, k)).astype(np.float32)
    ys = nimf_gpu.Weight.matmul_group(ws, x, m)
    for w, y, (p, s, z, ngr, n) in zip(ws, ys, qs):
        ref = O.dequant_matmul_q4(x, p, s, z, m, k, n, gs, ngr)
        assert rel_err(y, ref) <= TOL
        # the x digit scale is per k-split, which a grouped launch may choose
        # differently from a single one: agreement to ~1e-5, far inside TOL
        assert rel_err(y, w.matmul(x, m)) <= 1e-4
        w.free()


@pytest.mark.parametrize("m", [1, 3])
def test_grouped_host_outputs_contiguous_or_scattered(nimf_gpu, m):
    """nimf_matmul_w_group with host outputs that follow one another in one
    buffer (returned in one copy), in reverse order inside that buffer, and
    with a zero-row weight between them: every layout gives the same bytes."""
    k, gs = 1024, 128
    shapes = [384, 256, 0, 512]
    ws = []
    for i, n in enumerate(shapes):
        p, s, z, _ = quantized(max(n, 64), k, gs, seed=70 + i)
        # n == 0: an empty row shard of a 64-row weight
        ws.append(nimf_gpu.Weight.q4g(p, s, z, max(n, 64), k, gs, rows=(0, n)))
    x = np.random.default_rng(5).standard_normal((m, k)).astype(np.float32)
    want = nimf_gpu.Weight.matmul_group(ws, x, m)
    L = nimf_gpu.lib()
    hs = (ctypes.c_uint64 * len(ws))(*[w.handle for w in ws])
    total = m * sum(shapes)
    offs = np.cumsum([0] + [m * n for n in shapes])
    # contiguous, in call order
    buf = np.full(total, np.nan, np.float32)
    yp = (ctypes.c_void_p * len(ws))(*[buf.ctypes.data + 4 * int(o) for o in offs[:-1]])
    nimf_gpu.check(L.nimf_matmul_w_group(hs, len(ws), x.ctypes.data, m, yp))
    for i, n in enumerate(shapes):
        got = buf[offs[i]:offs[i + 1]].reshape(m, n)
        assert np.array_equal(got, want[i])
    # reverse order inside one buffer: no two outputs follow one another
    roffs = np.cumsum([0] + [m * n for n in shapes[::-1]])[:-1][::-1]
    buf2 = np.full(total, np.nan, np.float32)
    yp2 = (ctypes.c_void_p * len(ws))(*[buf2.ctypes.data + 4 * int(o) for o in roffs])
    nimf_gpu.check(L.nimf_matmul_w_group(hs, len(ws), x.ctypes.data, m, yp2))
    for i, n in enumerate(shapes):
        got = buf2[roffs[i]:roffs[i] + m * n].reshape(m, n)
        assert np.array_equal(got, want[i])
    # the same two layouts in pinned memory: copied straight into the buffers,
    # one copy per run of outputs that follow one another
    import torch
    for layout in (offs[:-1], roffs):
        pbuf = torch.full((total,), float("nan")).pin_memory()
        ypp = (ctypes.c_void_p * len(ws))(*[pbuf.data_ptr() + 4 * int(o) for o in layout])
        nimf_gpu.check(L.nimf_matmul_w_group(hs, len(ws), x.ctypes.data, m, ypp))
        got_all = pbuf.numpy()
        for i, n in enumerate(shapes):
            o = int(layout[i])
            assert np.array_equal(got_all[o:o + m * n].reshape(m, n), want[i])
    for w in ws:
        w.free()


def test_host_buffers_pageable_pinned_and_over_the_stage(nimf_gpu):
    """nimf_matmul_w with pageable x / y (through the library's pinned stage),
    with pinned x / y (copied directly), and with a pageable y larger than the
    4 MiB stage (copied directly): the same bytes every way."""
    import torch
    k, gs, n = 1024, 128, 8192
    p, s, z, ngr = quantized(n, k, gs, seed=81)
    w = nimf_gpu.Weight.q4g(p, s, z, n, k, gs)
    L = nimf_gpu.lib()
    for m in (1, 130):   # 130 rows of y are 4.26 MB
        x = np.random.default_rng(m).standard_normal((m, k)).astype(np.float32)
        y_pageable = w.matmul(x, m)
        assert rel_err(y_pageable, O.dequant_matmul_q4(x, p, s, z, m, k, n, gs, ngr)) <= TOL
        xp = torch.from_numpy(x).pin_memory()
        yp = torch.full((m, n), float("nan")).pin_memory()
        nimf_gpu.check(L.nimf_matmul_w(w.handle, ctypes.c_void_p(xp.data_ptr()), m,
                                       ctypes.c_void_p(yp.data_ptr())))
        assert np.array_equal(yp.numpy(), y_pageable)
        # pinned x, pageable y and the reverse
        yq = np.full((m, n), np.nan, np.float32)
        nimf_gpu.check(L.nimf_matmul_w(w.handle, ctypes.c_void_p(xp.data_ptr()), m,
                                       ctypes.c_void_p(yq.ctypes.data)))
        assert np.array_equal(yq, y_pageable)
        yp.fill_(float("nan"))
        nimf_gpu.check(L.nimf_matmul_w(w.handle, ctypes.c_void_p(x.ctypes.data), m,
                                       ctypes.c_void_p(yp.data_ptr())))
        assert np.array_equal(yp.numpy(), y_pageable)
    w.free()
