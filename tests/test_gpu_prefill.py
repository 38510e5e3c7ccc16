"""int4 group-quantised weights times a prefill-sized x (more than 16 rows):
the tcgen05 tensor-core GEMM, through the C ABI, against the reference path.

Bar: max|y - y_ref| / max|y_ref| <= 1e-3 (fp32 accumulate) against
cpuDequantMatmulQ4Fallback + cpuMatmul (gpubackend.nim:628-653) at sizes the
C restatement finishes quickly, and against the bit-exact dequantised weights
times x in float64 at prefill sizes.
"""
import numpy as np
import pytest

import pyoracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.fixture(autouse=True, params=[0, 1], ids=["fp16_tiles", "exact_nibbles"])
def prefill_mode(request, nimf_gpu):
    """Every test runs on both int4 GEMMs: AUTO (the fp16-tile GEMM for weights
    that fit fp16 tiles) and EXACT (the exact-nibble GEMM)."""
    nimf_gpu.check(nimf_gpu.lib().nimf_q4_prefill_mode(request.param))
    yield request.param
    nimf_gpu.check(nimf_gpu.lib().nimf_q4_prefill_mode(0))


def rel_err(y, ref):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def quantized(n, k, gs, seed):
    w = (np.random.default_rng(seed).standard_normal((n, k)) * 0.02).astype(np.float32)
    p, s, z = O.quantize_int4_asym_per_group(w, gs)
    return p, s, z, (k + gs - 1) // gs


@pytest.mark.parametrize("n,k,gs,m", [(64, 4096, 128, 17), (200, 1000, 128, 64),
                                      (256, 512, 64, 130), (37, 640, 128, 33),
                                      (128, 256, 64, 128), (48, 512, 256, 40)])
def test_prefill_matches_reference_path(nimf_gpu, n, k, gs, m):
    p, s, z, ngr = quantized(n, k, gs, seed=n + m)
    x = np.random.default_rng(m).standard_normal((m, k)).astype(np.float32)
    w = nimf_gpu.Weight.q4g(p, s, z, n, k, gs, ngr)
    y = w.matmul(x, m)
    y2 = w.matmul(x, m)
    w.free()
    assert np.array_equal(y.view(np.uint32), y2.view(np.uint32))  # deterministic
    ref = O.dequant_matmul_q4(x, p, s, z, m, k, n, gs, ngr)
    assert rel_err(y, ref) <= TOL


@pytest.mark.parametrize("n,k,m", [(4096, 4096, 512), (11008, 4096, 128), (4096, 11008, 256)])
def test_prefill_config_shapes(nimf_gpu, n, k, m):
    """7B-shape prefill projections (512 prompt tokens split in row tiles)."""
    gs = 128
    p, s, z, ngr = quantized(n, k, gs, seed=3)
    x = np.random.default_rng(4).standard_normal((m, k)).astype(np.float32)
    w = nimf_gpu.Weight.q4g(p, s, z, n, k, gs)
    y = w.matmul(x, m)
    w.free()
    wd = O.dequantize_int4_asym(p, s, z, n, k, gs).astype(np.float64)
    ref = x.astype(np.float64) @ wd.T
    assert rel_err(y, ref) <= TOL


def test_prefill_grouped_and_rows_of_x_beyond_tiles(nimf_gpu):
    k, gs, m = 1024, 128, 200
    shapes = [256, 48, 129]
    ws, qs = [], []
    for i, n in enumerate(shapes):
        p, s, z, ngr = quantized(n, k, gs, seed=40 + i)
        qs.append((p, s, z, ngr, n))
        ws.append(nimf_gpu.Weight.q4g(p, s, z, n, k, gs))
    x = np.random.default_rng(7).standard_normal((m, k)).astype(np.float32)
    ys = nimf_gpu.Weight.matmul_group(ws, x, m)
    for w, y, (p, s, z, ngr, n) in zip(ws, ys, qs):
        ref = O.dequant_matmul_q4(x, p, s, z, m, k, n, gs, ngr)
        assert rel_err(y, ref) <= TOL
        w.free()


def test_prefill_zero_and_large_x(nimf_gpu):
    n, k, gs, m = 64, 512, 128, 40
    p, s, z, ngr = quantized(n, k, gs, seed=9)
    w = nimf_gpu.Weight.q4g(p, s, z, n, k, gs)
    assert np.all(w.matmul(np.zeros((m, k), np.float32), m) == 0.0)
    x = np.random.default_rng(2).standard_normal((m, k)).astype(np.float32) * 1e4
    x[5] = 0.0
    ref = O.dequant_matmul_q4(x, p, s, z, m, k, n, gs, ngr)
    assert rel_err(w.matmul(x, m), ref) <= TOL
    w.free()


def test_prefill_group_of_six_shares_one_x_preparation(nimf_gpu):
    """More weights than one launch takes (four): two launches, one prepared x."""
    k, gs, m = 512, 64, 150
    shapes = [128, 64, 200, 16, 130, 256]
    ws, qs = [], []
    for i, n in enumerate(shapes):
        p, s, z, ngr = quantized(n, k, gs, seed=60 + i)
        qs.append((p, s, z, ngr))
        ws.append(nimf_gpu.Weight.q4g(p, s, z, n, k, gs))
    x = np.random.default_rng(8).standard_normal((m, k)).astype(np.float32)
    ys = nimf_gpu.Weight.matmul_group(ws, x, m)
    for w, y, (p, s, z, ngr), n in zip(ws, ys, qs, shapes):
        ref = O.dequant_matmul_q4(x, p, s, z, m, k, n, gs, ngr)
        assert rel_err(y, ref) <= TOL
        w.free()


def test_prefill_mixed_group_sizes_in_one_call(nimf_gpu):
    """Weights of different group sizes sharing x run as one call each."""
    k, m = 512, 48
    specs = [(96, 64), (80, 128)]
    ws, qs = [], []
    for i, (n, gs) in enumerate(specs):
        p, s, z, ngr = quantized(n, k, gs, seed=70 + i)
        qs.append((p, s, z, ngr, n, gs))
        ws.append(nimf_gpu.Weight.q4g(p, s, z, n, k, gs))
    x = np.random.default_rng(9).standard_normal((m, k)).astype(np.float32)
    ys = nimf_gpu.Weight.matmul_group(ws, x, m)
    for w, y, (p, s, z, ngr, n, gs) in zip(ws, ys, qs):
        ref = O.dequant_matmul_q4(x, p, s, z, m, k, n, gs, ngr)
        assert rel_err(y, ref) <= TOL
        w.free()


def test_prefill_zero_points_outside_fp16_split(nimf_gpu):
    """A weight whose zero points do not fit the exact GEMM's split-fp16
    zero-point step (|zp| >= 60000) is computed by the fp16-tile GEMM (its
    values fit fp16 tiles) or, in EXACT mode, on the CUDA-core path; both to
    the bar."""
    n, k, gs, m = 64, 256, 128, 40
    rng = np.random.default_rng(12)
    p = rng.integers(0, 256, size=n * k // 2, dtype=np.uint8)
    s = rng.uniform(1e-6, 2e-6, size=n * 2).astype(np.float32)
    z = rng.uniform(6.0, 9.0, size=n * 2).astype(np.float32)
    z[5] = -70000.0
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = nimf_gpu.Weight.q4g(p, s, z, n, k, gs)
    y = w.matmul(x, m)
    w.free()
    ref = O.dequant_matmul_q4(x, p, s, z, m, k, n, gs, 2)
    assert rel_err(y, ref) <= TOL


@pytest.mark.parametrize("scale", [1e-6, 3e-3, 40.0])
def test_prefill_weight_scales_across_fp16_range(nimf_gpu, scale):
    """Weights far from N(0, 0.02): tiny scales (the fp16 tiles take a
    per-weight power of two) and large ones; within 1e-3 of float64 on every
    path (weights whose groups span too wide a scale range use the exact
    GEMM)."""
    n, k, gs, m = 256, 1024, 128, 300
    rng = np.random.default_rng(31)
    w = (rng.standard_normal((n, k)) * scale).astype(np.float32)
    p, s, z = O.quantize_int4_asym_per_group(w, gs)
    x = rng.standard_normal((m, k)).astype(np.float32)
    h = nimf_gpu.Weight.q4g(p, s, z, n, k, gs)
    y = h.matmul(x, m)
    h.free()
    wd = O.dequantize_int4_asym(p, s, z, n, k, gs).astype(np.float64)
    assert rel_err(y, x.astype(np.float64) @ wd.T) <= TOL


def test_prefill_groups_with_scales_2e30_apart(nimf_gpu):
    """One weight whose group scales differ by 2^30 (one group of each row
    scaled down): too wide for fp16 tiles, so AUTO falls back to the exact
    GEMM; still within 1e-3."""
    n, k, gs, m = 64, 512, 128, 40
    rng = np.random.default_rng(32)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    w[:, :128] *= 2.0 ** -30
    p, s, z = O.quantize_int4_asym_per_group(w, gs)
    x = rng.standard_normal((m, k)).astype(np.float32)
    h = nimf_gpu.Weight.q4g(p, s, z, n, k, gs)
    y = h.matmul(x, m)
    h.free()
    wd = O.dequantize_int4_asym(p, s, z, n, k, gs).astype(np.float64)
    assert rel_err(y, x.astype(np.float64) @ wd.T) <= TOL


def test_prefill_batch8_prompt_rows(nimf_gpu):
    """4096 rows of x (eight 512-token prompts) through a grouped gate/up pair:
    16 x tiles of 256 rows on the fp16-tile GEMM."""
    k, gs, m = 4096, 128, 4096
    ws, ref = [], []
    x = np.random.default_rng(33).standard_normal((m, k)).astype(np.float32)
    for i, n in enumerate((1024, 512)):
        p, s, z, _ = quantized(n, k, gs, seed=40 + i)
        ws.append(nimf_gpu.Weight.q4g(p, s, z, n, k, gs))
        ref.append(O.dequantize_int4_asym(p, s, z, n, k, gs).astype(np.float64))
    ys = nimf_gpu.Weight.matmul_group(ws, x, m)
    for w in ws:
        w.free()
    xd = x.astype(np.float64)
    for y, wd in zip(ys, ref):
        assert rel_err(y, xd @ wd.T) <= TOL
