"""Tensor-core GEMV of the byte-coded float formats (int8, one-byte CustomFloat
E4M3 / E5M2, FP4 E2M1 block-16) through the C ABI, against the CPU oracle.

Dequantisation read back from the tensor-core layout is bit-exact with the
reference rules (quant.nim:64 for int8, customfloat.nim:84-102 for
CustomFloat, the FP4 format definition for FP4); matmul outputs meet
max|y - y_ref| / max|y_ref| <= 1e-3 against float64 sums of the dequantised
weights.  Shapes cover every x-row mode (M <= 4, <= 8, <= 16, chunks of 16),
ragged rows and k, k-splits through the scratch buffer, and the config-3
shape K=8192 (a row slice of N=28672; the full N at the end).  Up to 8 rows
of x run on the mma.sync GEMV, more on the tcgen05 GEMM."""
import numpy as np
import pytest

import pyoracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-3


def rel_err(y, ref):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def config3_weights(n, k, seed=2):
    """W ~ N(0, 0.015) with 0.1% of entries x20 (the FP4 / fp8 config)."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.015).astype(np.float32)
    idx = rng.choice(w.size, max(1, w.size // 1000), replace=False)
    w.flat[idx] *= 20
    return w


def make_fp8(nimf, w, per_channel=True):
    """CustomFloat(4,3) codes of w / s_row with s_row = max|w_row| / 224."""
    n, k = w.shape
    rs = (np.abs(w).max(axis=1) / 224.0).astype(np.float32) if per_channel else None
    src = w / rs[:, None] if per_channel else w
    enc = O.cf_encode(src.astype(np.float32), 4, 3)
    dec = O.cf_decode(enc, 4, 3).reshape(n, k)
    wd = (dec * rs[:, None]).astype(np.float32) if per_channel else dec
    h = nimf.Weight.cf(enc, nimf.newCustomFloat(4, 3), n, k, row_scales=rs)
    return h, wd


def make_fp4(nimf, w):
    n, k = w.shape
    ts = float(np.abs(w).max()) / (6 * 448)
    p, b = O.quantize_fp4_block16(w, ts)
    h = nimf.Weight.fp4(p, b, ts, n, k)
    return h, O.dequantize_fp4_block16(p, b, ts, n, k)


def make_i8(nimf, w, per_channel):
    n, k = w.shape
    if per_channel:
        sc = (np.abs(w).max(axis=1) / 127).astype(np.float32)
        q = np.clip(np.round(w / sc[:, None]), -127, 127).astype(np.int8)
        wd = (q.astype(np.float32) * sc[:, None]).astype(np.float32)
        return nimf.Weight.i8(q, sc, n, k), wd
    q, s = O.quantize_int8(w)
    return nimf.Weight.i8(q, s, n, k), O.dequantize_int8(q, s).reshape(n, k)


MAKERS = {
    "fp8": lambda nimf, w: make_fp8(nimf, w),
    "fp4": make_fp4,
    "i8_tensor": lambda nimf, w: make_i8(nimf, w, False),
    "i8_channel": lambda nimf, w: make_i8(nimf, w, True),
}


@pytest.mark.parametrize("fmt", sorted(MAKERS))
@pytest.mark.parametrize("n,k", [(37, 200), (16, 64), (300, 1000), (129, 4097)])
def test_ragged_shapes_all_modes(nimf_gpu, fmt, n, k):
    w = config3_weights(n, k, seed=n + k)
    h, wd = MAKERS[fmt](nimf_gpu, w)
    assert np.array_equal(h.dequant().view(np.uint32), wd.view(np.uint32))
    rng = np.random.default_rng(k)
    for m in (1, 2, 3, 4, 5, 8, 9, 16, 17, 35):
        x = rng.standard_normal((m, k)).astype(np.float32)
        assert rel_err(h.matmul(x, m), O.gemv_f64(x, wd)) <= TOL, (fmt, n, k, m)
    h.free()


@pytest.mark.parametrize("fmt", ["fp8", "fp4", "i8_channel"])
def test_config3_k8192_row_slice(nimf_gpu, fmt):
    """K=8192 as in the FP4 / fp8 config, 1024 of its 28672 rows, M in {1, 8, 16}
    (M=8 splits k two ways through the scratch partials; M=16 runs on the
    tcgen05 GEMM)."""
    n, k = 1024, 8192
    w = config3_weights(n, k)
    h, wd = MAKERS[fmt](nimf_gpu, w)
    assert np.array_equal(h.dequant().view(np.uint32), wd.view(np.uint32))
    rng = np.random.default_rng(7)
    for m in (1, 8, 16):
        x = rng.standard_normal((m, k)).astype(np.float32)
        y = h.matmul(x, m)
        assert rel_err(y, O.gemv_f64(x, wd)) <= TOL
        # deterministic: a repeated call gives the same bits
        assert np.array_equal(h.matmul(x, m).view(np.uint32), y.view(np.uint32))
    h.free()


def test_e5m2_fast_path_and_special_codes(nimf_gpu):
    """E5M2 runs on the tensor cores; an E4M3 weight holding a code the
    reference decodes differently from OCP FP8 (inf, exponent 0 with a
    mantissa) keeps the generic kernel and still matches the reference."""
    n, k = 48, 512
    rng = np.random.default_rng(5)
    w = rng.standard_normal((n, k)).astype(np.float32)
    x = rng.standard_normal((3, k)).astype(np.float32)
    enc = O.cf_encode(w, 5, 2)
    wd = O.cf_decode(enc, 5, 2).reshape(n, k)
    h = nimf_gpu.Weight.cf(enc, nimf_gpu.newCustomFloat(5, 2), n, k)
    assert np.array_equal(h.dequant().view(np.uint32), wd.view(np.uint32))
    assert rel_err(h.matmul(x, 3), O.gemv_f64(x, wd)) <= TOL
    h.free()
    for special in (0x03, 0x78, 0xFF):
        enc = O.cf_encode(w, 4, 3)
        enc[17] = special
        wd = O.cf_decode(enc, 4, 3).reshape(n, k)
        h = nimf_gpu.Weight.cf(enc, nimf_gpu.newCustomFloat(4, 3), n, k)
        assert np.array_equal(h.dequant().view(np.uint32), wd.view(np.uint32))
        y = h.matmul(x, 3)
        ref = O.gemv_f64(x, wd)
        fin = np.isfinite(ref)
        assert np.array_equal(np.isfinite(y), fin)
        if special == 0x03:
            assert rel_err(y, ref) <= TOL
        h.free()


def test_x_scale_extremes(nimf_gpu):
    """Per-row power-of-two x scaling keeps tiny and huge rows accurate."""
    n, k = 64, 2048
    w = config3_weights(n, k, seed=9)
    h, wd = make_fp4(nimf_gpu, w)
    rng = np.random.default_rng(3)
    x = rng.standard_normal((4, k)).astype(np.float32)
    x[0] *= 1e-30
    x[1] *= 1e30
    x[2] = 0.0
    y = h.matmul(x, 4)
    ref = O.gemv_f64(x, wd)
    for r in (0, 1, 3):
        assert rel_err(y[r], ref[r]) <= TOL
    assert np.all(y[2] == 0.0)
    h.free()


def test_config3_full_size_properties(nimf_gpu):
    """Full FP4 config shape K=8192, N=28672: oddness in x and exact
    power-of-two scaling hold bit for bit, and a row slice matches float64."""
    n, k = 28672, 8192
    rng = np.random.default_rng(2)
    # codes drawn directly (the quantiser on 235M weights is slow on the CPU)
    packed = rng.integers(0, 256, size=n * k // 2, dtype=np.uint8)
    bs = rng.integers(0x20, 0x48, size=n * k // 16, dtype=np.uint8)
    ts = 1e-3
    h = nimf_gpu.Weight.fp4(packed, bs, ts, n, k)
    x = rng.standard_normal((16, k)).astype(np.float32)
    y = h.matmul(x, 16)
    assert np.array_equal(h.matmul(-x, 16), -y)
    assert np.array_equal(h.matmul(x * 4.0, 16), y * 4.0)
    rows = slice(28672 - 512, 28672)
    wd = O.dequantize_fp4_block16(packed[rows.start * k // 2:], bs[rows.start * k // 16:], ts,
                                  512, k)
    assert rel_err(y[:, rows], O.gemv_f64(x, wd)) <= TOL
    h.free()


@pytest.mark.parametrize("fmt", ["fp8", "fp4", "i8_channel", "i8_tensor"])
def test_prefill_tensor_core_gemm(nimf_gpu, fmt):
    """More than 16 rows of x run on the tcgen05 GEMM (x rounded once to fp16
    after a per-row power-of-two scale; measured error about 3e-4 of max|y|):
    K=8192 as in the FP4 / fp8 config, 384 of its rows, prompts of 128 and 512
    rows and a ragged 200 (a partial x tile)."""
    n, k = 384, 8192
    w = config3_weights(n, k, seed=12)
    h, wd = MAKERS[fmt](nimf_gpu, w)
    rng = np.random.default_rng(13)
    for m in (128, 200, 512):
        x = rng.standard_normal((m, k)).astype(np.float32)
        y = h.matmul(x, m)
        assert rel_err(y, O.gemv_f64(x, wd)) <= TOL, (fmt, m)
        assert np.array_equal(h.matmul(x, m).view(np.uint32), y.view(np.uint32))
    h.free()
