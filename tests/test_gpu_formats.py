"""CustomFloat / APF, int8, FP4 and fp32 paths on the GPU through the C ABI,
against the CPU oracle.  Encode / decode / dequantisation are bit-exact;
matmul outputs meet  max|y - y_ref| / max|y_ref| <= 1e-3."""
import numpy as np
import pytest

import pyoracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-3


def rel_err(y, ref):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def specials():
    v = [0.0, -0.0, 1.0, -1.0, 2.0 ** -6, 2.0 ** -7, 240.0, 256.0, 448.0, 65504.0, 65536.0,
         1e-38, 1e-45, -1e-45, 3.4e38, np.inf, -np.inf, np.nan, 1.9999, 0.1, -0.3]
    return np.array(v, np.float32)


def apf_input(n, seed=3):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(n).astype(np.float32)
    idx = rng.choice(n, max(1, n // 100), replace=False)
    x[idx] *= 50
    return x


FORMATS = [(4, 3), (5, 2), (5, 10), (6, 10), (8, 23), (8, 15), (3, 4), (2, 1), (1, 0), (0, 7),
           (11, 52), (8, 39), (7, 31), (10, 5)]


@pytest.mark.parametrize("e,m", FORMATS)
def test_encode_decode_bit_exact(nimf_gpu, e, m):
    ctx = nimf_gpu.newBackend()
    cf = nimf_gpu.newCustomFloat(e, m)
    x = np.concatenate([specials(), apf_input(10007, seed=e * 31 + m),
                        np.random.default_rng(e).standard_normal(33).astype(np.float32) * 1e6])
    enc = nimf_gpu.beCustomfloatEncode(ctx, x, cf)
    ref = O.cf_encode(x, e, m)
    assert np.array_equal(enc, ref)
    dec = nimf_gpu.beCustomfloatDecode(ctx, enc, cf)
    dref = O.cf_decode(ref, e, m)
    assert np.array_equal(dec.view(np.uint32), dref.view(np.uint32))


@pytest.mark.parametrize("e,m", [(4, 3), (5, 10), (6, 10)])
def test_decode_every_byte_pattern(nimf_gpu, e, m):
    """Decoding covers codes the encoder never emits (exp 0 with mantissa,
    exp max with mantissa) exactly as packedU64ToFp32 does."""
    cf = nimf_gpu.newCustomFloat(e, m)
    item = cf.itemSize
    if item == 1:
        buf = np.arange(256, dtype=np.uint8)
    else:
        rng = np.random.default_rng(0)
        buf = rng.integers(0, 256, size=item * 70001, dtype=np.uint8)
    dec = nimf_gpu.beCustomfloatDecode(nimf_gpu.newBackend(), buf, cf)
    assert np.array_equal(dec.view(np.uint32), O.cf_decode(buf, e, m).view(np.uint32))


def test_unaligned_and_ragged_lengths(nimf_gpu):
    ctx = nimf_gpu.newBackend()
    for n in [0, 1, 15, 16, 17, 1023]:
        x = np.random.default_rng(n).standard_normal(n).astype(np.float32)
        for e, m in [(4, 3), (6, 10)]:
            cf = nimf_gpu.newCustomFloat(e, m)
            enc = nimf_gpu.beCustomfloatEncode(ctx, x, cf)
            assert np.array_equal(enc, O.cf_encode(x, e, m))
    with pytest.raises(nimf_gpu.CatchableError):
        nimf_gpu.beCustomfloatDecode(ctx, np.zeros(5, np.uint8), nimf_gpu.newCustomFloat(6, 10))
    with pytest.raises(nimf_gpu.CatchableError):
        nimf_gpu.beCustomfloatEncode(ctx, np.zeros(4, np.float32), nimf_gpu.newCustomFloat(11, 60))


def test_apf_autoselect_and_cast(nimf_gpu):
    ctx = nimf_gpu.newBackend()
    for n, seed in [(1000, 1), (200000, 3), (1 << 20, 4)]:
        x = apf_input(n, seed)
        cf = nimf_gpu.buildCustomDtypeForTensor(x)
        assert (cf.exponentBits, cf.mantissaBits) == O.cf_build_for_tensor(x)
        data, cf2 = nimf_gpu.beApfCastForTraining(ctx, x)
        assert cf2 == cf
        assert np.array_equal(data, O.cf_encode(x, cf.exponentBits, cf.mantissaBits))
    # gradient-aware mantissa width uses medians (customfloat.nim:179-196)
    rng = np.random.default_rng(8)
    w = rng.standard_normal(100001).astype(np.float32)
    g = (rng.standard_normal(50001) * 1e-6).astype(np.float32)
    g[::7] = 0.0
    cf = nimf_gpu.buildCustomDtypeForTensor(w, g)
    assert (cf.exponentBits, cf.mantissaBits) == O.cf_build_for_tensor(w, g)
    assert cf.mantissaBits > 10
    # all-zero / non-finite tensors
    z = np.array([0.0, np.inf, np.nan], np.float32)
    cf = nimf_gpu.buildCustomDtypeForTensor(z)
    assert (cf.exponentBits, cf.mantissaBits) == (1, 2)


def test_cf_weight_gemv_and_dequant(nimf_gpu):
    n, k = 96, 4096
    rng = np.random.default_rng(11)
    w = rng.standard_normal((n, k)).astype(np.float32)
    x = rng.standard_normal((3, k)).astype(np.float32)
    for e, m in [(4, 3), (5, 10), (6, 10)]:
        enc = O.cf_encode(w, e, m)
        wd = O.cf_decode(enc, e, m).reshape(n, k)
        h = nimf_gpu.Weight.cf(enc, nimf_gpu.newCustomFloat(e, m), n, k)
        assert np.array_equal(h.dequant().view(np.uint32), wd.view(np.uint32))
        ref = O.cpu_matmul(x, np.ascontiguousarray(wd.T), 3, k, n)
        assert rel_err(h.matmul(x, 3), ref) <= TOL
        h.free()
    # per-channel scale extension
    rs = rng.uniform(0.5, 2, n).astype(np.float32)
    enc = O.cf_encode(w, 4, 3)
    h = nimf_gpu.Weight.cf(enc, nimf_gpu.newCustomFloat(4, 3), n, k, row_scales=rs)
    wd = (O.cf_decode(enc, 4, 3).reshape(n, k) * rs[:, None]).astype(np.float32)
    assert np.array_equal(h.dequant().view(np.uint32), wd.view(np.uint32))
    assert rel_err(h.matmul(x, 3), O.gemv_f64(x, wd)) <= TOL
    h.free()


def test_int8_config_layer(nimf_gpu):
    """x[1,1024] ~N(0,1), W[1024,1024] ~N(0,0.02) seed 0, quant.nim int8."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((1, 1024)).astype(np.float32)
    w = (rng.standard_normal((1024, 1024)) * 0.02).astype(np.float32)
    q, s = O.quantize_int8(w)
    h = nimf_gpu.Weight.i8(q, s, 1024, 1024)
    wd = O.dequantize_int8(q, s).reshape(1024, 1024)
    assert np.array_equal(h.dequant().view(np.uint32), wd.view(np.uint32))
    # the reference path: dequantizeTensorTransposed + beMatmul (cpuMatmul)
    wt = O.dequantize_transposed(1, q.view(np.uint8), np.array([s]), np.array([0.0]), 1024, 1024, 0)
    ref = O.cpu_matmul(x, wt, 1, 1024, 1024)
    assert rel_err(h.matmul(x, 1), ref) <= TOL
    h.free()
    # per-output-channel scales (extension)
    sc = (np.abs(w).max(axis=1) / 127).astype(np.float32)
    qc = np.clip(np.round(w / sc[:, None]), -127, 127).astype(np.int8)
    h = nimf_gpu.Weight.i8(qc, sc, 1024, 1024)
    wd = (qc.astype(np.float32) * sc[:, None]).astype(np.float32)
    assert np.array_equal(h.dequant().view(np.uint32), wd.view(np.uint32))
    for m in (1, 5, 8, 11):
        xm = rng.standard_normal((m, 1024)).astype(np.float32)
        assert rel_err(h.matmul(xm, m), O.gemv_f64(xm, wd)) <= TOL
    h.free()


@pytest.mark.parametrize("fmt", ["e4m3", "fp4"])
def test_byte_format_gemv_every_row_count(nimf_gpu, fmt):
    """The byte-format GEMV at every x row count it serves (1 .. 16): hi + lo
    x parts up to 4 rows, one fp16 term above, a k-split at K = 8192 for the
    larger counts; each within 1e-3 of float64, and the same bits on a repeat
    (fixed summation order)."""
    rng = np.random.default_rng(21)
    n, k = 272, 8192
    w = (rng.standard_normal((n, k)) * 0.015).astype(np.float32)
    if fmt == "e4m3":
        enc = O.cf_encode(w, 4, 3)
        wd = O.cf_decode(enc, 4, 3).reshape(n, k)
        h = nimf_gpu.Weight.cf(enc, nimf_gpu.newCustomFloat(4, 3), n, k)
    else:
        ts = float(np.abs(w).max()) / (6 * 448)
        p, b = O.quantize_fp4_block16(w, ts)
        h = nimf_gpu.Weight.fp4(p, b, ts, n, k)
        wd = O.dequantize_fp4_block16(p, b, ts, n, k)
    for m in (1, 2, 4, 5, 7, 8, 9, 12, 16):
        x = rng.standard_normal((m, k)).astype(np.float32)
        y = h.matmul(x, m)
        assert rel_err(y, O.gemv_f64(x, wd)) <= TOL, m
        assert np.array_equal(y, h.matmul(x, m)), m
    h.free()


def test_fp4_block16(nimf_gpu):
    rng = np.random.default_rng(2)
    n, k = 64, 8192
    w = (rng.standard_normal((n, k)) * 0.015).astype(np.float32)
    idx = rng.choice(w.size, w.size // 1000, replace=False)
    w.flat[idx] *= 20
    ts = float(np.abs(w).max()) / (6 * 448)
    p, b = O.quantize_fp4_block16(w, ts)
    h = nimf_gpu.Weight.fp4(p, b, ts, n, k)
    wd = O.dequantize_fp4_block16(p, b, ts, n, k)
    assert np.array_equal(h.dequant().view(np.uint32), wd.view(np.uint32))
    for m in (1, 16):
        x = rng.standard_normal((m, k)).astype(np.float32)
        assert rel_err(h.matmul(x, m), O.gemv_f64(x, wd)) <= TOL
    h.free()


def test_beMatmul_and_beMatmul2(nimf_gpu):
    ctx = nimf_gpu.newBackend()
    rng = np.random.default_rng(4)
    a = rng.standard_normal((5, 300)).astype(np.float32)
    b = rng.standard_normal((300, 70)).astype(np.float32)
    y = nimf_gpu.beMatmul(ctx, a, 5, 300, b, 300, 70)
    assert rel_err(y, O.cpu_matmul(a, b, 5, 300, 70).ravel()) <= TOL
    a2 = rng.standard_normal((3, 70)).astype(np.float32)
    b2 = rng.standard_normal((70, 11)).astype(np.float32)
    y1, y2 = nimf_gpu.beMatmul2(ctx, a, 5, 300, b, 300, 70, a2, 3, 70, b2, 70, 11)
    assert np.array_equal(y1, y)
    assert rel_err(y2, O.cpu_matmul(a2, b2, 3, 70, 11).ravel()) <= TOL
    with pytest.raises(nimf_gpu.CatchableError, match="SHAPE"):
        nimf_gpu.check(nimf_gpu.lib().nimf_matmul_f32(None, 1, 2, None, 3, 1, None))
    h = nimf_gpu.Weight.f32(b, 300, 70)
    assert np.array_equal(h.dequant(), np.ascontiguousarray(b.T))
    assert rel_err(h.matmul(a, 5), O.cpu_matmul(a, b, 5, 300, 70)) <= TOL
    h.free()


@pytest.mark.parametrize("m,k,n", [(1, 1024, 1024), (3, 4096, 1000), (8, 300, 70), (9, 257, 131),
                                   (130, 512, 384), (256, 1024, 640), (1, 7, 5), (17, 3, 2)])
def test_beMatmul_hand_written_kernels(nimf_gpu, m, k, n):
    """beMatmul's fp32 kernels (f32.cu: the GEMV for M <= 8 with its split-K
    reduction, the tiled GEMM above), vector and ragged shapes, against the
    reference's cpuMatmul order and against float64; repeat calls are
    bit-identical (fixed summation order)."""
    ctx = nimf_gpu.newBackend()
    rng = np.random.default_rng(m * 1000 + n)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    a[0, : min(k, 5)] = 0.0          # cpuMatmul skips zero a values
    y = np.asarray(nimf_gpu.beMatmul(ctx, a, m, k, b, k, n), dtype=np.float32)
    assert rel_err(y, O.cpu_matmul(a, b, m, k, n).ravel()) <= TOL
    assert rel_err(y, (a.astype(np.float64) @ b.astype(np.float64)).ravel()) <= 1e-5
    y2 = np.asarray(nimf_gpu.beMatmul(ctx, a, m, k, b, k, n), dtype=np.float32)
    assert np.array_equal(y.view(np.uint32), y2.view(np.uint32))
