"""The CPU oracle against the reference's own outputs (golden fixtures made by
tests/golden/gen_golden.py from export_to_nimq.py) and against known-answer
vectors derived by hand from customfloat.nim / quant.nim."""
import glob
import json
import os
import struct

import numpy as np
import pytest

import pyoracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _u32(a):
    return np.asarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "q4g_*.npz"))),
                         ids=lambda p: os.path.basename(p))
def test_int4_per_group_quantizer_matches_reference(path):
    d = np.load(path)
    packed, scales, zeros = O.quantize_int4_asym_per_group(d["w"], int(d["group_size"]))
    assert np.array_equal(packed, d["packed"])
    assert np.array_equal(_u32(scales), _u32(d["scales"]))
    assert np.array_equal(_u32(zeros), _u32(d["zeros"]))


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "i8_*.npz"))),
                         ids=lambda p: os.path.basename(p))
def test_int8_quantizer_matches_reference(path):
    d = np.load(path)
    q, s = O.quantize_int8_vectorized(d["w"])
    assert np.array_equal(q, d["q"].ravel())
    assert float(s) == float(d["scale"])


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "gptq_*.npz"))),
                         ids=lambda p: os.path.basename(p))
def test_gptq_dequant_matches_reference(path):
    d = np.load(path)
    w = O.dequantize_gptq_linear(d["qweight"], d["qzeros"], d["scales"], d["g_idx"])
    assert np.array_equal(_u32(w), _u32(d["weight"]))


def test_fixture_provenance_recorded():
    meta = json.load(open(os.path.join(GOLD, "meta.json")))
    assert meta["reference_module"] == "export_to_nimq.py"
    assert "numpy" in meta


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "q4g_*.npz"))),
                         ids=lambda p: os.path.basename(p))
def test_int4_dequant_is_the_lut_formula(path):
    """quant.nim:146-167: w = (float32(nib) - zp) * sc per group, with the
    same two float32 roundings numpy applies element-wise."""
    d = np.load(path)
    w, gs = d["w"], int(d["group_size"])
    rows, cols = w.shape
    out = O.dequantize_int4_asym(d["packed"], d["scales"], d["zeros"], rows, cols, gs)
    bpr = (cols + 1) // 2
    pk = d["packed"].reshape(rows, bpr)
    c = np.arange(cols)
    nib = np.where(c % 2 == 0, pk[:, c // 2] & 15, pk[:, c // 2] >> 4).astype(np.float32)
    ngr = (cols + gs - 1) // gs
    sc = d["scales"].reshape(rows, ngr)[:, c // gs]
    zp = d["zeros"].reshape(rows, ngr)[:, c // gs]
    ref = (nib - zp).astype(np.float32) * sc
    assert np.array_equal(_u32(out), _u32(ref.astype(np.float32)))
    # quantisation error is bounded by half a step per element
    assert np.all(np.abs(out - w) <= 0.5 * sc * (1 + 1e-5) + 1e-7)
    # transposed variant (quant.nim:256-290) is the exact transpose
    outT = O.dequantize_transposed(3, d["packed"], d["scales"], d["zeros"], rows, cols, gs)
    assert np.array_equal(_u32(outT), _u32(out.T))
    # gpubackend.nim:628-653 uses the same LUT
    x = np.random.default_rng(0).standard_normal((2, cols)).astype(np.float32)
    y = O.dequant_matmul_q4(x, d["packed"], d["scales"], d["zeros"], 2, cols, rows, gs, ngr)
    y2 = O.cpu_matmul(x, np.ascontiguousarray(out.T), 2, cols, rows)
    assert np.array_equal(_u32(y), _u32(y2))


def test_cpu_matmul_order_and_zero_skip():
    """gpubackend.nim:560-582 sums over k ascending and skips a == 0, so
    0 * inf never poisons the result."""
    a = np.array([[1.0, 0.0, 2.0]], np.float32)
    b = np.array([[1.0], [np.inf], [3.0]], np.float32)
    assert O.cpu_matmul(a, b, 1, 3, 1)[0, 0] == 7.0
    rng = np.random.default_rng(5)
    a = rng.standard_normal((3, 130)).astype(np.float32)
    b = rng.standard_normal((130, 70)).astype(np.float32)
    c = O.cpu_matmul(a, b, 3, 130, 70)
    ref = np.zeros((3, 70), np.float32)
    for p in range(130):          # sequential float32 sum over k
        ref = (ref + (a[:, p:p + 1] * b[p:p + 1, :]).astype(np.float32)).astype(np.float32)
    assert np.array_equal(_u32(c), _u32(ref))


def test_int8_nim_rounding_is_half_away_from_zero():
    """quant.nim:60 uses Nim round (half away from zero), unlike numpy."""
    w = np.array([127.0, 0.5, -0.5, 1.5, 2.5], np.float32)
    q, s = O.quantize_int8(w)
    assert s == np.float32(1.0)
    assert list(q) == [127, 1, -1, 2, 3]
    assert np.array_equal(O.dequantize_int8(q, s), np.array([127, 1, -1, 2, 3], np.float32))


def test_int4_symmetric_roundtrip():
    w = np.array([-7, -3.5, 0, 3.5, 7, 1], np.float32)
    p, s = O.quantize_int4_sym(w)
    assert s == np.float32(1.0)
    out = O.dequantize_int4_sym(p, w.size, s)
    assert list(out) == [-7, -4, 0, 4, 7, 1]


# ------------------------------------------------------------ CustomFloat KATs
E4M3 = (4, 3)
E5M10 = (5, 10)


@pytest.mark.parametrize("x,code", [
    (1.0, 0x38), (-1.0, 0xB8), (240.0, 0x77), (255.9, 0x77), (256.0, 0x78), (1e30, 0x78),
    (2.0 ** -6, 0x08), (2.0 ** -7, 0x00), (-2.0 ** -7, 0x80), (0.0, 0x00), (-0.0, 0x80),
    (float("inf"), 0x78), (float("-inf"), 0xF8), (float("nan"), 0x78), (1.9999, 0x3F),
    (1e-45, 0x00),
])
def test_e4m3_encode_kat(x, code):
    """customfloat.nim:49-78: bias 7, truncation, overflow/NaN -> inf, no subnormals."""
    assert O.cf_pack(np.float32(x), *E4M3) == code


@pytest.mark.parametrize("code,val", [
    (0x38, 1.0), (0x77, 240.0), (0x08, 2.0 ** -6), (0x00, 0.0), (0x01, 2.0 ** -7 * 1.125),
    (0x78, float("inf")), (0x7F, float("inf")), (0xF8, float("-inf")),
])
def test_e4m3_decode_kat(code, val):
    """customfloat.nim:80-102: exp==maxExp -> inf regardless of mantissa;
    exp==0 with a non-zero mantissa decodes as 2^(0-bias) * 1.m."""
    assert O.cf_unpack(code, *E4M3) == np.float32(val)


def test_e4m3_negative_zero_sign():
    v = O.cf_unpack(0x80, *E4M3)
    assert v == 0.0 and np.signbit(v)


def test_e5m10_equals_fp16_on_encoder_outputs():
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(4096) * 10).astype(np.float32)
    enc = O.cf_encode(x, *E5M10).view(np.uint16)
    # truncation toward zero of the float32 mantissa
    dec = O.cf_decode(enc.view(np.uint8), *E5M10)
    ref = enc.view(np.float16).astype(np.float32)
    assert np.array_equal(_u32(dec), _u32(ref))
    assert np.all(np.abs(dec) <= np.abs(x))


def test_multi_byte_items_little_endian():
    e, m = 6, 10     # 17 bits -> itemSize 3
    x = np.array([1.0, -3.5, 1e-12, 1e12], np.float32)
    enc = O.cf_encode(x, e, m)
    assert enc.size == 12
    for i, v in enumerate(x):
        p = O.cf_pack(v, e, m)
        assert list(enc[3 * i:3 * i + 3]) == [p & 255, (p >> 8) & 255, (p >> 16) & 255]
    assert np.array_equal(O.cf_decode(enc, e, m)[:2], np.array([1.0, -3.5], np.float32))


def test_wide_formats_roundtrip_exactly():
    """Formats with >= 8 exponent bits and >= 23 mantissa bits hold every
    normal float32 exactly (e8m23, e8m31, e11m52)."""
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(1000) * np.exp(rng.uniform(-30, 30, 1000))).astype(np.float32)
    for e, m in [(8, 23), (8, 31), (8, 39), (11, 52)]:
        assert np.array_equal(_u32(O.cf_decode(O.cf_encode(x, e, m), e, m)), _u32(x))


def test_apf_autoselect_kats():
    """customfloat.nim:149-198."""
    x = np.array([1.0, 2.0, 4.0], np.float32)
    # span = 2 - 0 + 2 + 2 = 6 -> ceil(log2 6) = 3
    assert O.cf_required_exponent_bits(x) == 3
    assert O.cf_required_mantissa_bits(x) == 10      # ceil(log2(1000))
    assert O.cf_required_exponent_bits(np.zeros(4, np.float32)) == 1
    assert O.cf_required_mantissa_bits(np.zeros(4, np.float32)) == 2
    # gradients far smaller than weights need extra mantissa bits
    g = np.full(3, 2.0 ** -15, np.float32)
    # ratio = 2^-15 / 2 = 2^-16 -> need 16 -> extra 6 -> 16
    assert O.cf_required_mantissa_bits(x, 1e-3, g) == 16
    # N(0,1) with 1% x50 outliers (the APF workload): the exponent width
    # follows from the dynamic range of |x| (e5 at 2e5 samples; the 64M-sample
    # workload spans more binades and selects e6)
    rng = np.random.default_rng(3)
    x = rng.standard_normal(200000).astype(np.float32)
    idx = rng.choice(x.size, x.size // 100, replace=False)
    x[idx] *= 50
    a = np.abs(x[x != 0]).astype(np.float64)
    span = int(np.floor(np.log2(a.max()))) - int(np.floor(np.log2(a.min()))) + 4
    assert O.cf_build_for_tensor(x) == (int(np.ceil(np.log2(span))), 10)


def test_fp4_e2m1_value_set_and_roundtrip():
    vals = [O.lib().orc_e2m1_to_float(i) for i in range(16)]
    assert vals[:8] == [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    assert vals[8:] == [-0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]
    for code in range(256):
        v = O.e4m3_ocp_to_float(code)
        if np.isnan(v):
            continue
        assert O.float_to_e4m3_ocp(v) == code or v == 0.0
    rng = np.random.default_rng(2)
    w = (rng.standard_normal((8, 64)) * 0.015).astype(np.float32)
    ts = float(np.abs(w).max()) / (6 * 448)
    p, b = O.quantize_fp4_block16(w, ts)
    d = O.dequantize_fp4_block16(p, b, ts, 8, 64)
    blocks = np.abs(w.reshape(8, 4, 16)).max(axis=2, keepdims=True)
    err = np.abs(d - w).reshape(8, 4, 16)
    assert np.all(err <= blocks * 0.25 + 1e-9)      # half an E2M1 step at the top binade


def test_nimq_stream_layout():
    """The exporter's .nimq stream (export_to_nimq.py:580-605) carries the
    int4 per-group tensor bit-exactly as the quantizer produced it."""
    raw = open(os.path.join(GOLD, "nimq_small.bin"), "rb").read()
    src = np.load(os.path.join(GOLD, "nimq_small_src.npz"))
    off = 0

    def take(fmt):
        nonlocal off
        v = struct.unpack_from(fmt, raw, off)
        off += struct.calcsize(fmt)
        return v

    (n,) = take("<i")
    assert raw[off:off + n] == b"NIMQ2"
    off += n
    arch = take("<5i")
    assert list(arch) == [256, 2, 4, 64, 512]
    (count,) = take("<i")
    assert count == 4
    seen = {}
    for _ in range(count):
        (ln,) = take("<i")
        name = raw[off:off + ln].decode()
        off += ln
        (kind,) = take("<B")
        (nd,) = take("<i")
        dims = take("<%di" % nd)
        (ns,) = take("<i")
        sc = np.frombuffer(raw, np.float32, ns, off); off += 4 * ns
        zp = np.frombuffer(raw, np.float32, ns, off); off += 4 * ns
        gs, eb, mb, dlen = take("<4i")
        data = np.frombuffer(raw, np.uint8, dlen, off); off += dlen
        seen[name] = (kind, dims, sc, zp, gs, data)
    assert off == len(raw)
    kind, dims, sc, zp, gs, data = seen["layers.0.attention.wq.weight"]
    assert kind == 3 and dims == (64, 256) and gs == 128
    p, s, z = O.quantize_int4_asym_per_group(src["layers_0_attention_wq_weight"], 128)
    assert np.array_equal(data, p) and np.array_equal(_u32(sc), _u32(s)) and np.array_equal(_u32(zp), _u32(z))
