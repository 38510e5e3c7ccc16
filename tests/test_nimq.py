""".nimq (NIMQ2) state dicts: the library's reader (quant.nim:386-448) against
the stream the reference's own exporter wrote (tests/golden/nimq_small.bin,
export_to_nimq.py:580-605), and registration of every tensor kind as a
device weight, dequantised bit-exactly as quant.nim's
dequantizeTensorTransposed (quant.nim:256-345) and customfloat.nim decode."""
import ctypes
import os
import struct

import numpy as np
import pytest

import pyoracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden():
    return open(os.path.join(GOLD, "nimq_small.bin"), "rb").read()


def py_records(raw):
    """Independent struct walk of a NIMQ2 stream (the writer's field order)."""
    off = 0

    def take(fmt):
        nonlocal off
        v = struct.unpack_from(fmt, raw, off)
        off += struct.calcsize(fmt)
        return v

    (n,) = take("<i")
    off += n
    arch = list(take("<5i"))
    (count,) = take("<i")
    recs = []
    for _ in range(count):
        (ln,) = take("<i")
        name = raw[off:off + ln].decode()
        off += ln
        (kind,) = take("<B")
        (nd,) = take("<i")
        dims = list(take("<%di" % nd))
        (ns,) = take("<i")
        sc = np.frombuffer(raw, np.float32, ns, off).copy()
        off += 4 * ns
        zp = np.frombuffer(raw, np.float32, ns, off).copy()
        off += 4 * ns
        gs, eb, mb, dlen = take("<4i")
        data = np.frombuffer(raw, np.uint8, dlen, off).copy()
        off += dlen
        recs.append((name, kind, dims, sc, zp, gs, eb, mb, data))
    return arch, recs


def write_stream(arch, tensors):
    """NIMQ2 bytes in the writer's field order (quant.nim:365-398)."""
    out = bytearray()

    def string(s):
        b = s.encode()
        out.extend(struct.pack("<i", len(b)) + b)

    string("NIMQ2")
    out.extend(struct.pack("<5i", *arch))
    out.extend(struct.pack("<i", len(tensors)))
    for name, kind, dims, sc, zp, gs, eb, mb, data in tensors:
        string(name)
        out.extend(struct.pack("<B", kind) + struct.pack("<i", len(dims)))
        out.extend(struct.pack("<%di" % len(dims), *dims))
        sc = np.asarray(sc, np.float32)
        out.extend(struct.pack("<i", sc.size) + sc.tobytes() + np.asarray(zp, np.float32).tobytes())
        data = np.asarray(data, np.uint8)
        out.extend(struct.pack("<4i", gs, eb, mb, data.size) + data.tobytes())
    return bytes(out)


def test_parse_golden_stream(nimf_mod):
    raw = golden()
    arch, recs = py_records(raw)
    a2, tensors, _ = nimf_mod.loadQuantStateDict(raw)
    assert a2 == arch == [256, 2, 4, 64, 512]
    assert [t[0] for t in tensors] == [r[0] for r in recs]
    for (name, info), (_, kind, dims, sc, zp, gs, eb, mb, data) in zip(tensors, recs):
        assert info["kind"] == kind and info["shape"] == dims and info["group_size"] == gs
        assert (info["exponentBits"], info["mantissaBits"]) == (eb, mb)
        assert np.array_equal(info["scales"].view(np.uint32), sc.view(np.uint32))
        assert np.array_equal(info["zero_point"].view(np.uint32), zp.view(np.uint32))
        assert np.array_equal(info["data"], data)


def test_parse_rejects_bad_streams(nimf_mod):
    raw = golden()
    L = nimf_mod.lib()
    cnt = ctypes.c_int64()
    buf = np.frombuffer(raw, np.uint8)
    # every truncation is refused (NIMF_ERR_SHAPE -2, or NIMF_ERR_ARG -1 inside the magic)
    for cut in list(range(0, 64)) + list(range(64, len(raw), 97)) + [len(raw) - 1]:
        st = L.nimf_nimq_parse(nimf_mod._ptr(buf[:cut].copy()), cut, None, ctypes.byref(cnt))
        assert st in (-2, -1), cut
    bad = bytearray(raw)
    bad[4:9] = b"NIMQ1"
    with pytest.raises(nimf_mod.CatchableError, match="ARG"):
        nimf_mod.loadQuantStateDict(bytes(bad))
    assert L.nimf_nimq_parse(nimf_mod._ptr(buf), buf.size, None, ctypes.byref(cnt)) == 0
    assert cnt.value == 4


def synthetic_stream():
    """Every kind quant.nim stores, in the layouts its quantisers produce."""
    rng = np.random.default_rng(21)
    n, k = 40, 70   # odd rows, K not a multiple of 16 or of the group
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    t = []
    p, s, z = O.quantize_int4_asym_per_group(w, 32)
    t.append(("q4_group", 3, [n, k], s, z, 32, 1, 0, p))
    bpr = (k + 1) // 2
    codes = rng.integers(0, 256, size=n * bpr, dtype=np.uint8)
    t.append(("q4_row", 3, [n, k], rng.uniform(1e-3, 2e-3, n), rng.uniform(6, 9, n), 0, 1, 0, codes))
    t.append(("q4_tensor", 3, [n, k], [1.5e-3], [7.25], 0, 1, 0, codes))
    t.append(("q4_sym", 2, [n, k], [2e-3], [0.0], 0, 1, 0, codes))
    q, sc = O.quantize_int8(w)
    t.append(("i8", 1, [n, k], [sc], [0.0], 0, 1, 0, q.view(np.uint8)))
    t.append(("e4m3", 4, [n, k], [1.0], [0.0], 0, 4, 3, O.cf_encode(w * 100, 4, 3)))
    t.append(("e6m10", 6, [n, k], [1.0], [0.0], 0, 6, 10, O.cf_encode(w, 6, 10)))
    t.append(("raw", 0, [n, k], [1.0], [0.0], 0, 1, 0, w.view(np.uint8).ravel()))
    t.append(("norm", 0, [k], [1.0], [0.0], 0, 1, 0, np.ones(k, np.float32).view(np.uint8)))
    return write_stream([1, 2, 3, 4, 5], t), n, k, t


def reference_weight(kind, dims, sc, zp, gs, eb, mb, data):
    n, k = dims
    if kind in (1, 2, 3):
        return O.dequantize_transposed(kind, data, np.asarray(sc, np.float32),
                                       np.asarray(zp, np.float32), n, k, gs).T
    if kind == 0:
        return np.frombuffer(np.asarray(data, np.uint8).tobytes(), np.float32).reshape(n, k)
    return O.cf_decode(data, eb, mb).reshape(n, k)


@pytest.mark.gpu
def test_register_every_kind(nimf_gpu):
    raw, n, k, tensors = synthetic_stream()
    _, infos, sd = nimf_gpu.loadQuantStateDict(raw)
    x = np.random.default_rng(5).standard_normal((3, k)).astype(np.float32)
    for i, rec in enumerate(tensors):
        name, kind, dims = rec[0], rec[1], rec[2]
        if len(dims) != 2:
            with pytest.raises(nimf_gpu.CatchableError, match="SHAPE"):
                sd.register(i)
            continue
        ref = np.ascontiguousarray(reference_weight(kind, *rec[2:]), np.float32)
        h = sd.register(i)
        assert np.array_equal(h.dequant().view(np.uint32), ref.view(np.uint32)), name
        y = h.matmul(x, 3)
        yr = O.gemv_f64(x, ref)
        assert np.max(np.abs(y - yr)) <= 1e-3 * max(np.max(np.abs(yr)), 1e-30), name
        h.free()
        if kind != 0:
            # an N-shard of the same record
            hs = sd.register(i, rows=(16, 32))
            assert np.array_equal(hs.dequant().view(np.uint32), ref[16:32].view(np.uint32)), name
            hs.free()


@pytest.mark.gpu
def test_register_golden_stream(nimf_gpu):
    raw = golden()
    _, recs = py_records(raw)
    _, infos, sd = nimf_gpu.loadQuantStateDict(raw)
    i = sd.index("layers.0.attention.wq.weight")
    name, kind, dims, sc, zp, gs, eb, mb, data = recs[i]
    h = sd.register(i)
    ref = O.dequantize_int4_asym(data, sc, zp, dims[0], dims[1], gs)
    assert np.array_equal(h.dequant().view(np.uint32), ref.view(np.uint32))
    h.free()
    i = sd.index("layers.0.feed_forward.w1.weight")
    h = sd.register(i)
    _, kind, dims, sc, zp, gs, eb, mb, data = recs[i]
    assert np.array_equal(h.dequant().view(np.uint32),
                          O.dequantize_int8(data.view(np.int8), sc[0]).reshape(dims).view(np.uint32))
    h.free()
