"""GPTQ-native int4 tensors (qweight / qzeros / fp16 scales / g_idx) registered
without an fp32 round-trip, against the reference's own dequantize_gptq_linear
(export_to_nimq.py:219-254) run on seeded inputs (tests/golden/gptq_*.npz,
written by tests/golden/gen_golden.py).  Dequantisation is bit-exact, with
contiguous groups and with act-order g_idx; matmuls meet
max|y - y_ref| / max|y_ref| <= 1e-3 on the decode GEMV and the tcgen05 GEMM."""
import os

import numpy as np
import pytest

import pyoracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOL = 1e-3


def rel_err(y, ref):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def load(name):
    d = np.load(os.path.join(GOLD, name + ".npz"))
    return d["qweight"], d["qzeros"], d["scales"], d["g_idx"], d["weight"]


def test_oracle_matches_reference_fixtures():
    for name in ("gptq_basic", "gptq_actorder"):
        qw, qz, sc, gi, ref = load(name)
        w = O.dequantize_gptq_linear(qw, qz, sc, gi)
        assert np.array_equal(np.asarray(w).reshape(ref.shape).view(np.uint32), ref.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["gptq_basic", "gptq_actorder"])
def test_register_gptq_bit_exact_and_matmul(nimf_gpu, name):
    qw, qz, sc, gi, ref = load(name)
    n, k = ref.shape
    h = nimf_gpu.Weight.gptq(qw, qz, sc, gi)
    assert (h.rows, h.k) == (n, k)
    assert np.array_equal(h.dequant().view(np.uint32), ref.view(np.uint32))
    rng = np.random.default_rng(3)
    for m in (1, 3, 8, 40):
        x = rng.standard_normal((m, k)).astype(np.float32)
        assert rel_err(h.matmul(x, m), O.gemv_f64(x, ref)) <= TOL, (name, m)
    # an N-shard and a grouped call with an ordinary int4 weight of the same K
    hs = nimf_gpu.Weight.gptq(qw, qz, sc, gi, rows=(8, n))
    assert np.array_equal(hs.dequant().view(np.uint32), ref[8:].view(np.uint32))
    x = rng.standard_normal((2, k)).astype(np.float32)
    ys = nimf_gpu.Weight.matmul_group([h, hs], x, 2)
    assert rel_err(ys[0], O.gemv_f64(x, ref)) <= TOL
    assert rel_err(ys[1], O.gemv_f64(x, ref[8:])) <= TOL
    hs.free()
    h.free()


@pytest.mark.gpu
def test_gptq_rejects_bad_inputs(nimf_gpu):
    qw, qz, sc, gi, _ = load("gptq_basic")
    bad = gi.copy()
    bad[3] = 99
    with pytest.raises(nimf_gpu.CatchableError, match="SHAPE"):
        nimf_gpu.Weight.gptq(qw, qz, sc, bad)
    uneven = np.ones_like(gi)
    uneven[:100] = 0   # group 0 holds 100 features, the last group 156
    with pytest.raises(nimf_gpu.CatchableError, match="UNSUPPORTED"):
        nimf_gpu.Weight.gptq(qw, qz, sc, uneven)
    # 130 + 126 is a valid split (groups of 130, the last one shorter)
    ok = np.ones_like(gi)
    ok[:130] = 0
    h = nimf_gpu.Weight.gptq(qw, qz, sc, ok)
    assert np.array_equal(h.dequant().view(np.uint32),
                          O.dequantize_gptq_linear(qw, qz, sc, ok).view(np.uint32))
    h.free()
