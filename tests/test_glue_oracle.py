"""The oracle's LayerNorm against a float32 loop written from cpuLayernorm
(vendor/bybylang/gpubackend.nim:252-266, the path LayerNorm.forward takes,
nimformer.nim:188-197): bit-exact on small rows, and within 1e-5 of a float64
evaluation on rows with a large mean (two-pass variance)."""
import numpy as np

import pyoracle as O


def layernorm_loop(x, gamma, beta, eps):
    f = np.float32
    rows, cols = x.shape
    y = np.empty_like(x)
    for r in range(rows):
        mean = f(0)
        for c in range(cols):
            mean = f(mean + x[r, c])
        mean = f(mean / f(cols))
        var = f(0)
        for c in range(cols):
            d = f(x[r, c] - mean)
            var = f(var + f(d * d))
        var = f(var / f(cols))
        inv = f(f(1) / np.sqrt(f(var + f(eps))))
        for c in range(cols):
            y[r, c] = f(f(f(f(x[r, c] - mean) * inv) * gamma[c]) + beta[c])
    return y


def test_layernorm_matches_reference_loop():
    rng = np.random.default_rng(0)
    for rows, cols in ((1, 1), (2, 7), (3, 96)):
        x = (rng.standard_normal((rows, cols)) * 3 + 1).astype(np.float32)
        g = rng.uniform(0.5, 1.5, cols).astype(np.float32)
        b = rng.standard_normal(cols).astype(np.float32)
        y = O.layernorm(x, g, b, 1e-5)
        assert np.array_equal(y.view(np.uint32), layernorm_loop(x, g, b, 1e-5).view(np.uint32))


def test_layernorm_two_pass_accuracy():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((4, 4096)) * 0.5 + 300.0).astype(np.float32)
    g = np.ones(4096, np.float32)
    b = np.zeros(4096, np.float32)
    y = O.layernorm(x, g, b, 1e-5)
    xd = x.astype(np.float64)
    m = xd.mean(1, keepdims=True)
    ref = (xd - m) / np.sqrt(((xd - m) ** 2).mean(1, keepdims=True) + 1e-5)
    assert np.max(np.abs(y - ref)) <= 1e-3 * np.max(np.abs(ref))
