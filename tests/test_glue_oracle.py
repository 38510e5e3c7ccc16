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


def greedy_loop(logits, recent, penalty):
    """sampleTopP with temperature <= 0 (nim_inference.nim:1019-1036), in float32."""
    f = np.float32
    out = []
    for r in range(logits.shape[0]):
        adj = logits[r].copy()
        if penalty != 1.0:
            for i in recent[r]:
                if 0 <= i < adj.size:
                    adj[i] = f(adj[i] / f(penalty)) if adj[i] > 0 else f(adj[i] * f(penalty))
        best = 0
        for i in range(1, adj.size):
            if adj[i] > adj[best]:
                best = i
        out.append(best)
    return np.array(out, np.int32)


def greedy_cases():
    rng = np.random.default_rng(3)
    lg = rng.standard_normal((4, 300)).astype(np.float32)
    rec = rng.integers(-3, 310, size=(4, 20)).astype(np.int32)
    top = np.argmax(lg, axis=1)
    rec[:, 0] = top          # the raw winner is penalised
    rec[:, 1] = top          # twice
    yield lg, rec, 1.3
    yield lg, rec, 1.0       # no penalty
    yield lg, rec[:, :0], 1.3
    ties = np.zeros((2, 50), np.float32)
    ties[:, [7, 30]] = 2.0   # first of equal maxima
    yield ties, np.array([[7], [30]], np.int32), 1.0
    yield ties, np.array([[7], [30]], np.int32), 1.3
    neg = -np.abs(lg[:2])    # all negative: the penalty multiplies
    yield neg, rec[:2], 1.3
    nan = lg[:2].copy()
    nan[0, 0] = np.nan       # a NaN at index 0 wins the strict scan
    nan[1, 5] = np.nan       # elsewhere it never wins
    yield nan, rec[:2], 1.3


def test_greedy_and_embedding_match_reference_loops():
    for lg, rec, pen in greedy_cases():
        assert np.array_equal(O.greedy_sample(lg, rec, pen), greedy_loop(lg, rec, pen))
    rng = np.random.default_rng(4)
    table = rng.standard_normal((10, 6)).astype(np.float32)
    ids = np.array([3, -1, 9, 10, 0], np.int32)
    out = O.embedding_lookup(table, ids)
    ref = np.stack([table[i] if 0 <= i < 10 else np.zeros(6, np.float32) for i in ids])
    assert np.array_equal(out, ref)


def test_prefill_attention_oracle_against_float64():
    """orc_attention_prefill (cpuAttentionFused, causal, with appendKV) within
    float32 rounding of a float64 evaluation, GQA and a chunk at pos0 > 0; the
    appended rows are the new K / V rows and earlier rows are untouched."""
    rng = np.random.default_rng(3)
    H, HKV, D, MS, T, pos0 = 6, 3, 64, 40, 11, 7
    kc = rng.standard_normal(HKV * MS * D).astype(np.float32)
    vc = rng.standard_normal(HKV * MS * D).astype(np.float32)
    q = rng.standard_normal(T * H * D).astype(np.float32)
    kn = rng.standard_normal(T * HKV * D).astype(np.float32)
    vn = rng.standard_normal(T * HKV * D).astype(np.float32)
    out, kc2, vc2 = O.attention_prefill(q, kn, vn, kc, vc, T, H, HKV, D, MS, pos0, 0.125)
    K, V = kc2.reshape(HKV, MS, D), vc2.reshape(HKV, MS, D)
    assert np.array_equal(K[:, :pos0], kc.reshape(HKV, MS, D)[:, :pos0])
    assert np.array_equal(K[:, pos0:pos0 + T], kn.reshape(T, HKV, D).transpose(1, 0, 2))
    assert np.array_equal(V[:, pos0:pos0 + T], vn.reshape(T, HKV, D).transpose(1, 0, 2))
    Q = q.reshape(T, H, D).astype(np.float64)
    ref = np.zeros((T, H, D))
    for h in range(H):
        for t in range(T):
            S = pos0 + t + 1
            sc = (K[h // 2, :S].astype(np.float64) @ Q[t, h]) * 0.125
            pr = np.exp(sc - sc.max())
            pr /= pr.sum()
            ref[t, h] = pr @ V[h // 2, :S].astype(np.float64)
    assert np.max(np.abs(out.reshape(T, H, D) - ref)) <= 1e-5 * np.max(np.abs(ref))
