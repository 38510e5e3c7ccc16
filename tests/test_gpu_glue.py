"""Device-resident decode glue (RMSNorm, LayerNorm, residual add, SwiGLU gating, RoPE,
decode attention with the KV-cache append) through the C ABI against the CPU
oracle's restatements of nim_inference.nim.  Element-wise steps whose every
rounding the reference fixes (residual add, RoPE with the caller's tables, the
KV-cache append) are bit-exact; steps with reductions (row sums, dot
products, softmax sums) or exp are held to max|y - y_ref| / max|y_ref| <= 1e-4,
well inside the path's 1e-3 bar."""
import ctypes

import numpy as np
import pytest

import pyoracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-4   # sequential vs tree fp32 sums of up to 11008 terms differ by ~1e-5


def rel_err(y, ref):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


@pytest.fixture(scope="module")
def torch_dev(nimf_gpu):
    import torch
    return torch


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def p(t):
    return ctypes.c_void_p(t.data_ptr())


def test_rmsnorm_add_swiglu(nimf_gpu, torch_dev):
    torch = torch_dev
    L = nimf_gpu.lib()
    rng = np.random.default_rng(1)
    for rows, cols in ((1, 4096), (3, 1000), (2, 4097), (8, 11008)):
        x = rng.standard_normal((rows, cols)).astype(np.float32)
        w = rng.uniform(0.5, 1.5, cols).astype(np.float32)
        y = torch.empty(rows, cols, device="cuda")
        dx, dw = dev(torch, x), dev(torch, w)   # held until the kernel has run
        nimf_gpu.check(L.nimf_rmsnorm_dev(p(dx), p(dw), rows, cols, 1e-6, p(y), None))
        torch.cuda.synchronize()
        assert rel_err(y.cpu().numpy(), O.rmsnorm(x, w, 1e-6)) <= TOL
    # residual add fused with the next RMSNorm: h bit-exact, y as rmsnorm(h);
    # rows of up to 4096 values stay in registers, longer rows are re-read
    for rows, cols in ((2, 4096), (1, 4097), (3, 11008)):
        a0 = rng.standard_normal((rows, cols)).astype(np.float32)
        r0 = rng.standard_normal((rows, cols)).astype(np.float32)
        w0 = rng.uniform(0.5, 1.5, cols).astype(np.float32)
        da0, dr0, dw0 = dev(torch, a0), dev(torch, r0), dev(torch, w0)
        hh = torch.empty(rows, cols, device="cuda")
        yy = torch.empty(rows, cols, device="cuda")
        nimf_gpu.check(L.nimf_add_rmsnorm_dev(p(da0), p(dr0), p(dw0), rows, cols, 1e-6, p(hh), p(yy), None))
        torch.cuda.synchronize()
        assert np.array_equal(hh.cpu().numpy().view(np.uint32), (a0 + r0).view(np.uint32))
        assert rel_err(yy.cpu().numpy(), O.rmsnorm(a0 + r0, w0, 1e-6)) <= TOL
    a = rng.standard_normal(10007).astype(np.float32)
    b = rng.standard_normal(10007).astype(np.float32)
    out = torch.empty(10007, device="cuda")
    da, db = dev(torch, a), dev(torch, b)
    nimf_gpu.check(L.nimf_add_dev(p(da), p(db), a.size, p(out), None))
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), (a + b).view(np.uint32))
    g = (rng.standard_normal(11008) * 3).astype(np.float32)
    u = rng.standard_normal(11008).astype(np.float32)
    gated = torch.empty(g.size, device="cuda")
    dg, du = dev(torch, g), dev(torch, u)
    nimf_gpu.check(L.nimf_swiglu_dev(p(dg), p(du), g.size, p(gated), None))
    torch.cuda.synchronize()
    assert rel_err(gated.cpu().numpy(), O.swiglu(g, u)) <= TOL


def test_layernorm(nimf_gpu, torch_dev):
    """nimf_layernorm_dev against the oracle's cpuLayernorm restatement, rows
    with a large mean (two-pass variance), both the register and the re-read
    path, and in place (y aliasing x)."""
    torch = torch_dev
    L = nimf_gpu.lib()
    rng = np.random.default_rng(4)
    for rows, cols in ((1, 4096), (3, 1000), (2, 4097), (8, 11008)):
        x = (rng.standard_normal((rows, cols)) * 2 + 40).astype(np.float32)
        g = rng.uniform(0.5, 1.5, cols).astype(np.float32)
        b = rng.standard_normal(cols).astype(np.float32)
        dx, dg, db = dev(torch, x), dev(torch, g), dev(torch, b)
        y = torch.empty(rows, cols, device="cuda")
        nimf_gpu.check(L.nimf_layernorm_dev(p(dx), p(dg), p(db), rows, cols, 1e-5, p(y), None))
        torch.cuda.synchronize()
        ref = O.layernorm(x, g, b, 1e-5)
        assert rel_err(y.cpu().numpy(), ref) <= TOL, (rows, cols)
        nimf_gpu.check(L.nimf_layernorm_dev(p(dx), p(dg), p(db), rows, cols, 1e-5, p(dx), None))
        torch.cuda.synchronize()
        assert np.array_equal(dx.cpu().numpy().view(np.uint32), y.cpu().numpy().view(np.uint32))
    with pytest.raises(nimf_gpu.CatchableError, match="ARG"):
        nimf_gpu.check(L.nimf_layernorm_dev(p(dx), None, p(db), 1, 16, 1e-5, p(y), None))


def rope_tables(D, max_seq, theta=10000.0):
    """newRoPEL (nim_inference.nim:246-259) in float32."""
    half = D // 2
    inv = (1.0 / np.power(np.float32(theta), np.arange(half, dtype=np.float32) / np.float32(half))).astype(np.float32)
    ang = (np.arange(max_seq, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def test_rope_bit_exact(nimf_gpu, torch_dev):
    torch = torch_dev
    L = nimf_gpu.lib()
    rng = np.random.default_rng(2)
    D, max_seq = 128, 640
    ct, st = rope_tables(D, max_seq)
    dct, dst = dev(torch, ct), dev(torch, st)
    for B, T, H, off in ((1, 1, 32, 517), (2, 3, 8, 5), (1, 16, 4, 0)):
        x = rng.standard_normal((B, T, H, D)).astype(np.float32)
        d = dev(torch, x)
        nimf_gpu.check(L.nimf_rope_dev(p(d), B, T, H, D, off, p(dct), p(dst), max_seq, None))
        torch.cuda.synchronize()
        ref = O.rope(x, B, T, H, D, off, ct, st)
        assert np.array_equal(d.cpu().numpy().ravel().view(np.uint32), ref.view(np.uint32))
    with pytest.raises(nimf_gpu.CatchableError, match="SHAPE"):
        nimf_gpu.check(L.nimf_rope_dev(p(d), 1, 2, 1, D, max_seq - 1, p(dct), p(dst), max_seq, None))


@pytest.mark.parametrize("H,HKV,pos", [(32, 32, 0), (32, 8, 1), (32, 8, 300), (8, 2, 639)])
def test_attention_decode(nimf_gpu, torch_dev, H, HKV, pos):
    torch = torch_dev
    L = nimf_gpu.lib()
    rng = np.random.default_rng(H + pos)
    D, max_seq = 128, 640
    kc = rng.standard_normal(HKV * max_seq * D).astype(np.float32)
    vc = rng.standard_normal(HKV * max_seq * D).astype(np.float32)
    q = rng.standard_normal(H * D).astype(np.float32)
    kn = rng.standard_normal(HKV * D).astype(np.float32)
    vn = rng.standard_normal(HKV * D).astype(np.float32)
    scale = np.float32(1.0 / np.sqrt(np.float32(D)))
    dkc, dvc = dev(torch, kc), dev(torch, vc)
    dq, dkn, dvn = dev(torch, q), dev(torch, kn), dev(torch, vn)
    out = torch.empty(H * D, device="cuda")
    nimf_gpu.check(L.nimf_attention_decode_dev(p(dq), p(dkn), p(dvn), p(dkc), p(dvc), H, HKV, D,
                                               max_seq, pos, float(scale), p(out), None))
    torch.cuda.synchronize()
    ref, rkc, rvc = O.attention_decode(q, kn, vn, kc, vc, H, HKV, D, max_seq, pos, float(scale))
    assert np.array_equal(dkc.cpu().numpy().view(np.uint32), rkc.view(np.uint32))
    assert np.array_equal(dvc.cpu().numpy().view(np.uint32), rvc.view(np.uint32))
    assert rel_err(out.cpu().numpy(), ref) <= TOL
    with pytest.raises(nimf_gpu.CatchableError, match="SHAPE"):
        nimf_gpu.check(L.nimf_attention_decode_dev(p(dq), p(dkn), p(dvn), p(dkc), p(dvc), H, HKV,
                                                   D, max_seq, max_seq, float(scale), p(out), None))


@pytest.mark.parametrize("T,H,HKV,D,pos0", [(37, 4, 2, 64, 0), (16, 8, 8, 128, 20), (1, 4, 1, 32, 9),
                                            (512, 32, 32, 128, 0), (40, 6, 3, 256, 100)])
def test_attention_prefill(nimf_gpu, torch_dev, T, H, HKV, D, pos0):
    """nimf_attention_prefill_dev: the appended cache rows bit-exact (earlier
    rows untouched) and the causal attention within 1e-4 of max|out| of the
    oracle's cpuAttentionFused restatement, including GQA, a later chunk
    (pos0 > 0), one token, head_dim 256 and the 7B prompt (512 x 32 x 128)."""
    torch = torch_dev
    L = nimf_gpu.lib()
    rng = np.random.default_rng(T * 7 + H)
    max_seq = pos0 + T + 3
    kc = rng.standard_normal(HKV * max_seq * D).astype(np.float32)
    vc = rng.standard_normal(HKV * max_seq * D).astype(np.float32)
    q = rng.standard_normal(T * H * D).astype(np.float32)
    kn = rng.standard_normal(T * HKV * D).astype(np.float32)
    vn = rng.standard_normal(T * HKV * D).astype(np.float32)
    scale = float(np.float32(1.0 / np.sqrt(np.float32(D))))
    dkc, dvc = dev(torch, kc), dev(torch, vc)
    dq, dkn, dvn = dev(torch, q), dev(torch, kn), dev(torch, vn)
    out = torch.empty(T * H * D, device="cuda")
    nimf_gpu.check(L.nimf_attention_prefill_dev(p(dq), p(dkn), p(dvn), p(dkc), p(dvc), T, H, HKV, D,
                                                max_seq, pos0, scale, p(out), None))
    torch.cuda.synchronize()
    ref, rkc, rvc = O.attention_prefill(q, kn, vn, kc, vc, T, H, HKV, D, max_seq, pos0, scale)
    assert np.array_equal(dkc.cpu().numpy().view(np.uint32), rkc.view(np.uint32))
    assert np.array_equal(dvc.cpu().numpy().view(np.uint32), rvc.view(np.uint32))
    assert rel_err(out.cpu().numpy(), ref) <= TOL
    with pytest.raises(nimf_gpu.CatchableError, match="SHAPE"):
        nimf_gpu.check(L.nimf_attention_prefill_dev(p(dq), p(dkn), p(dvn), p(dkc), p(dvc), T, H, HKV,
                                                    D, max_seq, max_seq - T + 1, scale, p(out), None))


def test_attention_decode_batch_device_positions(nimf_gpu, torch_dev):
    """nimf_attention_decode_batch_dev: three sequences at different positions
    read on the device, RoPE applied in place to q and k_new (bit-exact with
    the oracle's applyRoPEInplace), each sequence's cache row appended
    bit-exactly and its attention within 1e-4 of the oracle's forwardDecode
    core; advance_pos moves every position by one; a position past max_seq
    appends nothing and is reported by nimf_sync."""
    torch = torch_dev
    L = nimf_gpu.lib()
    rng = np.random.default_rng(17)
    B, H, HKV, D, MS = 3, 8, 4, 128, 64
    pos = np.array([5, 17, 0], np.int32)
    kc = rng.standard_normal((B, HKV * MS * D)).astype(np.float32)
    vc = rng.standard_normal((B, HKV * MS * D)).astype(np.float32)
    q = rng.standard_normal((B, H * D)).astype(np.float32)
    kn = rng.standard_normal((B, HKV * D)).astype(np.float32)
    vn = rng.standard_normal((B, HKV * D)).astype(np.float32)
    half = D // 2
    inv = 1.0 / np.power(np.float32(10000.0), np.arange(half, dtype=np.float32) / np.float32(half))
    ang = np.arange(MS, dtype=np.float32)[:, None] * inv[None, :].astype(np.float32)
    cos_t, sin_t = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    scale = float(np.float32(1.0 / np.sqrt(np.float32(D))))
    dq, dkn, dvn = dev(torch, q), dev(torch, kn), dev(torch, vn)
    dkc, dvc = dev(torch, kc), dev(torch, vc)
    dcos, dsin = dev(torch, cos_t), dev(torch, sin_t)
    dpos = torch.from_numpy(pos).cuda()
    out = torch.empty(B, H * D, device="cuda")
    nimf_gpu.check(L.nimf_attention_decode_batch_dev(p(dq), p(dkn), p(dvn), p(dkc), p(dvc), B, H, HKV,
                                                     D, MS, p(dpos), p(dcos), p(dsin), scale, 1,
                                                     p(out), None))
    torch.cuda.synchronize()
    nimf_gpu.check(L.nimf_sync())
    assert dpos.cpu().numpy().tolist() == (pos + 1).tolist()
    for b in range(B):
        qr = O.rope(q[b], 1, 1, H, D, int(pos[b]), cos_t, sin_t)
        kr = O.rope(kn[b], 1, 1, HKV, D, int(pos[b]), cos_t, sin_t)
        assert np.array_equal(dq[b].cpu().numpy().view(np.uint32), qr.view(np.uint32))
        assert np.array_equal(dkn[b].cpu().numpy().view(np.uint32), kr.view(np.uint32))
        ref, rkc, rvc = O.attention_decode(qr, kr, vn[b], kc[b], vc[b], H, HKV, D, MS, int(pos[b]),
                                           scale)
        assert np.array_equal(dkc[b].cpu().numpy().view(np.uint32), rkc.view(np.uint32))
        assert np.array_equal(dvc[b].cpu().numpy().view(np.uint32), rvc.view(np.uint32))
        assert rel_err(out[b].cpu().numpy(), ref) <= TOL
    # a position outside the cache: nothing appended, reported as an expired-wait class error
    bad = torch.tensor([MS, 3, 4], dtype=torch.int32, device="cuda")
    before = dkc[0].clone()
    nimf_gpu.check(L.nimf_attention_decode_batch_dev(p(dq), p(dkn), p(dvn), p(dkc), p(dvc), B, H, HKV,
                                                     D, MS, p(bad), None, None, scale, 0, p(out), None))
    torch.cuda.synchronize()
    assert L.nimf_sync() == -5
    assert torch.equal(before, dkc[0])


def test_embedding_and_greedy(nimf_gpu, torch_dev):
    """nimf_embedding_lookup_dev (zeros for ids out of range) bit-exact, and
    nimf_greedy_sample_dev giving the oracle's token ids: the penalised
    winner, a twice-listed id, ties, all-negative rows, NaNs, and 8 rows of
    the 7B vocabulary with 64 recent ids each."""
    from test_glue_oracle import greedy_cases
    torch = torch_dev
    L = nimf_gpu.lib()
    rng = np.random.default_rng(6)
    for vocab, dim in ((1000, 4096), (37, 4098)):
        table = rng.standard_normal((vocab, dim)).astype(np.float32)
        ids = np.array([5, -2, vocab - 1, vocab, 0, 5], np.int32)
        dt = dev(torch, table)
        di = torch.from_numpy(ids).cuda()
        out = torch.empty(ids.size, dim, device="cuda")
        nimf_gpu.check(L.nimf_embedding_lookup_dev(p(dt), vocab, dim, p(di), ids.size, p(out), None))
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy().view(np.uint32),
                              O.embedding_lookup(table, ids).view(np.uint32))
    big = rng.standard_normal((8, 32000)).astype(np.float32)
    brec = rng.integers(0, 32000, size=(8, 64)).astype(np.int32)
    brec[:, 0] = np.argmax(big, axis=1)
    cases = list(greedy_cases()) + [(big, brec, 1.3), (big, brec, 1.0)]
    for lg, rec, pen in cases:
        rows, vocab = lg.shape
        dl = dev(torch, lg)
        dr = torch.from_numpy(np.ascontiguousarray(rec, np.int32).reshape(-1).copy()
                              if rec.size else np.zeros(1, np.int32)).cuda()
        ids = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
        nimf_gpu.check(L.nimf_greedy_sample_dev(p(dl), rows, vocab, p(dr), rec.shape[1], pen, p(ids), None))
        torch.cuda.synchronize()
        assert np.array_equal(ids.cpu().numpy(), O.greedy_sample(lg, rec, pen)), (lg.shape, pen)
        assert np.array_equal(dl.cpu().numpy().view(np.uint32), lg.view(np.uint32))  # logits untouched
    with pytest.raises(nimf_gpu.CatchableError, match="SHAPE"):
        nimf_gpu.check(L.nimf_greedy_sample_dev(p(dl), 1, 300000, p(dr), 1, 1.3, p(ids), None))
