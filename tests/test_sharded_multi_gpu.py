"""The library's own multi-GPU path on 2 GPUs, one process per GPU, NCCL
opened by the library (nimf_comm_*), NVLS off:

* nimf_matmul_w_allgather_dev: each rank registers its nimf_shard_range rows
  of an int4-g128 weight; the gathered y on every rank equals the full
  weight's GEMV on one GPU (within 1e-4 of max|y|: the launch planner may cut
  K differently for a shard, and the x digit scale is per k-split) -- m = 1 with equal shards (in place) and m = 3
  with unequal shards (gather buffer and layout pass);
* nimf_decode_create_sharded: a 2-layer Llama-shape int4 stack whose
  projections are N-sharded and whose heads are split between the ranks runs
  its whole decode step as one launch per GPU, exchanging every stage's
  outputs over peer memory.  Logit rows, greedy tokens and appended KV rows
  are bit-identical to the one-GPU plan over the full weights (the same
  arithmetic in the same order), over three chained steps;
* nimf_p2p_connect_comm: the peer-memory all-gather connected through the
  library's communicator instead of host-exchanged handles.

Skipped with fewer than 2 GPUs."""
import ctypes
import datetime
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))

D, H, HD, F, V, LAYERS, MAX_SEQ, POS = 1024, 8, 128, 2816, 4000, 2, 64, 40


def _setup(rank, world, port):
    import torch
    import torch.distributed as dist
    sys.path.insert(0, os.path.join(HERE, "..", "nimformers-framework_b200"))
    import nimf
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120))
    nimf.init(rank)
    L = nimf.lib()
    uid = ctypes.create_string_buffer(128)
    if rank == 0:
        nimf.check(L.nimf_comm_unique_id(uid))
    box = [uid.raw]
    dist.broadcast_object_list(box, src=0)
    nimf.check(L.nimf_comm_init(world, rank, ctypes.create_string_buffer(box[0], 128)))
    w, r = ctypes.c_int(), ctypes.c_int()
    nimf.check(L.nimf_comm_info(ctypes.byref(w), ctypes.byref(r)))
    assert (w.value, r.value) == (world, rank)
    return torch, dist, nimf, L


def _teardown(dist, L):
    import nimf
    nimf.check(L.nimf_comm_barrier())
    nimf.check(L.nimf_comm_destroy())
    dist.barrier()
    dist.destroy_process_group()


def _quant(rng, n, k):
    import nimf
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    return nimf.quantize_int4_per_group(w, 128)


def _allgather_worker(rank, world, port, q):
    try:
        torch, dist, nimf, L = _setup(rank, world, port)
        rng = np.random.default_rng(11)
        for n, k, m in [(4096, 1024, 1), (1000, 512, 3), (12288, 4096, 1)]:
            p, s, z = _quant(rng, n, k)
            x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()
            full = nimf.Weight.q4g(p, s, z, n, k, 128)
            shard = nimf.Weight.q4g(p, s, z, n, k, 128, rows=nimf.shard_rows(n, world, rank))
            y_full = torch.empty(m, n, device="cuda")
            y = torch.full((m, n), -7.0, device="cuda")
            full.matmul_dev(x.data_ptr(), m, y_full.data_ptr(), None)
            for _ in range(2):
                nimf.check(L.nimf_matmul_w_allgather_dev(shard.handle, ctypes.c_void_p(x.data_ptr()), m,
                                                         ctypes.c_void_p(y.data_ptr()), None))
            nimf.check(L.nimf_sync())
            a, b = y.cpu().numpy(), y_full.cpu().numpy()
            # a shard may pick another k-split than the full weight, and the
            # x digit scale is per k-split: agreement to ~1e-5 of max|y|
            err = float(np.max(np.abs(a - b)) / np.max(np.abs(b)))
            assert err <= 1e-4, (n, k, m, err)
            full.free()
            shard.free()
        # a weight that is not this rank's shard is refused
        p, s, z = _quant(rng, 256, 256)
        wrong = nimf.Weight.q4g(p, s, z, 256, 256, 128)
        x = torch.zeros(1, 256, device="cuda")
        y = torch.zeros(1, 256, device="cuda")
        rc = L.nimf_matmul_w_allgather_dev(wrong.handle, ctypes.c_void_p(x.data_ptr()), 1,
                                           ctypes.c_void_p(y.data_ptr()), None)
        assert rc == -2, rc
        wrong.free()
        _teardown(dist, L)
        q.put((rank, "ok"))
    except BaseException as e:  # noqa: BLE001
        q.put((rank, "%s: %s" % (type(e).__name__, e)))


def _model(rng):
    shapes = {"wq": (D, D), "wk": (D, D), "wv": (D, D), "wo": (D, D), "wgate": (F, D),
              "wup": (F, D), "wdown": (D, F)}
    layers = []
    for _ in range(LAYERS):
        layers.append({nm: _quant(rng, *nk) for nm, nk in shapes.items()})
    head = _quant(rng, V, D)
    norms = [(rng.random(D) + 0.5).astype(np.float32) for _ in range(2 * LAYERS + 1)]
    table = (rng.standard_normal((V, D)) * 0.5).astype(np.float32)
    kc = [(rng.standard_normal((H, MAX_SEQ, HD)) * 0.5).astype(np.float32) for _ in range(LAYERS)]
    vc = [(rng.standard_normal((H, MAX_SEQ, HD)) * 0.5).astype(np.float32) for _ in range(LAYERS)]
    half = HD // 2
    inv = 1.0 / np.power(np.float32(10000.0), np.arange(half, dtype=np.float32) / np.float32(half))
    ang = np.arange(MAX_SEQ, dtype=np.float32)[:, None] * inv[None, :].astype(np.float32)
    recent = rng.integers(0, V, size=32).astype(np.int32)
    return dict(shapes=shapes, layers=layers, head=head, norms=norms, table=table, kc=kc, vc=vc,
                cos=np.cos(ang).astype(np.float32), sin=np.sin(ang).astype(np.float32),
                recent=recent)


def _run_plan(torch, nimf, M, world, rank, sharded, steps=3):
    """Runs `steps` chained steps (token out -> token in, position advanced);
    returns per step (logits, token) and the final caches."""
    dev = torch.device("cuda")
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    hk = slice(rank * H // world, (rank + 1) * H // world) if sharded else slice(0, H)
    ws, keep, layers = [], [], []
    plan = None
    try:
        for li, lw in enumerate(M["layers"]):
            d = {}
            for nm, (p, s, z) in lw.items():
                n, k = M["shapes"][nm]
                rows = nimf.shard_rows(n, world, rank) if sharded else None
                d[nm] = nimf.Weight.q4g(p, s, z, n, k, 128, rows=rows)
                ws.append(d[nm])
            an, fn = T(M["norms"][2 * li]), T(M["norms"][2 * li + 1])
            kc, vc = T(M["kc"][li][hk]), T(M["vc"][li][hk])
            keep += [an, fn, kc, vc]
            d.update(attn_norm=an.data_ptr(), ffn_norm=fn.data_ptr(), k_cache=kc.data_ptr(),
                     v_cache=vc.data_ptr())
            layers.append(d)
        p, s, z = M["head"]
        head = nimf.Weight.q4g(p, s, z, V, D, 128,
                               rows=nimf.shard_rows(V, world, rank) if sharded else None)
        ws.append(head)
        table, fin = T(M["table"]), T(M["norms"][-1])
        cos_t, sin_t = T(M["cos"]), T(M["sin"])
        keep += [table, fin, cos_t, sin_t]
        plan = nimf.DecodePlan(layers=layers, embedding=table.data_ptr(), final_norm=fin.data_ptr(),
                               lm_head=head, rope_cos=cos_t.data_ptr(), rope_sin=sin_t.data_ptr(),
                               d_model=D, n_heads=H, n_kv_heads=H, head_dim=HD, ffn_dim=F, vocab=V,
                               max_seq=MAX_SEQ, norm_eps=1e-6, sharded=sharded)
        recent = T(M["recent"])
        tok = torch.tensor([123], dtype=torch.int32, device=dev)
        pos = torch.tensor([POS], dtype=torch.int32, device=dev)
        logits = torch.zeros(V, device=dev)
        out = []
        for _ in range(steps):
            logits.zero_()
            plan.step(tok.data_ptr(), tok.data_ptr(), pos.data_ptr(), logits.data_ptr(),
                      recent.data_ptr(), 32, 1.3, advance_pos=True)
            torch.cuda.synchronize()
            nimf.check(nimf.lib().nimf_sync())
            out.append((logits.cpu().numpy().copy(), int(tok.item())))
        assert int(pos.item()) == POS + steps
        caches = [(keep[4 * li + 2].cpu().numpy(), keep[4 * li + 3].cpu().numpy())
                  for li in range(LAYERS)]
        return out, caches
    finally:
        if plan is not None:
            plan.destroy()
        for w in ws:
            w.free()


def _decode_worker(rank, world, port, q):
    try:
        torch, dist, nimf, L = _setup(rank, world, port)
        M = _model(np.random.default_rng(21))
        one, one_caches = _run_plan(torch, nimf, M, 1, 0, sharded=False)
        dist.barrier()
        shd, shd_caches = _run_plan(torch, nimf, M, world, rank, sharded=True)
        r0, r1 = nimf.shard_rows(V, world, rank)
        hk = slice(rank * H // world, (rank + 1) * H // world)
        for (l1, t1), (l2, t2) in zip(one, shd):
            assert t1 == t2, (t1, t2)
            assert np.array_equal(l1[r0:r1].view(np.uint32), l2[r0:r1].view(np.uint32))
        for (k1, v1), (k2, v2) in zip(one_caches, shd_caches):
            assert np.array_equal(k1[hk].view(np.uint32), k2.view(np.uint32))
            assert np.array_equal(v1[hk].view(np.uint32), v2.view(np.uint32))
        toks = [None] * world
        dist.all_gather_object(toks, [t for _, t in shd])
        assert toks[0] == toks[1]
        _teardown(dist, L)
        q.put((rank, "ok"))
    except BaseException as e:  # noqa: BLE001
        q.put((rank, "%s: %s" % (type(e).__name__, e)))


def _p2p_comm_worker(rank, world, port, q):
    try:
        torch, dist, nimf, L = _setup(rank, world, port)
        h = ctypes.create_string_buffer(64)
        gid = ctypes.c_int64()
        nimf.check(L.nimf_p2p_create(world, rank, 4096, h, ctypes.byref(gid)))
        nimf.check(L.nimf_p2p_connect_comm(gid.value))
        cols = 300
        src = torch.full((2, cols), float(rank + 1), device="cuda")
        dst = torch.full((2, world * cols), -1.0, device="cuda")
        nimf.check(L.nimf_p2p_allgather_dev(gid.value, ctypes.c_void_p(src.data_ptr()), 2, cols, cols,
                                            ctypes.c_void_p(dst.data_ptr()), world * cols, None))
        nimf.check(L.nimf_sync())
        want = np.concatenate([np.full((2, cols), float(r + 1), np.float32) for r in range(world)], 1)
        assert np.array_equal(dst.cpu().numpy(), want)
        nimf.check(L.nimf_comm_barrier())
        nimf.check(L.nimf_p2p_destroy(gid.value))
        _teardown(dist, L)
        q.put((rank, "ok"))
    except BaseException as e:  # noqa: BLE001
        q.put((rank, "%s: %s" % (type(e).__name__, e)))


def _gather_worker(rank, world, port, q):
    """The all-gather fused into the grouped GEMV: three weights (q/k/v-like,
    one of them with unequal shards) at M = 1, 3 and 8, each call repeated;
    the gathered outputs on every rank equal the full weights' GEMV on one GPU
    (within 1e-4 of max|y|: the x digit scale follows the k-split).  Then rank 1 skips one call: rank 0's arrival
    wait runs out after the bound and nimf_sync reports NIMF_ERR_TIMEOUT."""
    try:
        torch, dist, nimf, L = _setup(rank, world, port)
        rng = np.random.default_rng(12)
        K = 2048
        ns = [4096, 1000, 2048]
        quants = [_quant(rng, n, K) for n in ns]
        full = [nimf.Weight.q4g(p, s, z, n, K, 128) for (p, s, z), n in zip(quants, ns)]
        shard = [nimf.Weight.q4g(p, s, z, n, K, 128, rows=nimf.shard_rows(n, world, rank))
                 for (p, s, z), n in zip(quants, ns)]
        total = sum(ns) * 8 * 4
        gid, base = ctypes.c_int64(), ctypes.c_void_p()
        nimf.check(L.nimf_gather_create(total, ctypes.byref(gid), ctypes.byref(base)))
        hs = (ctypes.c_uint64 * 3)(*[w.handle for w in shard])
        for m in (1, 3, 8):
            x = torch.from_numpy(rng.standard_normal((m, K)).astype(np.float32)).cuda()
            offs = np.cumsum([0] + [m * n * 4 for n in ns])
            yp = (ctypes.c_void_p * 3)(*[base.value + int(o) for o in offs[:3]])
            want = []
            for w, n in zip(full, ns):
                y = torch.empty(m, n, device="cuda")
                w.matmul_dev(x.data_ptr(), m, y.data_ptr(), None)
                want.append(y)
            # the library stream does not order with torch's: wait for it
            nimf.check(L.nimf_sync())
            want = [y.cpu().numpy() for y in want]
            for _ in range(3):
                nimf.check(L.nimf_matmul_w_group_gather_dev(gid.value, hs, 3,
                                                            ctypes.c_void_p(x.data_ptr()), m, yp, None))
            nimf.check(L.nimf_sync())
            # read the gathered outputs back through a device copy
            got = torch.empty(int(offs[3]) // 4, device="cuda")
            import cuda.bindings.runtime as crt   # cuda-python
            err, = crt.cudaMemcpy(got.data_ptr(), base.value, int(offs[3]),
                                  crt.cudaMemcpyKind.cudaMemcpyDeviceToDevice)
            assert int(err) == 0, err
            flat = got.cpu().numpy()
            for i, n in enumerate(ns):
                a = flat[offs[i] // 4: offs[i + 1] // 4].reshape(m, n)
                e = float(np.max(np.abs(a - want[i])) / np.max(np.abs(want[i])))
                assert e <= 1e-4, (m, n, e)   # k-split dependent x digit scale
            dist.barrier()
        # a rank that leaves between calls: the other's bounded wait expires
        nimf.check(L.nimf_gather_set_timeout_ms(300))
        x = torch.zeros(1, K, device="cuda")
        yp = (ctypes.c_void_p * 3)(*[base.value + i * 4 * 4096 for i in range(3)])
        dist.barrier()
        if rank == 0:
            nimf.check(L.nimf_matmul_w_group_gather_dev(gid.value, hs, 3, ctypes.c_void_p(x.data_ptr()),
                                                        1, yp, None))
            rc = L.nimf_sync()
            assert rc == -5, (rc, L.nimf_last_error())
        dist.barrier()
        nimf.check(L.nimf_gather_set_timeout_ms(2000))
        nimf.check(L.nimf_gather_destroy(gid.value))
        for w in full + shard:
            w.free()
        _teardown(dist, L)
        q.put((rank, "ok"))
    except BaseException as e:  # noqa: BLE001
        q.put((rank, "%s: %s" % (type(e).__name__, e)))


def _run(target, salt):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29000 + (os.getpid() * 7 + salt) % 500
    env = dict(os.environ)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        ps = [ctx.Process(target=target, args=(r, 2, port, q)) for r in range(2)]
        for p in ps:
            p.start()
    finally:
        os.environ.clear()
        os.environ.update(env)
    import queue
    res = {}
    try:
        while len(res) < len(ps):
            # a rank that failed may leave the other waiting in a collective:
            # after the first failure give the rest 30 s, then end them
            failed = any(v != "ok" for v in res.values())
            try:
                r, v = q.get(timeout=30 if failed else 600)
            except queue.Empty:
                break
            res[r] = v
    finally:
        for p in ps:
            p.join(timeout=30)
        for p in ps:
            if p.is_alive():
                p.kill()
                p.join(timeout=30)
    return res


def test_sharded_matmul_allgather_two_gpus():
    assert _run(_allgather_worker, 1) == {0: "ok", 1: "ok"}


def test_sharded_decode_step_bit_identical_to_one_gpu():
    assert _run(_decode_worker, 2) == {0: "ok", 1: "ok"}


def test_gemv_with_fused_allgather_two_gpus():
    assert _run(_gather_worker, 4) == {0: "ok", 1: "ok"}


def test_p2p_connect_through_library_communicator():
    assert _run(_p2p_comm_worker, 3) == {0: "ok", 1: "ok"}
