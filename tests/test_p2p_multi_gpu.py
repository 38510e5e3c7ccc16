"""The peer-memory all-gather (nimf_p2p_*) on 2 GPUs, one process per GPU:
every rank's slice lands bit-exactly in every rank's dst, over several calls
(both buffer parities, reused), with a source row stride wider than the slice
and an empty call; and when one rank leaves between steps (skips a call), the
other's bounded wait expires, nimf_sync reports NIMF_ERR_TIMEOUT, dst keeps
its old contents, and a call queued behind the expired one gives up at once.
No multicast object is involved (plain peer stores; NVLS is off).  Skipped
with fewer than 2 GPUs."""
import ctypes
import datetime
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _worker(rank, world, port, q):
    try:
        import torch
        import torch.distributed as dist
        sys.path.insert(0, os.path.join(HERE, "..", "nimformers-framework_b200"))
        import nimf
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60))
        nimf.init(rank)
        L = nimf.lib()
        h = ctypes.create_string_buffer(64)
        gid = ctypes.c_int64()
        nimf.check(L.nimf_p2p_create(world, rank, 4096, h, ctypes.byref(gid)))
        hs = [None] * world
        dist.all_gather_object(hs, h.raw)
        nimf.check(L.nimf_p2p_connect(gid.value, ctypes.create_string_buffer(b"".join(hs), 64 * world)))
        dist.barrier()
        for call, (rows, cols, ld) in enumerate([(1, 512, 512), (8, 300, 301), (3, 1000, 1000),
                                                  (0, 16, 16), (2, 7, 9), (8, 512, 512)]):
            def slice_of(r):
                v = np.arange(max(rows, 1) * ld, dtype=np.float32).reshape(max(rows, 1), ld)
                return (v * 0.5 + 1000.0 * r + call)[:rows]
            src = torch.from_numpy(np.ascontiguousarray(slice_of(rank))).cuda()
            dst = torch.full((max(rows, 1), world * cols), -1.0, device="cuda")
            nimf.check(L.nimf_p2p_allgather_dev(gid.value, ctypes.c_void_p(src.data_ptr()), rows, cols,
                                                ld, ctypes.c_void_p(dst.data_ptr()), world * cols, None))
            torch.cuda.synchronize()
            nimf.check(L.nimf_sync())
            want = np.concatenate([slice_of(r)[:, :cols] for r in range(world)], axis=1)
            got = dst.cpu().numpy()[:rows]
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (rank, call)
        dist.barrier()
        nimf.check(L.nimf_p2p_destroy(gid.value))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except BaseException as e:  # noqa: BLE001
        q.put((rank, "%s: %s" % (type(e).__name__, e)))


def _timeout_worker(rank, world, port, q):
    """Rank 1 skips the second exchange (it leaves between steps, with nothing
    of its own in flight); rank 0's wait for it runs out after the bound."""
    try:
        import time
        import torch
        import torch.distributed as dist
        sys.path.insert(0, os.path.join(HERE, "..", "nimformers-framework_b200"))
        import nimf
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60))
        nimf.init(rank)
        L = nimf.lib()
        bound_ms = 300
        nimf.check(L.nimf_p2p_set_timeout_ms(bound_ms))
        assert L.nimf_p2p_set_timeout_ms(0) == -1
        h = ctypes.create_string_buffer(64)
        gid = ctypes.c_int64()
        nimf.check(L.nimf_p2p_create(world, rank, 1024, h, ctypes.byref(gid)))
        hs = [None] * world
        dist.all_gather_object(hs, h.raw)
        nimf.check(L.nimf_p2p_connect(gid.value, ctypes.create_string_buffer(b"".join(hs), 64 * world)))
        cols = 256
        src = torch.full((1, cols), float(rank + 1), device="cuda")
        dst = torch.full((1, world * cols), -1.0, device="cuda")

        def call():
            nimf.check(L.nimf_p2p_allgather_dev(gid.value, ctypes.c_void_p(src.data_ptr()), 1, cols,
                                                cols, ctypes.c_void_p(dst.data_ptr()), world * cols,
                                                None))
        dist.barrier()
        call()                                   # step 1: both ranks
        nimf.check(L.nimf_sync())
        assert dst.cpu().numpy().tolist()[0] == [1.0] * cols + [2.0] * cols
        dist.barrier()
        if rank == 0:
            dst.fill_(-1.0)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            call()                               # step 2: rank 1 never joins
            call()                               # queued behind it: gives up at once
            rc = L.nimf_sync()
            el = time.perf_counter() - t0
            assert rc == -5, (rc, L.nimf_last_error())
            assert b"expired" in L.nimf_last_error()
            assert bound_ms * 1e-3 * 0.9 <= el < bound_ms * 1e-3 * 1.9 + 0.5, el
            got = dst.cpu().numpy()[0]
            assert np.all(got[cols:] == -1.0)    # the peer's columns were not written
            assert L.nimf_sync() == 0            # the error word was cleared
        dist.barrier()
        nimf.check(L.nimf_p2p_destroy(gid.value))
        nimf.check(L.nimf_p2p_set_timeout_ms(2000))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except BaseException as e:  # noqa: BLE001
        q.put((rank, "%s: %s" % (type(e).__name__, e)))


def _run(target):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200 + (7 if target is _timeout_worker else 0)
    env = dict(os.environ)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        ps = [ctx.Process(target=target, args=(r, 2, port, q)) for r in range(2)]
        for p in ps:
            p.start()
    finally:
        os.environ.clear()
        os.environ.update(env)
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    return res


def test_p2p_wait_expires_when_a_rank_skips_a_call():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _run(_timeout_worker)
    assert res == {0: "ok", 1: "ok"}, res


def test_p2p_allgather_two_gpus():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res
