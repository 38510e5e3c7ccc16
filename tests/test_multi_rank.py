"""N-sharding host logic across ranks, on CPU with the gloo backend.

Every rank holds a contiguous row range of the int4 weight (nimf.shard_rows),
computes its shard's GEMV with the oracle's reference path, and the ranks
all-gather their slices; the reassembled output must equal the full-matrix
result bit for bit (the row order of cpuMatmul does not depend on the shard).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import nimf
import pyoracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n, k, m, gs, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(5)
        w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        x = rng.standard_normal((m, k)).astype(np.float32)
        p, s, z = O.quantize_int4_asym_per_group(w, gs)
        ngr = (k + gs - 1) // gs
        bpr = (k + 1) // 2
        r0, r1 = nimf.shard_rows(n, world, rank)
        y = O.dequant_matmul_q4(x, p[r0 * bpr:r1 * bpr], s[r0 * ngr:r1 * ngr],
                                z[r0 * ngr:r1 * ngr], m, k, r1 - r0, gs, ngr)
        # shards differ in size: gather through a padded, equal-size buffer
        width = max(nimf.shard_rows(n, world, r)[1] - nimf.shard_rows(n, world, r)[0]
                    for r in range(world))
        buf = torch.zeros(m, width)
        buf[:, : r1 - r0] = torch.from_numpy(np.asarray(y, np.float32).reshape(m, -1))
        out = [torch.zeros(m, width) for _ in range(world)]
        dist.all_gather(out, buf)
        if rank == 0:
            parts = []
            for r in range(world):
                a, b = nimf.shard_rows(n, world, r)
                parts.append(out[r][:, : b - a].numpy())
            full = O.dequant_matmul_q4(x, p, s, z, m, k, n, gs, ngr)
            got = nimf.gather_shards(parts, m)
            q.put(bool(np.array_equal(got.view(np.uint32),
                                      np.asarray(full, np.float32).reshape(m, n).view(np.uint32))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n,k,m", [(200, 256, 2), (4096 + 48, 512, 1)])
def test_sharded_gemv_gathers_to_full_result(n, k, m):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, k, m, 128, q))
             for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=120)
    assert all(pr.exitcode == 0 for pr in procs)
    assert q.get(timeout=5)


def test_shard_rows_cover_rows_once():
    for n in (1, 15, 16, 17, 4096, 11008, 32000):
        for world in (1, 2, 4, 8):
            rng = [nimf.shard_rows(n, world, r) for r in range(world)]
            assert rng[0][0] == 0 and rng[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(rng, rng[1:]))
            assert all(r0 % 16 == 0 for r0, _ in rng)
            sizes = [r1 - r0 for r0, r1 in rng]
            assert max(sizes) - min(sizes) <= 16
    with pytest.raises(ValueError):
        nimf.shard_rows(10, 2, 2)


def test_7b_projection_shards_are_equal():
    """The sharded decode measurement all-gathers equal shards: every 7B-shape
    projection (4096, 11008 and 32000 output channels) splits into whole
    16-row tiles of equal size at 1, 2, 4 and 8 GPUs."""
    import nimf
    for n in (4096, 11008, 32000):
        for world in (1, 2, 4, 8):
            sizes = [r1 - r0 for r0, r1 in (nimf.shard_rows(n, world, r) for r in range(world))]
            assert sizes == [n // world] * world, (n, world, sizes)
            assert all(s % 16 == 0 for s in sizes)


def _gather_layout_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)
        m, n, k = 3, 64, 32
        ws = [rng.standard_normal((n, k)).astype(np.float32) for _ in range(3)]   # q, k, v
        x = rng.standard_normal((m, k)).astype(np.float32)
        r0, r1 = nimf.shard_rows(n, world, rank)
        local = torch.from_numpy(np.stack([x @ w[r0:r1].T for w in ws]).astype(np.float32))
        g = torch.empty(world, 3, m, r1 - r0)
        dist.all_gather_into_tensor(g.view(-1), local.contiguous().view(-1))
        # the sharded decode step's reassembly of the q output as the next x
        x_o = g[:, 0].permute(1, 0, 2).reshape(m, n).numpy()
        # reference: the shards' q outputs side by side, computed the same way
        ref = np.concatenate([x @ ws[0][a:b].T for a, b in
                              (nimf.shard_rows(n, world, r) for r in range(world))], axis=1)
        q.put((rank, bool(np.array_equal(x_o, ref.astype(np.float32)))))
    finally:
        dist.destroy_process_group()


def test_sharded_decode_gather_layout():
    """The layout the N-sharded decode measurement rebuilds after each
    projection group's all-gather ([rank][proj][M][N/G] -> [M][N]) equals the
    unsharded output, with two gloo ranks."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_layout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p_ in procs:
        p_.start()
    res = [q.get(timeout=120) for _ in range(2)]
    for p_ in procs:
        p_.join(timeout=120)
    assert all(ok for _, ok in res), res


def test_library_shard_range_matches_host_rule():
    """nimf_shard_range (the library's rule, used by the sharded matmul and the
    sharded decode plan to locate every rank's rows) equals nimf.shard_rows."""
    import ctypes
    L = nimf.lib()
    a, b = ctypes.c_int64(), ctypes.c_int64()
    for n in (0, 1, 15, 16, 17, 4096, 11008, 12288, 28672, 32000, 32001):
        for world in range(1, 9):
            for rank in range(world):
                nimf.check(L.nimf_shard_range(n, world, rank, ctypes.byref(a), ctypes.byref(b)))
                assert (a.value, b.value) == nimf.shard_rows(n, world, rank), (n, world, rank)
    assert L.nimf_shard_range(16, 2, 2, ctypes.byref(a), ctypes.byref(b)) == -1   # NIMF_ERR_ARG
