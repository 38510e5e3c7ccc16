"""The library's communicator paths on one GPU (a communicator of one rank):
nimf_matmul_w_allgather_dev (which is then the plain GEMV), the gather group
with the fused-gather GEMV (its outputs land in the group's buffer; the
arrival exchange is skipped for one rank), and the argument checks.  The
2-GPU behaviour is in test_sharded_multi_gpu.py."""
import ctypes

import numpy as np
import pytest

import pyoracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def comm1(nimf_gpu):
    L = nimf_gpu.lib()
    uid = ctypes.create_string_buffer(128)
    nimf_gpu.check(L.nimf_comm_unique_id(uid))
    nimf_gpu.check(L.nimf_comm_init(1, 0, uid))
    yield nimf_gpu
    nimf_gpu.check(L.nimf_comm_destroy())


def test_comm_info_and_second_init_refused(comm1):
    L = comm1.lib()
    w, r = ctypes.c_int(), ctypes.c_int()
    comm1.check(L.nimf_comm_info(ctypes.byref(w), ctypes.byref(r)))
    assert (w.value, r.value) == (1, 0)
    uid = ctypes.create_string_buffer(128)
    comm1.check(L.nimf_comm_unique_id(uid))
    assert L.nimf_comm_init(1, 0, uid) == -7            # NIMF_ERR_STATE: already exists
    assert L.nimf_comm_init(9, 0, uid) == -1            # world out of range


def test_allgather_matmul_one_rank(comm1):
    import torch
    L = comm1.lib()
    rng = np.random.default_rng(3)
    n, k, m = 1000, 512, 3
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    p, s, z = O.quantize_int4_asym_per_group(w, 128)
    x = rng.standard_normal((m, k)).astype(np.float32)
    h = comm1.Weight.q4g(p, s, z, n, k, 128)
    xd = torch.from_numpy(x).cuda()
    y = torch.empty(m, n, device="cuda")
    y2 = torch.empty(m, n, device="cuda")
    comm1.check(L.nimf_matmul_w_allgather_dev(h.handle, ctypes.c_void_p(xd.data_ptr()), m,
                                              ctypes.c_void_p(y.data_ptr()), None))
    h.matmul_dev(xd.data_ptr(), m, y2.data_ptr())
    torch.cuda.synchronize()
    assert torch.equal(y, y2)
    h.free()


def test_gather_group_one_rank(comm1):
    import cuda.bindings.runtime as crt   # cuda-python
    import torch
    L = comm1.lib()
    rng = np.random.default_rng(4)
    k = 1024
    ns = [512, 1000]
    ws = []
    for n in ns:
        w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        p, s, z = O.quantize_int4_asym_per_group(w, 128)
        ws.append(comm1.Weight.q4g(p, s, z, n, k, 128))
    gid, base = ctypes.c_int64(), ctypes.c_void_p()
    comm1.check(L.nimf_gather_create(8 * sum(ns) * 4, ctypes.byref(gid), ctypes.byref(base)))
    hs = (ctypes.c_uint64 * 2)(*[w.handle for w in ws])
    for m in (1, 5):
        x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()
        offs = [0, m * ns[0] * 4]
        yp = (ctypes.c_void_p * 2)(*[base.value + o for o in offs])
        comm1.check(L.nimf_matmul_w_group_gather_dev(gid.value, hs, 2, ctypes.c_void_p(x.data_ptr()),
                                                     m, yp, None))
        comm1.check(L.nimf_sync())
        got = torch.empty(m * sum(ns), device="cuda")
        err, = crt.cudaMemcpy(got.data_ptr(), base.value, got.numel() * 4,
                              crt.cudaMemcpyKind.cudaMemcpyDeviceToDevice)
        assert int(err) == 0
        g = got.cpu().numpy()
        # the same grouped launch without the gather buffer gives the same bits
        want = [torch.empty(m, n, device="cuda") for n in ns]
        comm1.Weight.matmul_group_dev(ws, x.data_ptr(), m, [t.data_ptr() for t in want])
        torch.cuda.synchronize()
        for i, n in enumerate(ns):
            a = g[offs[i] // 4: offs[i] // 4 + m * n].reshape(m, n)
            assert np.array_equal(a, want[i].cpu().numpy())
    # outputs outside the buffer, too many rows, a non-int4 weight: refused
    x = torch.zeros(1, k, device="cuda")
    bad = (ctypes.c_void_p * 2)(base.value, base.value + 8 * sum(ns) * 4)
    assert L.nimf_matmul_w_group_gather_dev(gid.value, hs, 2, ctypes.c_void_p(x.data_ptr()), 1, bad,
                                            None) == -1
    ok = (ctypes.c_void_p * 2)(base.value, base.value + ns[0] * 4)
    assert L.nimf_matmul_w_group_gather_dev(gid.value, hs, 2, ctypes.c_void_p(x.data_ptr()), 9, ok,
                                            None) == -2
    f = comm1.Weight.f32(np.zeros((k, 16), np.float32), k, 16)
    h1 = (ctypes.c_uint64 * 1)(f.handle)
    assert L.nimf_matmul_w_group_gather_dev(gid.value, h1, 1, ctypes.c_void_p(x.data_ptr()), 1, ok,
                                            None) == -6
    f.free()
    comm1.check(L.nimf_gather_destroy(gid.value))
    for w in ws:
        w.free()
