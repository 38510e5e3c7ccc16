#!/usr/bin/env python
"""Benchmark of the int4-g128 decode GEMV (the quantised-weight matmul hot path).

Workload (one step): y_r[M, N] = x[M, K] . W_r^T for R distinct int4 group-128
asymmetric weights W_r (K=4096, N=12288, M=1; W ~ N(0, 0.02), quantised with
the exporter's per-group rule), all resident in HBM, issued as one grouped
launch (nimf_matmul_w_group_dev: the weights share x, like fused projections).
R copies (> 3x L2 in total) rotate, so every step streams its weights from
HBM.  The same R GEMVs issued as R separate launches (PDL-chained in a CUDA
graph) are reported as "single_launch".  With --gpus G the
weight rows are N-sharded (each GPU holds 12288 rows of a 12288*G-row weight:
per-GPU work is fixed, "weak" scaling) and the output slices are all-gathered
over NCCL inside the step.

Prints one JSON line (rank 0): value = algorithmic bytes streamed by all ranks
per second (GB/s), the roofline of the GEMV kernel, an end-to-end number
through the C ABI with host buffers, and (N=1) the CPU reference path timed on
the host.  --impl reference times the reference's CPU path (the C restatement
of gpubackend.nim cpuDequantMatmulQ4Fallback + cpuMatmul) instead.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "nimformers-framework_b200"))

K, N_PER_GPU, M, GS = 4096, 12288, 1, 128
METRIC = "int4 GEMV HBM GB/s"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0}


def algo_bytes(n, k, m, gs):
    """Bytes a GEMV must move: packed nibbles + fp32 scale and zero per group
    + x + y (the per-unit figure the roofline uses)."""
    return n * k // 2 + n * ((k + gs - 1) // gs) * 8 + 4 * m * k + 4 * m * n


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return d, "measured"
    except Exception:
        return PEAKS_FALLBACK, "fallback"


def profile_traffic():
    """DRAM bytes per GEMV launch from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "q4g_gemv_k4096_n12288_m1.txt")
    try:
        for line in open(p):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    except OSError:
        pass
    return None


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), "--query-gpu=" + self.FIELDS,
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [v.strip() for v in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def workload_config(world, copies):
    """The bench workload, identical in both arms' JSON lines."""
    return {"workload": "int4-g128 decode GEMV K=4096 N=12288 M=1 per GPU",
            "K": K, "N_per_gpu": N_PER_GPU, "N_total": N_PER_GPU * world, "M": M,
            "group_size": GS, "weight_copies": copies,
            "l2": "inputs larger than L2: %d rotating weight copies, %.0f MB per GPU"
                  % (copies, copies * algo_bytes(N_PER_GPU, K, M, GS) / 1e6),
            "parallelism": ("N-shard x%d, output all-gather fused into the GEMV launch"
                            % world) if world > 1 else "single GPU"}


def cpu_reference_gemv_rate(p, s, z, x, seconds, rows=None):
    """Times the reference CPU path (oracle restatement of
    gpubackend.nim:628-653 + :560-582) on the first `rows` output rows.
    Returns (GB/s of the metric, description)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import pyoracle as O
    n = N_PER_GPU if rows is None else rows
    bpr = K // 2
    ngr = K // GS
    pp, ss, zz = p[: n * bpr], s[: n * ngr], z[: n * ngr]
    it, t0 = 0, time.perf_counter()
    while True:
        O.dequant_matmul_q4(x, pp, ss, zz, M, K, n, GS, ngr)
        it += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    rate = algo_bytes(n, K, M, GS) * it / el / 1e9
    desc = ("%d x GEMV K=%d N=%d M=%d through cpuDequantMatmulQ4Fallback+cpuMatmul "
            "(C restatement, 1 thread) in %.1f s" % (it, K, n, M, el))
    return rate, desc


def run_reference(args, rank, world):
    """The reference's CPU path (oracle port), on every host core the process
    may use: the reference runs it on one thread, here disjoint row ranges of
    each step's GEMV run on parallel threads (the C restatement releases the
    interpreter lock), so the baseline is the fastest this CPU code gets."""
    if rank != 0:
        return
    import threading

    import numpy as np
    import nimf
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle as O
    w = (np.random.default_rng(0).standard_normal((N_PER_GPU, K)) * 0.02).astype(np.float32)
    p, s, z = nimf.quantize_int4_per_group(w, GS)
    x = np.random.default_rng(1).standard_normal((M, K)).astype(np.float32)
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    cores = max(1, int(cores or 1))
    bpr, ngr = K // 2, K // GS

    def gemv(rows):
        # rows split into `cores` contiguous slices, one thread each
        bounds = [rows * i // cores for i in range(cores + 1)]
        ts = []
        for i in range(cores):
            r0, r1 = bounds[i], bounds[i + 1]
            if r1 <= r0:
                continue
            ts.append(threading.Thread(target=O.dequant_matmul_q4, args=(
                x, p[r0 * bpr: r1 * bpr], s[r0 * ngr: r1 * ngr], z[r0 * ngr: r1 * ngr],
                M, K, r1 - r0, GS, ngr)))
        for t in ts:
            t.start()
        for t in ts:
            t.join()

    # every step is the whole GEMV (all 12288 output rows), its rows split into
    # one contiguous range per thread (each thread's transposed slice is small
    # enough to stay in its cache, which a single thread's full slice is not)
    rows = N_PER_GPU
    for _ in range(args.warmup):
        gemv(rows)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        gemv(rows)
    el = time.perf_counter() - t0
    value = algo_bytes(rows, K, M, GS) * args.steps / el / 1e9
    sample = ("each step: the whole GEMV K=%d N=%d M=%d through "
              "cpuDequantMatmulQ4Fallback+cpuMatmul (C restatement), its rows split into %d "
              "contiguous ranges on %d threads" % (K, rows, M, cores, cores))
    line = {"metric": METRIC, "value": value, "unit": "GB/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": el / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u4 weights, f32 activations/accumulate",
            "data": "synthetic",
            "config": workload_config(world, args.copies),
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# 7B-shape decoder stack (32 layers, d_model 4096, 32 heads x 128, SiLU-gated
# FFN 11008, vocab 32000), int4 group-128 weights: the matmul path of one
# decode step = per layer q/k/v (one grouped launch), o, gate/up (one grouped
# launch), down; then lm_head.
D7, F7, V7, L7 = 4096, 11008, 32000, 32


def decode7b_bytes(batch):
    """Weight + activation bytes one decode step streams (algorithmic)."""
    per_layer = (algo_bytes(3 * D7, D7, batch, GS) + algo_bytes(D7, D7, batch, GS)
                 + algo_bytes(2 * F7, D7, batch, GS) + algo_bytes(D7, F7, batch, GS))
    return L7 * per_layer + algo_bytes(V7, D7, batch, GS)


def p2p_group(nimf, world, rank, slot_floats):
    """A peer-memory all-gather group of the library (CUDA IPC handles
    exchanged over the process group)."""
    import ctypes
    import torch.distributed as dist
    L = nimf.lib()
    h = ctypes.create_string_buffer(64)
    gid = ctypes.c_int64()
    err = None
    try:
        nimf.check(L.nimf_p2p_create(world, rank, slot_floats, h, ctypes.byref(gid)))
    except Exception as e:  # noqa: BLE001
        err = str(e)
    # every rank learns every rank's outcome, so a failure raises on all of them
    got = [None] * world
    dist.all_gather_object(got, (h.raw, err))
    bad = [(r, e) for r, (_, e) in enumerate(got) if e]
    if bad:
        raise RuntimeError("peer-memory group: create failed on %s" % bad)
    allh = ctypes.create_string_buffer(b"".join(g[0] for g in got), 64 * world)
    try:
        nimf.check(L.nimf_p2p_connect(gid.value, allh))
    except Exception as e:  # noqa: BLE001
        err = str(e)
    errs = [None] * world
    dist.all_gather_object(errs, err)
    bad = [(r, e) for r, e in enumerate(errs) if e]
    if bad:
        raise RuntimeError("peer-memory group: connect failed on %s" % bad)
    return gid.value


def run_decode_7b(nimf, torch, steps, warmup, rank=0, world=1, exchange="p2p", batches=(1, 8)):
    """tok/s of the 7B-shape int4 decode matmul path, batch 1 and 8.

    Weights are synthetic int4 codes (seeded random bytes) with group scales
    and zeros of the magnitude N(0, 0.02) weights quantise to; every layer has
    its own device copy, so each step streams all 3.7 GB from HBM.  The
    activation glue between projections (norms, attention, SiLU) is not on
    this path; each projection reads the previous one's output.

    With world > 1 GPUs every projection is N-sharded (rank r holds rows
    nimf.shard_rows(N, world, r) of every weight, 3.7 GB / world per GPU) and
    the output slice the next projection reads is all-gathered inside the
    captured step into that projection's x [batch][N]: exchange "p2p" with the
    library's peer-memory all-gather (one kernel: peer stores over NVLink, a
    flag per peer), "nccl" with NCCL all-gathers of each group's outputs
    followed by a layout copy.  Step time is the max over ranks."""
    import numpy as np
    rng = np.random.default_rng(4)
    dist = None
    if world > 1:
        import torch.distributed as dist

    def make(n, k):
        ngr = k // GS
        p = rng.integers(0, 256, size=n * (k // 2), dtype=np.uint8)
        sc = rng.uniform(0.002, 0.004, size=n * ngr).astype(np.float32)
        zp = rng.uniform(6.0, 9.0, size=n * ngr).astype(np.float32)
        return p, sc, zp

    shapes = {"q": (D7, D7), "o": (D7, D7), "gu": (F7, D7), "down": (D7, F7), "head": (V7, D7)}
    host = {kname: make(*nk) for kname, nk in shapes.items()}

    def reg(kname):
        n, k = shapes[kname]
        return nimf.Weight.q4g(*host[kname], n, k, GS, rows=nimf.shard_rows(n, world, rank))

    layers = []
    for _ in range(L7):
        q, k, v = [reg("q") for _ in range(3)]
        o = reg("o")
        gate, up = [reg("gu") for _ in range(2)]
        down = reg("down")
        layers.append((q, k, v, o, gate, up, down))
    head = reg("head")
    nd, nf, nv = D7 // world, F7 // world, V7 // world   # equal shards at 1/2/4/8 GPUs
    out = {}
    L = nimf.lib()
    gid = None
    try:
        if world > 1 and exchange == "p2p":
            gid = p2p_group(nimf, world, rank, max(batches) * max(nd, nf, nv))

        def p2p(src, cols, ld_src, dst, st, batch):
            nimf.check(L.nimf_p2p_allgather_dev(gid, src.data_ptr(), batch, cols, ld_src,
                                                dst.data_ptr(), cols * world, st))

        for batch in batches:
            dev = torch.device("cuda")
            x = torch.randn(batch, D7, device=dev)
            qkv = torch.empty(3, batch, nd, device=dev)
            att = torch.empty(batch, nd, device=dev)
            gu = torch.empty(2, batch, nf, device=dev)
            dn = torch.empty(batch, nd, device=dev)
            logits = torch.empty(batch, nv, device=dev)
            if world > 1:
                g_qkv = torch.empty(world, 3, batch, nd, device=dev)
                g_att = torch.empty(world, batch, nd, device=dev)
                g_gu = torch.empty(world, 2, batch, nf, device=dev)
                g_dn = torch.empty(world, batch, nd, device=dev)
                g_log = torch.empty(world, batch, nv, device=dev)
                x_o = torch.empty(batch, D7, device=dev)     # full q output
                x_gu = torch.empty(batch, D7, device=dev)    # full o output
                x_dn = torch.empty(batch, F7, device=dev)    # full gate output
                x_l = torch.empty(batch, D7, device=dev)     # full down output
                x_log = torch.empty(batch, V7, device=dev)   # full logits
            stream = torch.cuda.Stream()

            def step(st):
                h = x
                for (q, k, v, o, gate, up, down) in layers:
                    nimf.Weight.matmul_group_dev([q, k, v], h.data_ptr(), batch,
                                                 [qkv[i].data_ptr() for i in range(3)], st)
                    xo = qkv[0]
                    if world > 1 and gid is not None:
                        p2p(qkv[0], nd, nd, x_o, st, batch)
                        xo = x_o
                    elif world > 1:
                        dist.all_gather_into_tensor(g_qkv.view(-1), qkv.view(-1))
                        x_o.copy_(g_qkv[:, 0].permute(1, 0, 2).reshape(batch, D7))
                        xo = x_o
                    o.matmul_dev(xo.data_ptr(), batch, att.data_ptr(), st)
                    xg = att
                    if world > 1 and gid is not None:
                        p2p(att, nd, nd, x_gu, st, batch)
                        xg = x_gu
                    elif world > 1:
                        dist.all_gather_into_tensor(g_att.view(-1), att.view(-1))
                        x_gu.copy_(g_att.permute(1, 0, 2).reshape(batch, D7))
                        xg = x_gu
                    nimf.Weight.matmul_group_dev([gate, up], xg.data_ptr(), batch,
                                                 [gu[0].data_ptr(), gu[1].data_ptr()], st)
                    xd = gu[0]
                    if world > 1 and gid is not None:
                        p2p(gu[0], nf, nf, x_dn, st, batch)
                        xd = x_dn
                    elif world > 1:
                        dist.all_gather_into_tensor(g_gu.view(-1), gu.view(-1))
                        x_dn.copy_(g_gu[:, 0].permute(1, 0, 2).reshape(batch, F7))
                        xd = x_dn
                    down.matmul_dev(xd.data_ptr(), batch, dn.data_ptr(), st)
                    h = dn
                    if world > 1 and gid is not None:
                        p2p(dn, nd, nd, x_l, st, batch)
                        h = x_l
                    elif world > 1:
                        dist.all_gather_into_tensor(g_dn.view(-1), dn.view(-1))
                        x_l.copy_(g_dn.permute(1, 0, 2).reshape(batch, D7))
                        h = x_l
                head.matmul_dev(h.data_ptr(), batch, logits.data_ptr(), st)
                if world > 1 and gid is not None:
                    p2p(logits, nv, nv, x_log, st, batch)
                elif world > 1:
                    dist.all_gather_into_tensor(g_log.view(-1), logits.view(-1))

            with torch.cuda.stream(stream):
                step(stream.cuda_stream)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                step(stream.cuda_stream)
            for _ in range(warmup):
                graph.replay()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(steps):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            bad = L.nimf_sync() != 0   # a peer wait that ran out is reported here
            ms = e0.elapsed_time(e1) / steps
            if world > 1:
                # the status travels with the time, so every rank raises together
                t = torch.tensor([ms, float(bad)], device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms, bad = float(t[0].item()), t[1].item() > 0
                dist.barrier()
            if bad:
                raise RuntimeError("a device wait of the sharded decode expired on some rank")
            graph.reset()
            del graph
            out["batch%d" % batch] = {
                "tok_s": batch / (ms * 1e-3), "ms_per_step": ms,
                "gb_s": decode7b_bytes(batch) / (ms * 1e-3) / 1e9,
                "bytes_per_step": decode7b_bytes(batch)}
    finally:
        if gid is not None:
            torch.cuda.synchronize()
            dist.barrier()
            nimf.check(L.nimf_p2p_destroy(gid))
        for lw in layers:
            for w in lw:
                w.free()
        head.free()
    out["launches_per_step"] = 4 * L7 + 1 + ((4 * L7 + 1) if exchange == "p2p" and world > 1 else 0)
    out["n_gpus"] = world
    if world > 1:
        out["all_gathers_per_step"] = 4 * L7 + 1
        out["exchange"] = exchange
    out["note"] = ("matmul path only (grouped q/k/v and gate/up), one CUDA graph per step, "
                   "synthetic int4-g128 weights, %d timed steps%s" % (
                       steps, "" if world == 1 else
                       "; N-sharded over %d GPUs, the output slice each next projection reads "
                       "all-gathered (%s) after every projection group, step time = max over "
                       "ranks" % (world, "one peer-memory kernel over NVLink" if exchange == "p2p"
                                  else "NCCL + layout copy")))
    return out


def decode_timeline(nimf, torch, plan, one, tok):
    """Per-stage averages (microseconds) of one recorded step of a decode plan
    for CTA 0, from nimf_decode_timeline's %globaltimer marks: for each stage
    kind of a layer (q/k/v GEMV, attention, o GEMV, gate/up GEMV, down GEMV;
    lm_head last) the wait at the grid barrier after the previous stage
    (`gap`), the x prologue (`pro`: inputs, norm, max|x|, digits) and the body
    up to the CTA's arrival (`body`); `chunk0` is consumer warp 0's first
    chunk (16 rows x 512 k: fragment loads, 16 MMAs, scales)."""
    import ctypes
    L = nimf.lib()
    nst = plan.info()["stages"]
    marks = 12
    tl = torch.zeros(marks * nst, dtype=torch.int64, device="cuda")
    nimf.check(L.nimf_decode_timeline(plan.plan, ctypes.c_void_p(tl.data_ptr()), marks * nst, 0))
    one(tok)
    torch.cuda.synchronize()
    nimf.check(L.nimf_sync())
    nimf.check(L.nimf_decode_timeline(plan.plan, None, 0, 0))
    t = tl.cpu().numpy().reshape(nst, marks).astype(float) / 1e3
    names = ["qkv", "attn", "o", "gate_up", "down"]
    agg = {}
    for i in range(nst):
        kind = "lm_head" if i == nst - 1 else names[i % 5]
        r = t[i]
        gap = r[0] - t[i - 1][2] if i > 0 else 0.0
        pro = r[1] - r[0] if r[1] > 0 else 0.0
        body = r[2] - (r[1] if r[1] > 0 else r[0])
        c0 = r[9] - r[6] if (r[9] > 0 and r[6] > 0) else 0.0
        d = agg.setdefault(kind, [0, 0.0, 0.0, 0.0, 0.0])
        d[0] += 1
        d[1] += gap
        d[2] += pro
        d[3] += body
        d[4] += c0
    out = {k: {"gap": round(v[1] / v[0], 2), "pro": round(v[2] / v[0], 2), "body": round(v[3] / v[0], 2),
               "chunk0": round(v[4] / v[0], 2)} for k, v in agg.items()}
    out["step_us"] = round(float(t[-1][2] - t[t > 0].min()), 1)
    return out


def run_decode_7b_full(nimf, torch, steps, warmup, pos=512, max_seq=640, layers=L7):
    """tok/s of one whole 7B-shape decode step at batch 1 with the glue on the
    device: per layer RMSNorm, fused q/k/v GEMV, RoPE on q and k (one launch),
    KV-cache append + attention over pos + 1 positions (32 heads x 128), o GEMV,
    residual add fused with the next RMSNorm, fused gate/up GEMV, SwiGLU, down
    GEMV, residual add fused with the next layer's (or the final) RMSNorm; then
    the lm_head GEMV (nim_inference.nim:847-921's order).  The step starts from
    a token id on the device (embedding row lookup) and ends with the greedy
    choice of the next id with the repetition penalty over 64 recent ids
    (sampleTopP at temperature 0), which the next replay embeds: token in,
    token out, nothing crosses PCIe.  One CUDA graph per step; synthetic
    int4-g128 weights, random embedding table, norm weights and KV caches
    (fp32, 32 x 2 x 32 x 640 x 128)."""
    import ctypes
    import numpy as np
    rng = np.random.default_rng(6)
    L = nimf.lib()
    H, HD = 32, 128

    def make(n, k):
        ngr = k // GS
        p = rng.integers(0, 256, size=n * (k // 2), dtype=np.uint8)
        sc = rng.uniform(0.002, 0.004, size=n * ngr).astype(np.float32)
        zp = rng.uniform(6.0, 9.0, size=n * ngr).astype(np.float32)
        return p, sc, zp

    hq, hg, hd, hh = make(D7, D7), make(F7, D7), make(D7, F7), make(V7, D7)
    dev = torch.device("cuda")
    nlayers = layers
    layers = []
    for _ in range(nlayers):
        q, k, v, o = [nimf.Weight.q4g(*hq, D7, D7, GS) for _ in range(4)]
        gate, up = [nimf.Weight.q4g(*hg, F7, D7, GS) for _ in range(2)]
        down = nimf.Weight.q4g(*hd, D7, F7, GS)
        n1 = torch.rand(D7, device=dev) + 0.5
        n2 = torch.rand(D7, device=dev) + 0.5
        kc = torch.randn(H * max_seq * HD, device=dev)
        vc = torch.randn(H * max_seq * HD, device=dev)
        layers.append((q, k, v, o, gate, up, down, n1, n2, kc, vc))
    head = nimf.Weight.q4g(*hh, V7, D7, GS)
    nf = torch.rand(D7, device=dev) + 0.5
    half = HD // 2
    inv = 1.0 / np.power(np.float32(10000.0), np.arange(half, dtype=np.float32) / np.float32(half))
    ang = np.arange(max_seq, dtype=np.float32)[:, None] * inv[None, :].astype(np.float32)
    cos_t = torch.from_numpy(np.cos(ang).astype(np.float32)).to(dev)
    sin_t = torch.from_numpy(np.sin(ang).astype(np.float32)).to(dev)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    table = torch.randn(V7, D7, device=dev) * 0.02
    tok = torch.tensor([1234], dtype=torch.int32, device=dev)
    recent = torch.from_numpy(rng.integers(0, V7, size=64).astype(np.int32)).to(dev)
    x = torch.empty(1, D7, device=dev)
    h = torch.empty(1, D7, device=dev)
    xn = torch.empty(1, D7, device=dev)
    qkv = torch.empty(3, 1, D7, device=dev)
    att = torch.empty(1, D7, device=dev)
    ao = torch.empty(1, D7, device=dev)
    gu = torch.empty(2, 1, F7, device=dev)
    act = torch.empty(1, F7, device=dev)
    dn = torch.empty(1, D7, device=dev)
    logits = torch.empty(1, V7, device=dev)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(HD)))

    def step(st):
        sp = ctypes.c_void_p(st)
        nimf.check(L.nimf_embedding_lookup_dev(P(table), V7, D7, P(tok), 1, P(x), sp))
        nimf.check(L.nimf_rmsnorm_dev(P(x), P(layers[0][7]), 1, D7, ctypes.c_float(1e-6), P(xn), sp))
        for li, (q, k, v, o, gate, up, down, n1, n2, kc, vc) in enumerate(layers):
            nimf.Weight.matmul_group_dev([q, k, v], xn.data_ptr(), 1,
                                         [qkv[i].data_ptr() for i in range(3)], st)
            # q and k are adjacent in qkv: one launch rotates both (2 H heads)
            nimf.check(L.nimf_rope_dev(P(qkv[0]), 1, 1, 2 * H, HD, pos, P(cos_t), P(sin_t), max_seq, sp))
            nimf.check(L.nimf_attention_decode_dev(P(qkv[0]), P(qkv[1]), P(qkv[2]), P(kc), P(vc),
                                                   H, H, HD, max_seq, pos, ctypes.c_float(scale),
                                                   P(att), sp))
            o.matmul_dev(att.data_ptr(), 1, ao.data_ptr(), st)
            # h = x + attention output, xn = RMSNorm(h)
            nimf.check(L.nimf_add_rmsnorm_dev(P(x), P(ao), P(n2), 1, D7, ctypes.c_float(1e-6),
                                              P(h), P(xn), sp))
            nimf.Weight.matmul_group_dev([gate, up], xn.data_ptr(), 1,
                                         [gu[0].data_ptr(), gu[1].data_ptr()], st)
            nimf.check(L.nimf_swiglu_dev(P(gu[0]), P(gu[1]), F7, P(act), sp))
            down.matmul_dev(act.data_ptr(), 1, dn.data_ptr(), st)
            # x = h + FFN output, xn = the next layer's (or the final) RMSNorm of x
            nxt = layers[li + 1][7] if li + 1 < len(layers) else nf
            nimf.check(L.nimf_add_rmsnorm_dev(P(h), P(dn), P(nxt), 1, D7, ctypes.c_float(1e-6),
                                              P(x), P(xn), sp))
        head.matmul_dev(xn.data_ptr(), 1, logits.data_ptr(), st)
        nimf.check(L.nimf_greedy_sample_dev(P(logits), 1, V7, P(recent), 64, ctypes.c_float(1.3),
                                            P(tok), sp))

    kv_bytes = nlayers * 2 * H * (pos + 1) * HD * 4
    res = {"position": pos, "weight_bytes_per_step": decode7b_bytes(1),
           "kv_bytes_per_step": kv_bytes}
    plan = None
    try:
        # (1) one launch per op, captured in a CUDA graph
        tok.fill_(1234)
        ms = graph_ms(torch, step, steps, warmup)
        tok.fill_(1234)
        st0 = torch.cuda.current_stream().cuda_stream
        step(st0)
        torch.cuda.synchronize()
        ref_logits, ref_tok = logits.clone(), int(tok.item())
        assert 0 <= ref_tok < V7
        res["per_op"] = {"tok_s": 1.0 / (ms * 1e-3), "ms_per_step": ms,
                         "gb_s": (decode7b_bytes(1) + kv_bytes) / (ms * 1e-3) / 1e9,
                         "launches_per_step": nlayers * 9 + 4}
        # (2) the whole step as one persistent launch (nimf_decode_step_dev)
        lds = [{"wq": q, "wk": k, "wv": v, "wo": o, "wgate": gate, "wup": up, "wdown": down,
                "attn_norm": n1.data_ptr(), "ffn_norm": n2.data_ptr(),
                "k_cache": kc.data_ptr(), "v_cache": vc.data_ptr()}
               for li, (q, k, v, o, gate, up, down, n1, n2, kc, vc) in enumerate(layers)]
        plan = nimf.DecodePlan(layers=lds, embedding=table.data_ptr(), final_norm=nf.data_ptr(),
                               lm_head=head, rope_cos=cos_t.data_ptr(), rope_sin=sin_t.data_ptr(),
                               d_model=D7, n_heads=H, n_kv_heads=H, head_dim=HD, ffn_dim=F7,
                               vocab=V7, max_seq=max_seq, norm_eps=1e-6)
        pos_d = torch.tensor([pos], dtype=torch.int32, device=dev)
        tok1 = torch.tensor([1234], dtype=torch.int32, device=dev)
        nxt1 = torch.empty(1, dtype=torch.int32, device=dev)
        logits1 = torch.empty(V7, device=dev)
        sp = torch.cuda.Stream()

        def one(out_tok):
            plan.step(tok1.data_ptr(), out_tok.data_ptr(), pos_d.data_ptr(), logits1.data_ptr(),
                      recent.data_ptr(), 64, 1.3, stream=sp.cuda_stream)

        one(nxt1)
        torch.cuda.synchronize()
        nimf.check(L.nimf_sync())
        err = float((logits1 - ref_logits.view(-1)).abs().max() / ref_logits.abs().max())
        one_tok = int(nxt1.item())
        for _ in range(warmup):
            one(tok1)                      # token in -> token out, as the graph above
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(sp):
            e0.record()
            for _ in range(steps):
                one(tok1)
            e1.record()
        torch.cuda.synchronize()
        nimf.check(L.nimf_sync())
        ms1 = e0.elapsed_time(e1) / steps
        res["one_launch"] = {"tok_s": 1.0 / (ms1 * 1e-3), "ms_per_step": ms1,
                             "gb_s": (decode7b_bytes(1) + kv_bytes) / (ms1 * 1e-3) / 1e9,
                             "launches_per_step": 1, "plan": plan.info(),
                             "logits_rel_err_vs_per_op": err,
                             "same_token_as_per_op": one_tok == ref_tok,
                             "timeline_cta0_us": decode_timeline(nimf, torch, plan, one, tok1)}
        # the same plan with the producers' L2 look-ahead, for comparison
        plan.destroy()
        os.environ["NIMF_DECODE_L2_AHEAD"] = "2"
        try:
            plan = nimf.DecodePlan(layers=lds, embedding=table.data_ptr(), final_norm=nf.data_ptr(),
                                   lm_head=head, rope_cos=cos_t.data_ptr(), rope_sin=sin_t.data_ptr(),
                                   d_model=D7, n_heads=H, n_kv_heads=H, head_dim=HD, ffn_dim=F7,
                                   vocab=V7, max_seq=max_seq, norm_eps=1e-6)
        finally:
            del os.environ["NIMF_DECODE_L2_AHEAD"]
        for _ in range(warmup):
            one(tok1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(sp):
            e0.record()
            for _ in range(steps):
                one(tok1)
            e1.record()
        torch.cuda.synchronize()
        nimf.check(L.nimf_sync())
        ms0 = e0.elapsed_time(e1) / steps
        res["one_launch_l2_ahead2"] = {"tok_s": 1.0 / (ms0 * 1e-3), "ms_per_step": ms0}
    finally:
        if plan is not None:
            plan.destroy()
        for lw in layers:
            for w in lw[:7]:
                w.free()
        head.free()
    res["tok_s"] = max(res["per_op"]["tok_s"], res.get("one_launch", {}).get("tok_s", 0.0))
    res["note"] = ("batch 1, whole decode step on the device, token id in -> greedy token id out "
                   "(embedding lookup, glue, int4-g128 matmuls, lm_head, repetition-penalised "
                   "argmax); per_op: one launch per op in one CUDA graph; one_launch: "
                   "nimf_decode_step_dev; KV caches fp32 [32 heads][640][128] per layer, %d timed "
                   "steps each" % steps)
    return res


def lib_comm_init(nimf, rank, world):
    """The library's own NCCL communicator (nimf_comm_init); rank 0's unique
    id travels over the process group."""
    import ctypes
    import torch.distributed as dist
    L = nimf.lib()
    w, r = ctypes.c_int(), ctypes.c_int()
    nimf.check(L.nimf_comm_info(ctypes.byref(w), ctypes.byref(r)))
    if w.value == world and world > 1:
        return                      # already initialised
    uid = ctypes.create_string_buffer(128)
    if rank == 0:
        nimf.check(L.nimf_comm_unique_id(uid))
    box = [uid.raw]
    dist.broadcast_object_list(box, src=0)
    nimf.check(L.nimf_comm_init(world, rank, ctypes.create_string_buffer(box[0], 128)))


def run_decode_7b_sharded(nimf, torch, steps, warmup, rank, world, pos=512, max_seq=640,
                          layers=L7):
    """tok/s of the whole 7B-shape batch-1 decode step N-sharded over `world`
    GPUs as one launch per GPU (nimf_decode_create_sharded): rank r holds
    nimf.shard_rows rows of every projection and lm_head (3.7 GB / world) and
    the KV caches of heads [r*32/world, (r+1)*32/world); inside the launch
    every stage's outputs go to every GPU over NVLink with plain peer stores
    and cross-GPU arrival counters.  Token id in -> greedy token id out, as
    run_decode_7b_full; step time = max over ranks of CUDA-event time."""
    import torch.distributed as dist
    import numpy as np
    rng = np.random.default_rng(6)
    H, HD = 32, 128
    hl = H // world

    def make(n, k):
        ngr = k // GS
        p = rng.integers(0, 256, size=n * (k // 2), dtype=np.uint8)
        sc = rng.uniform(0.002, 0.004, size=n * ngr).astype(np.float32)
        zp = rng.uniform(6.0, 9.0, size=n * ngr).astype(np.float32)
        return p, sc, zp

    hq, hg, hd, hh = make(D7, D7), make(F7, D7), make(D7, F7), make(V7, D7)
    dev = torch.device("cuda")
    rows = lambda n: nimf.shard_rows(n, world, rank)
    lws, keep, ws = [], [], []
    plan = None
    try:
        for _ in range(layers):
            q, k, v, o = [nimf.Weight.q4g(*hq, D7, D7, GS, rows=rows(D7)) for _ in range(4)]
            gate, up = [nimf.Weight.q4g(*hg, F7, D7, GS, rows=rows(F7)) for _ in range(2)]
            down = nimf.Weight.q4g(*hd, D7, F7, GS, rows=rows(D7))
            ws += [q, k, v, o, gate, up, down]
            n1 = torch.rand(D7, device=dev) + 0.5
            n2 = torch.rand(D7, device=dev) + 0.5
            kc = torch.randn(hl * max_seq * HD, device=dev)
            vc = torch.randn(hl * max_seq * HD, device=dev)
            keep += [n1, n2, kc, vc]
            lws.append({"wq": q, "wk": k, "wv": v, "wo": o, "wgate": gate, "wup": up, "wdown": down,
                        "attn_norm": n1.data_ptr(), "ffn_norm": n2.data_ptr(),
                        "k_cache": kc.data_ptr(), "v_cache": vc.data_ptr()})
        head = nimf.Weight.q4g(*hh, V7, D7, GS, rows=rows(V7))
        ws.append(head)
        nf = torch.rand(D7, device=dev) + 0.5
        half = HD // 2
        inv = 1.0 / np.power(np.float32(10000.0), np.arange(half, dtype=np.float32) / np.float32(half))
        ang = np.arange(max_seq, dtype=np.float32)[:, None] * inv[None, :].astype(np.float32)
        cos_t = torch.from_numpy(np.cos(ang).astype(np.float32)).to(dev)
        sin_t = torch.from_numpy(np.sin(ang).astype(np.float32)).to(dev)
        table = torch.randn(V7, D7, device=dev) * 0.02
        recent = torch.from_numpy(np.random.default_rng(7).integers(0, V7, size=64)
                                  .astype(np.int32)).to(dev)
        keep += [nf, cos_t, sin_t, table, recent]
        nimf.check(nimf.lib().nimf_decode_set_timeout_ms(500))
        plan = nimf.DecodePlan(layers=lws, embedding=table.data_ptr(), final_norm=nf.data_ptr(),
                               lm_head=head, rope_cos=cos_t.data_ptr(), rope_sin=sin_t.data_ptr(),
                               d_model=D7, n_heads=H, n_kv_heads=H, head_dim=HD, ffn_dim=F7,
                               vocab=V7, max_seq=max_seq, norm_eps=1e-6, sharded=True)
        pos_d = torch.tensor([pos], dtype=torch.int32, device=dev)
        tok = torch.tensor([1234], dtype=torch.int32, device=dev)
        logits = torch.empty(V7, device=dev)
        sp = torch.cuda.Stream()

        def one():
            plan.step(tok.data_ptr(), tok.data_ptr(), pos_d.data_ptr(), logits.data_ptr(),
                      recent.data_ptr(), 64, 1.3, stream=sp.cuda_stream)

        for _ in range(warmup):
            one()
        torch.cuda.synchronize()
        bad = nimf.lib().nimf_sync() != 0
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(sp):
            e0.record()
            for _ in range(steps):
                one()
            e1.record()
        torch.cuda.synchronize()
        bad = bad or nimf.lib().nimf_sync() != 0
        ms = e0.elapsed_time(e1) / steps
        toks = [None] * world
        dist.all_gather_object(toks, int(tok.item()))
        t = torch.tensor([ms, float(bad)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, bad = float(t[0].item()), t[1].item() > 0
        if bad:
            raise RuntimeError("a grid-barrier wait of the sharded decode step expired on some rank")
        info = plan.info()
    finally:
        if plan is not None:
            plan.destroy()
        for w in ws:
            w.free()
    kv_bytes = layers * 2 * H * (pos + 1) * HD * 4
    return {"one_launch": {"tok_s": 1.0 / (ms * 1e-3), "ms_per_step": ms,
                           "gb_s": (decode7b_bytes(1) + kv_bytes) / (ms * 1e-3) / 1e9,
                           "launches_per_step": 1, "plan": info,
                           "same_token_on_every_rank": len(set(toks)) == 1},
            "tok_s": 1.0 / (ms * 1e-3), "ms_per_step": ms, "position": pos, "n_gpus": world,
            "note": ("batch 1, whole decode step as one launch per GPU, N-sharded over %d GPUs "
                     "(projections by output rows, attention by heads), stage outputs exchanged "
                     "inside the launch over NVLink peer stores; %d timed steps, max over ranks"
                     % (world, steps))}


def run_generate_7b(nimf, torch, batch=1, prompt=512, new_tokens=128, layers=L7, max_seq=640):
    """The 7B-shape stack's whole generation (LlamaModelL.generate,
    nim_inference.nim:1064-1140) for `batch` independent sequences: each
    prompt of `prompt` random token ids goes through forwardPrefill
    (:574-620) -- per layer RMSNorm, the q/k/v, o, gate/up and down
    projections as tcgen05 GEMMs over all batch x prompt rows, RoPE, the
    causal prompt attention with appendKV (per sequence), SwiGLU and the
    residual adds -- then the final norm, lm_head on each sequence's last row
    and the greedy first tokens; then `new_tokens` greedy decode steps over
    the caches the prefill filled (token out -> token in, positions advanced
    on the device).  Batch 1 decodes with the one-launch plan; batch > 1 with
    one captured step of the per-op path (grouped GEMVs over the batch rows,
    nimf_attention_decode_batch_dev at device positions), replayed per token.
    Synthetic int4-g128 weights; CUDA events around each phase."""
    import ctypes
    import numpy as np
    rng = np.random.default_rng(8)
    L = nimf.lib()
    H, HD, B = 32, 128, batch

    def make(n, k):
        ngr = k // GS
        p = rng.integers(0, 256, size=n * (k // 2), dtype=np.uint8)
        sc = rng.uniform(0.002, 0.004, size=n * ngr).astype(np.float32)
        zp = rng.uniform(6.0, 9.0, size=n * ngr).astype(np.float32)
        return p, sc, zp

    hq, hg, hd, hh = make(D7, D7), make(F7, D7), make(D7, F7), make(V7, D7)
    dev = torch.device("cuda")
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    kvs = B * H * max_seq * HD       # one layer's K (or V) cache, all sequences
    lw, ws = [], []
    plan, graph = None, None
    try:
        for _ in range(layers):
            q, k, v, o = [nimf.Weight.q4g(*hq, D7, D7, GS) for _ in range(4)]
            gate, up = [nimf.Weight.q4g(*hg, F7, D7, GS) for _ in range(2)]
            down = nimf.Weight.q4g(*hd, D7, F7, GS)
            ws += [q, k, v, o, gate, up, down]
            n1 = torch.rand(D7, device=dev) + 0.5
            n2 = torch.rand(D7, device=dev) + 0.5
            kc = torch.zeros(kvs, device=dev)
            vc = torch.zeros(kvs, device=dev)
            lw.append((q, k, v, o, gate, up, down, n1, n2, kc, vc))
        head = nimf.Weight.q4g(*hh, V7, D7, GS)
        ws.append(head)
        nf = torch.rand(D7, device=dev) + 0.5
        half = HD // 2
        inv = 1.0 / np.power(np.float32(10000.0), np.arange(half, dtype=np.float32) / np.float32(half))
        ang = np.arange(max_seq, dtype=np.float32)[:, None] * inv[None, :].astype(np.float32)
        cos_t = torch.from_numpy(np.cos(ang).astype(np.float32)).to(dev)
        sin_t = torch.from_numpy(np.sin(ang).astype(np.float32)).to(dev)
        table = torch.randn(V7, D7, device=dev) * 0.02
        ids = torch.from_numpy(rng.integers(0, V7, size=B * prompt).astype(np.int32)).to(dev)
        T, R = prompt, B * prompt            # tokens per sequence, prefill rows
        x = torch.empty(R, D7, device=dev)
        h = torch.empty(R, D7, device=dev)
        xn = torch.empty(R, D7, device=dev)
        qkv = [torch.empty(R, D7, device=dev) for _ in range(3)]
        att = torch.empty(R, D7, device=dev)
        ao = torch.empty(R, D7, device=dev)
        gu = [torch.empty(R, F7, device=dev) for _ in range(2)]
        act = torch.empty(R, F7, device=dev)
        dn = torch.empty(R, D7, device=dev)
        last = torch.empty(B, D7, device=dev)
        logits = torch.empty(B, V7, device=dev)
        tok = torch.zeros(B, dtype=torch.int32, device=dev)
        recent = torch.zeros(B, 64, dtype=torch.int32, device=dev)
        scale = float(np.float32(1.0) / np.sqrt(np.float32(HD)))
        eps = ctypes.c_float(1e-6)
        seq_kv = H * max_seq * HD * 4        # bytes of one sequence's cache in a layer

        def prefill(st):
            sp = ctypes.c_void_p(st)
            nimf.check(L.nimf_embedding_lookup_dev(P(table), V7, D7, P(ids), R, P(x), sp))
            nimf.check(L.nimf_rmsnorm_dev(P(x), P(lw[0][7]), R, D7, eps, P(xn), sp))
            for li, (q, k, v, o, gate, up, down, n1, n2, kc, vc) in enumerate(lw):
                nimf.Weight.matmul_group_dev([q, k, v], xn.data_ptr(), R,
                                             [t.data_ptr() for t in qkv], st)
                nimf.check(L.nimf_rope_dev(P(qkv[0]), B, T, H, HD, 0, P(cos_t), P(sin_t), max_seq, sp))
                nimf.check(L.nimf_rope_dev(P(qkv[1]), B, T, H, HD, 0, P(cos_t), P(sin_t), max_seq, sp))
                for b in range(B):
                    off = b * T * D7 * 4
                    nimf.check(L.nimf_attention_prefill_dev(
                        ctypes.c_void_p(qkv[0].data_ptr() + off), ctypes.c_void_p(qkv[1].data_ptr() + off),
                        ctypes.c_void_p(qkv[2].data_ptr() + off), ctypes.c_void_p(kc.data_ptr() + b * seq_kv),
                        ctypes.c_void_p(vc.data_ptr() + b * seq_kv), T, H, H, HD, max_seq, 0,
                        ctypes.c_float(scale), ctypes.c_void_p(att.data_ptr() + off), sp))
                o.matmul_dev(att.data_ptr(), R, ao.data_ptr(), st)
                nimf.check(L.nimf_add_rmsnorm_dev(P(x), P(ao), P(n2), R, D7, eps, P(h), P(xn), sp))
                nimf.Weight.matmul_group_dev([gate, up], xn.data_ptr(), R,
                                             [gu[0].data_ptr(), gu[1].data_ptr()], st)
                nimf.check(L.nimf_swiglu_dev(P(gu[0]), P(gu[1]), R * F7, P(act), sp))
                down.matmul_dev(act.data_ptr(), R, dn.data_ptr(), st)
                nxt = lw[li + 1][7] if li + 1 < len(lw) else nf
                nimf.check(L.nimf_add_rmsnorm_dev(P(h), P(dn), P(nxt), R, D7, eps, P(x), P(xn), sp))
            # lm_head and the greedy choice on each sequence's last prompt row
            last.copy_(xn.view(B, T, D7)[:, T - 1])
            head.matmul_dev(last.data_ptr(), B, logits.data_ptr(), st)
            nimf.check(L.nimf_greedy_sample_dev(P(logits), B, V7, P(recent), 0, ctypes.c_float(1.0),
                                                P(tok), sp))

        pos = torch.zeros(B, dtype=torch.int32, device=dev)
        st = torch.cuda.Stream()
        out_ids = torch.zeros(new_tokens, B, dtype=torch.int32, device=dev)
        if B == 1:
            lds = [{"wq": q, "wk": k, "wv": v, "wo": o, "wgate": gate, "wup": up, "wdown": down,
                    "attn_norm": n1.data_ptr(), "ffn_norm": n2.data_ptr(),
                    "k_cache": kc.data_ptr(), "v_cache": vc.data_ptr()}
                   for (q, k, v, o, gate, up, down, n1, n2, kc, vc) in lw]
            plan = nimf.DecodePlan(layers=lds, embedding=table.data_ptr(), final_norm=nf.data_ptr(),
                                   lm_head=head, rope_cos=cos_t.data_ptr(), rope_sin=sin_t.data_ptr(),
                                   d_model=D7, n_heads=H, n_kv_heads=H, head_dim=HD, ffn_dim=F7,
                                   vocab=V7, max_seq=max_seq, norm_eps=1e-6)

            def decode_step(sv):
                plan.step(tok.data_ptr(), tok.data_ptr(), pos.data_ptr(), logits.data_ptr(),
                          None, 0, 1.0, advance_pos=True, stream=sv)
        else:
            xd = torch.empty(B, D7, device=dev)
            hd_ = torch.empty(B, D7, device=dev)
            xnd = torch.empty(B, D7, device=dev)
            qd = [torch.empty(B, D7, device=dev) for _ in range(3)]
            attd = torch.empty(B, D7, device=dev)
            aod = torch.empty(B, D7, device=dev)
            gud = [torch.empty(B, F7, device=dev) for _ in range(2)]
            actd = torch.empty(B, F7, device=dev)
            dnd = torch.empty(B, D7, device=dev)

            def step_ops(sv):
                sp = ctypes.c_void_p(sv)
                nimf.check(L.nimf_embedding_lookup_dev(P(table), V7, D7, P(tok), B, P(xd), sp))
                nimf.check(L.nimf_rmsnorm_dev(P(xd), P(lw[0][7]), B, D7, eps, P(xnd), sp))
                for li, (q, k, v, o, gate, up, down, n1, n2, kc, vc) in enumerate(lw):
                    nimf.Weight.matmul_group_dev([q, k, v], xnd.data_ptr(), B,
                                                 [t.data_ptr() for t in qd], sv)
                    nimf.check(L.nimf_attention_decode_batch_dev(
                        P(qd[0]), P(qd[1]), P(qd[2]), P(kc), P(vc), B, H, H, HD, max_seq, P(pos),
                        P(cos_t), P(sin_t), ctypes.c_float(scale), 1 if li + 1 == len(lw) else 0,
                        P(attd), sp))
                    o.matmul_dev(attd.data_ptr(), B, aod.data_ptr(), sv)
                    nimf.check(L.nimf_add_rmsnorm_dev(P(xd), P(aod), P(n2), B, D7, eps, P(hd_), P(xnd), sp))
                    nimf.Weight.matmul_group_dev([gate, up], xnd.data_ptr(), B,
                                                 [gud[0].data_ptr(), gud[1].data_ptr()], sv)
                    nimf.check(L.nimf_swiglu_dev(P(gud[0]), P(gud[1]), B * F7, P(actd), sp))
                    down.matmul_dev(actd.data_ptr(), B, dnd.data_ptr(), sv)
                    nxt = lw[li + 1][7] if li + 1 < len(lw) else nf
                    nimf.check(L.nimf_add_rmsnorm_dev(P(hd_), P(dnd), P(nxt), B, D7, eps, P(xd),
                                                      P(xnd), sp))
                head.matmul_dev(xnd.data_ptr(), B, logits.data_ptr(), sv)
                nimf.check(L.nimf_greedy_sample_dev(P(logits), B, V7, P(recent), 0, ctypes.c_float(1.0),
                                                    P(tok), sp))

            # capture one step (the first replay set-up runs eagerly once)
            with torch.cuda.stream(st):
                pos.fill_(prompt)
                step_ops(st.cuda_stream)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=st):
                step_ops(st.cuda_stream)

            def decode_step(sv):
                graph.replay()

        def run():
            with torch.cuda.stream(st):
                pos.fill_(prompt)
                e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
                e0.record()
                prefill(st.cuda_stream)
                e1.record()
                for i in range(new_tokens):
                    decode_step(st.cuda_stream)
                    out_ids[i].copy_(tok)
                e2.record()
            torch.cuda.synchronize()
            nimf.check(L.nimf_sync())
            return e0.elapsed_time(e1), e1.elapsed_time(e2)

        run()                            # warm-up (first tcgen05 calls set up their buffers)
        pre_ms, dec_ms = run()
        assert pos.cpu().numpy().tolist() == [prompt + new_tokens] * B
        ids_out = out_ids.cpu().numpy()
        assert ((ids_out >= 0) & (ids_out < V7)).all()
    finally:
        if graph is not None:
            graph.reset()
        if plan is not None:
            plan.destroy()
        for w in ws:
            w.free()
    pre_flops = layers * prefill7b_flops(B * prompt)
    return {"batch": B, "prompt_tokens": prompt, "new_tokens": new_tokens,
            "prefill_ms": pre_ms, "prefill_tok_s": B * prompt / (pre_ms * 1e-3),
            "prefill_tflop_s": pre_flops / (pre_ms * 1e-3) / 1e12,
            "decode_ms": dec_ms, "decode_tok_s": B * new_tokens / (dec_ms * 1e-3),
            "generate_ms": pre_ms + dec_ms,
            "generate_tok_s": B * new_tokens / ((pre_ms + dec_ms) * 1e-3),
            "note": ("%d sequence(s): prefill of %d prompt tokens each through 32 layers (tcgen05 "
                     "GEMMs, causal prompt attention, glue) + lm_head on the last rows; decode: %d "
                     "greedy steps (%s), token chained on the device; prefill_tflop_s counts the "
                     "projections only" % (B, prompt, new_tokens,
                                           "one-launch plan" if B == 1 else
                                           "one captured per-op step per token"))}


def prefill7b_flops(tokens):
    """Multiply-add FLOPs of one 7B layer's projections for `tokens` rows."""
    return 2 * tokens * (4 * D7 * D7 + 3 * F7 * D7)


def run_prefill_7b(nimf, torch, steps, warmup, tokens=512, copies=4):
    """TFLOP/s of the 7B-shape int4 prefill projections (tensor-core GEMM).

    One step runs `copies` layers (distinct weight copies, 4 x 0.1 GB, more
    than L2) of grouped q/k/v, o, grouped gate/up and down on x[tokens, 4096],
    captured in one CUDA graph; weights are synthetic int4-g128 codes with
    group scales and zeros as in the decode measurement.  Attention, norms and
    the LM head are not on this path."""
    import numpy as np
    rng = np.random.default_rng(5)

    def make(n, k):
        ngr = k // GS
        p = rng.integers(0, 256, size=n * (k // 2), dtype=np.uint8)
        sc = rng.uniform(0.002, 0.004, size=n * ngr).astype(np.float32)
        zp = rng.uniform(6.0, 9.0, size=n * ngr).astype(np.float32)
        return p, sc, zp

    hq, hg, hd = make(D7, D7), make(F7, D7), make(D7, F7)
    layers = []
    for _ in range(copies):
        q, k, v, o = [nimf.Weight.q4g(*hq, D7, D7, GS) for _ in range(4)]
        gate, up = [nimf.Weight.q4g(*hg, F7, D7, GS) for _ in range(2)]
        down = nimf.Weight.q4g(*hd, D7, F7, GS)
        layers.append((q, k, v, o, gate, up, down))
    try:
        dev = torch.device("cuda")
        x = torch.randn(tokens, D7, device=dev)
        qkv = torch.empty(3, tokens, D7, device=dev)
        att = torch.empty(tokens, D7, device=dev)
        gu = torch.empty(2, tokens, F7, device=dev)
        dn = torch.empty(tokens, D7, device=dev)
        stream = torch.cuda.Stream()

        def step(st):
            for (q, k, v, o, gate, up, down) in layers:
                nimf.Weight.matmul_group_dev([q, k, v], x.data_ptr(), tokens,
                                             [qkv[i].data_ptr() for i in range(3)], st)
                o.matmul_dev(qkv[0].data_ptr(), tokens, att.data_ptr(), st)
                nimf.Weight.matmul_group_dev([gate, up], att.data_ptr(), tokens,
                                             [gu[0].data_ptr(), gu[1].data_ptr()], st)
                down.matmul_dev(gu[0].data_ptr(), tokens, dn.data_ptr(), st)

        L = nimf.lib()
        ms_mode = {}
        for mode in (1, 0):      # the exact-nibble GEMM, then the default (fp16 tiles)
            nimf.check(L.nimf_q4_prefill_mode(mode))
            ms_mode[mode] = graph_ms(torch, step, steps, warmup)
        # each projection alone (default GEMM), one layer copy per replay in turn
        (q, k, v, o, gate, up, down) = layers[0]
        proj = {
            "qkv": (lambda st: nimf.Weight.matmul_group_dev([q, k, v], x.data_ptr(), tokens,
                                                            [qkv[i].data_ptr() for i in range(3)], st),
                    2 * tokens * 3 * D7 * D7),
            "o": (lambda st: o.matmul_dev(qkv[0].data_ptr(), tokens, att.data_ptr(), st),
                  2 * tokens * D7 * D7),
            "gate_up": (lambda st: nimf.Weight.matmul_group_dev([gate, up], att.data_ptr(), tokens,
                                                                [gu[0].data_ptr(), gu[1].data_ptr()], st),
                        2 * tokens * 2 * F7 * D7),
            "down": (lambda st: down.matmul_dev(gu[0].data_ptr(), tokens, dn.data_ptr(), st),
                     2 * tokens * F7 * D7),
        }
        per_proj = {}
        for nm, (fn, fl) in proj.items():
            pms = graph_ms(torch, fn, steps, warmup)
            per_proj[nm] = {"us": pms * 1e3, "tflop_s": fl / (pms * 1e-3) / 1e12}
    finally:
        nimf.check(nimf.lib().nimf_q4_prefill_mode(0))
        for lw in layers:
            for w in lw:
                w.free()
    ms = ms_mode[0]
    per_layer = ms / copies
    tflops = prefill7b_flops(tokens) / (per_layer * 1e-3) / 1e12
    tflops_exact = prefill7b_flops(tokens) / (ms_mode[1] / copies * 1e-3) / 1e12
    pk, kind = peaks()
    peak = float(pk.get("bf16_tflops", 1590.0)) if kind == "measured" else 1590.0
    return {"tokens": tokens, "ms_per_layer": per_layer, "tflop_s": tflops,
            "frac_of_bf16_peak": tflops / peak, "bf16_peak_tflop_s": peak,
            "peak_source": kind,
            "exact_nibble_gemm_tflop_s": tflops_exact,
            "per_projection": per_proj,
            "matmul_tok_s_32_layers": tokens / (32 * per_layer * 1e-3),
            "launches_per_layer": 4 * 3,
            "note": ("default GEMM: int4 dequantised into fp16 tiles, one accumulator over K; "
                     "exact_nibble_gemm: nibbles exact in fp16 with an fp32 epilogue per group; "
                     "x prepared once per call (row scale + fp16 tiles) then one tcgen05 GEMM "
                     "launch per call; %d layer copies per step, %d timed steps" % (copies, steps))}


def graph_ms(torch, fn, steps, warmup):
    """Milliseconds per replay of fn() captured in a CUDA graph (CUDA events on
    the capturing stream, after warm-up replays)."""
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        fn(stream.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        fn(stream.cuda_stream)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    graph.reset()
    return ms


def run_formats(nimf, torch, steps):
    """The other quantised formats at their config shapes, on one GPU:
      * FP4 E2M1 block-16 and fp8 (CustomFloat(4,3) codes with a per-channel
        fp32 scale) GEMV/GEMM, K=8192, N=28672, M in {1, 16, 128, 512};
        W ~ N(0, 0.015) with 0.1% of entries x20, seed 2; two weight copies
        alternate so every call streams its weight from HBM (each > L2);
      * APF / CustomFloat encode and decode of 64M fp32 ~ N(0,1) with 1% x50
        outliers (seed 3) for E4M3, E5M10 and the auto-selected format, and
        the allocation-free auto-selection itself;
      * the int8 layer x[1,1024] . W[1024,1024] (per-tensor quant.nim scale).
    GB/s counts algorithmic bytes (the per-call byte counts of each format); TFLOP/s
    counts 2 M N K."""
    import ctypes
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle as O
    pk, how = peaks()
    hbm = float(pk["hbm_gbs"])
    out = {"peak_hbm_gbs": hbm, "peak_source": how}
    dev = torch.device("cuda")
    L = nimf.lib()

    # ---- config 3: FP4 / fp8 at K=8192, N=28672
    n3, k3 = 28672, 8192
    rng = np.random.default_rng(2)
    w = (rng.standard_normal((n3, k3), dtype=np.float32) * np.float32(0.015))
    idx = rng.choice(w.size, w.size // 1000, replace=False)
    w.flat[idx] *= 20
    ts = float(np.abs(w).max()) / (6 * 448)
    rs = (np.abs(w).max(axis=1) / 224.0).astype(np.float32)
    # quantise row blocks on parallel threads (the C oracle releases the GIL)
    from concurrent.futures import ThreadPoolExecutor
    nblk = 32
    bounds = [n3 * i // nblk for i in range(nblk + 1)]
    with ThreadPoolExecutor(max_workers=min(nblk, os.cpu_count() or 1)) as ex:
        q4 = list(ex.map(lambda i: O.quantize_fp4_block16(w[bounds[i]:bounds[i + 1]], ts),
                         range(nblk)))
        e8 = list(ex.map(lambda i: O.cf_encode(w[bounds[i]:bounds[i + 1]]
                                               / rs[bounds[i]:bounds[i + 1], None], 4, 3),
                         range(nblk)))
    p4 = np.concatenate([a for a, _ in q4])
    b4 = np.concatenate([b for _, b in q4])
    e8 = np.concatenate(e8)
    del w, q4
    cf43 = nimf.newCustomFloat(4, 3)
    fmts = {
        "fp4_e2m1_b16": (lambda: nimf.Weight.fp4(p4, b4, ts, n3, k3),
                         n3 * k3 // 2 + n3 * k3 // 16 + 4),
        "fp8_e4m3_rowscale": (lambda: nimf.Weight.cf(e8, cf43, n3, k3, row_scales=rs),
                              n3 * k3 + 4 * n3),
    }
    res3 = {}
    for name, (mk, wbytes) in fmts.items():
        ws = [mk(), mk()]
        try:
            for m in (1, 4, 8, 16, 17, 128, 512):
                x = torch.randn(m, k3, device=dev)
                y = torch.empty(m, n3, device=dev)

                def step(st):
                    for wt in ws:
                        wt.matmul_dev(x.data_ptr(), m, y.data_ptr(), st)

                ms = graph_ms(torch, step, max(3, steps if m <= 16 else steps // 8), 3) / len(ws)
                nbytes = wbytes + 4 * m * k3 + 4 * m * n3
                gbs = nbytes / (ms * 1e-3) / 1e9
                res3["%s_m%d" % (name, m)] = {
                    "us": ms * 1e3, "gb_s": gbs, "frac_of_hbm": gbs / hbm,
                    "tflop_s": 2.0 * m * n3 * k3 / (ms * 1e-3) / 1e12,
                    "algorithmic_bytes": nbytes}
        finally:
            for wt in ws:
                wt.free()
    del p4, b4, e8
    out["config3_k8192_n28672"] = res3

    # ---- config 4: APF encode / decode, 64M elements
    n4 = 1 << 26
    rng = np.random.default_rng(3)
    xa = rng.standard_normal(n4, dtype=np.float32)
    oi = rng.choice(n4, n4 // 100, replace=False)
    xa[oi] *= 50
    xd = torch.from_numpy(xa).to(dev)
    eb, mb = ctypes.c_int(), ctypes.c_int()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    nimf.check(L.nimf_cf_autoselect_dev_noalloc(ctypes.c_void_p(xd.data_ptr()), n4, None, 0,
                                                1e-3, 1, ctypes.byref(eb), ctypes.byref(mb), None))
    auto_s = time.perf_counter() - t0
    t0 = time.perf_counter()
    reps = 5
    for _ in range(reps):
        nimf.check(L.nimf_cf_autoselect_dev_noalloc(ctypes.c_void_p(xd.data_ptr()), n4, None, 0,
                                                    1e-3, 1, ctypes.byref(eb), ctypes.byref(mb),
                                                    None))
    auto_s = (time.perf_counter() - t0) / reps
    res4 = {"auto_selected": "e%dm%d" % (eb.value, mb.value),
            "autoselect_ms": auto_s * 1e3, "autoselect_gb_s": 4 * n4 / auto_s / 1e9}
    for e, m in ((4, 3), (5, 10), (eb.value, mb.value)):
        item = (1 + e + m + 7) // 8
        enc = torch.empty(n4 * item, dtype=torch.uint8, device=dev)
        dec = torch.empty(n4, dtype=torch.float32, device=dev)
        ep = ctypes.c_void_p(enc.data_ptr())

        def encode(st, e=e, m=m, ep=ep):
            nimf.check(L.nimf_cf_encode_dev(ctypes.c_void_p(xd.data_ptr()), n4, e, m, ep,
                                            ctypes.c_void_p(st)))

        def decode(st, e=e, m=m, ep=ep, item=item):
            nimf.check(L.nimf_cf_decode_dev(ep, n4 * item, e, m, ctypes.c_void_p(dec.data_ptr()),
                                            ctypes.c_void_p(st)))

        ms_e = graph_ms(torch, encode, max(3, steps // 4), 3)
        ms_d = graph_ms(torch, decode, max(3, steps // 4), 3)
        nb = n4 * (4 + item)
        res4["e%dm%d" % (e, m)] = {
            "item_bytes": item,
            "encode_gb_s": nb / (ms_e * 1e-3) / 1e9, "encode_frac_of_hbm": nb / (ms_e * 1e-3) / 1e9 / hbm,
            "decode_gb_s": nb / (ms_d * 1e-3) / 1e9, "decode_frac_of_hbm": nb / (ms_d * 1e-3) / 1e9 / hbm,
            "encode_us": ms_e * 1e3, "decode_us": ms_d * 1e3}
        del enc, dec
    del xd
    out["config4_apf_64m"] = res4

    # ---- config 1: int8 layer
    rng = np.random.default_rng(0)
    x1 = rng.standard_normal((1, 1024)).astype(np.float32)
    w1 = (rng.standard_normal((1024, 1024)) * 0.02).astype(np.float32)
    q1, s1 = O.quantize_int8(w1)
    h1 = nimf.Weight.i8(q1, s1, 1024, 1024)
    try:
        xd1 = torch.from_numpy(x1).to(dev)
        yd1 = torch.empty(1, 1024, device=dev)
        ms1 = graph_ms(torch, lambda st: h1.matmul_dev(xd1.data_ptr(), 1, yd1.data_ptr(), st),
                       max(3, steps), 3)
        h1.matmul(x1, 1)
        t0 = time.perf_counter()
        for _ in range(200):
            h1.matmul(x1, 1)
        e2e_us = (time.perf_counter() - t0) / 200 * 1e6
    finally:
        h1.free()
    out["config1_int8_1024"] = {"us_device": ms1 * 1e3, "us_e2e_host_buffers": e2e_us,
                                "gb_s": 1056772 / (ms1 * 1e-3) / 1e9,
                                "note": "launch-bound: 1 MB of weight"}
    return out


def run_ncu_case(name):
    """Small fixed workloads for ncu captures (one GPU, a few GB at most): each
    case runs three warm-up rounds and one final round, every round one launch
    per case, so `-s` / `-c` select the final round.
      decode_step: the whole-step 7B decode of run_decode_7b_full with 2 layers
          (graph replays: 2 warm-up, 2 timed);
      prefill: run_prefill_7b with one layer copy (both int4 GEMMs, each
          projection alone);
      decode_matmul: the 7B-shape int4 decode matmul stack of run_decode_7b at
          batch 1 (one eager step, then graph replays: 2 warm-up, 2 timed; 129
          GEMV launches per step);
      fw: an FP4 E2M1 block-16 weight and a one-byte CustomFloat(4,3) weight
          with per-row scales, both 28672 x 8192 (random codes): GEMV launches
          FP4 M=1, fp8 M=1, FP4 M=8, fp8 M=8, fp8 M=16, then the tcgen05 GEMM at
          fp8 M=17, FP4 M=128 and fp8 M=512."""
    import numpy as np
    import torch
    import nimf
    if name == "decode_step":
        nimf.init(0)
        run_decode_7b_full(nimf, torch, 2, 2, layers=2)
        print("ncu case %s done" % name)
        return
    if name == "decode_matmul":
        nimf.init(0)
        run_decode_7b(nimf, torch, 2, 2, batches=(1,))
        print("ncu case %s done" % name)
        return
    if name == "prefill":
        # one 7B layer's q/k/v, o, gate/up and down at 512 prompt rows: 3 warm-up
        # rounds and one final round on the fp16-tile GEMM (12 launches per
        # round: a row scale, an x preparation and a GEMM per call), then the
        # same on the exact-nibble GEMM
        nimf.init(0)
        run_prefill_7b(nimf, torch, 1, 3, copies=1)
        print("ncu case %s done" % name)
        return
    if name != "fw":
        raise SystemExit("unknown --ncu-case %s" % name)
    nimf.init(0)
    n3, k3 = 28672, 8192
    rng = np.random.default_rng(2)
    packed = rng.integers(0, 256, size=n3 * k3 // 2, dtype=np.uint8)
    bs = rng.integers(0x20, 0x48, size=n3 * k3 // 16, dtype=np.uint8)
    h4 = nimf.Weight.fp4(packed, bs, 1e-3, n3, k3)
    codes = rng.integers(0, 0x78, size=n3 * k3, dtype=np.uint8)  # no inf codes
    codes[(codes & 0x78) == 0] = 0                                # no exponent-0 mantissas
    h8 = nimf.Weight.cf(codes, nimf.newCustomFloat(4, 3), n3, k3,
                        row_scales=np.ones(n3, np.float32))
    cases = [(h4, 1), (h8, 1), (h4, 8), (h8, 8), (h8, 16), (h8, 17), (h4, 128), (h8, 512)]
    xs = {m: torch.randn(m, k3, device="cuda") for _, m in cases}
    ys = {m: torch.empty(m, n3, device="cuda") for _, m in cases}
    for _ in range(4):
        for h, m in cases:
            h.matmul_dev(xs[m].data_ptr(), m, ys[m].data_ptr())
        torch.cuda.synchronize()
    h4.free()
    h8.free()
    print("ncu case %s done" % name)


def compact_7b(decode, decode_full, prefill, formats, generate=None):
    """Short summaries of the 7B-shape and format measurements for the end of
    the JSON line (the full objects are printed on comment lines first).  A
    record that keeps only the last ~1,500 characters of the output still
    holds these, the most important last: formats, prefill, the matmul-only
    decode, the whole decode step, the generation."""
    r = lambda v, d=0: None if v is None else (round(float(v)) if d == 0 else round(float(v), d))
    out = {}
    if formats:
        f3 = formats.get("config3_k8192_n28672", {})
        out["fmt_gb_s"] = {k.replace("_rowscale", "").replace("_block16", ""): r(v.get("gb_s"))
                           for k, v in f3.items() if k.endswith(("_m1", "_m8"))}
        out["fmt_tflop_s"] = {k.replace("_rowscale", "").replace("_block16", ""): r(v.get("tflop_s"))
                              for k, v in f3.items() if k.endswith("_m512")}
    if prefill:
        out["prefill_7b"] = {"tflop_s": r(prefill.get("tflop_s")),
                             "exact_tflop_s": r(prefill.get("exact_nibble_gemm_tflop_s")),
                             "ms_layer": r(prefill.get("ms_per_layer"), 3)}
    if decode:
        d = {}
        if "error" in decode:
            d["error"] = decode["error"][:160]
        for k, v in decode.items():
            if isinstance(v, dict) and "tok_s" in v:
                d[k] = r(v["tok_s"])
        out["decode_7b_matmul_tok_s"] = d
    if decode_full:
        d = {}
        if "error" in decode_full:
            d["error"] = decode_full["error"][:160]
        for k, v in decode_full.items():
            if isinstance(v, dict) and "tok_s" in v:
                d[k] = r(v["tok_s"])
        out["decode_7b_step_tok_s"] = d
    if generate:
        out["generate_7b"] = {
            bk: ({"error": g["error"][:160]} if "error" in g else
                 {"prefill_ms": r(g["prefill_ms"], 1), "decode_tok_s": r(g["decode_tok_s"]),
                  "generate_tok_s": r(g["generate_tok_s"])})
            for bk, g in generate.items()}
    return out


def run_ours(args, rank, world, local_rank):
    import numpy as np
    import torch
    import torch.distributed as dist
    import nimf

    torch.cuda.set_device(local_rank)
    nimf.init(local_rank)
    R = args.copies
    n_total = N_PER_GPU * world
    r0, r1 = nimf.shard_rows(n_total, world, rank)   # N_PER_GPU rows per rank

    # synthetic weights: the same quantised matrix on every rank's shard rows
    w = (np.random.default_rng(0).standard_normal((N_PER_GPU, K)) * 0.02).astype(np.float32)
    p, s, z = nimf.quantize_int4_per_group(w, GS)
    if world > 1:
        p = np.tile(p, world)
        s = np.tile(s, world)
        z = np.tile(z, world)
    weights = [nimf.Weight.q4g(p, s, z, n_total, K, GS, rows=(r0, r1)) for _ in range(R)]
    x = torch.randn(M, K, device="cuda", dtype=torch.float32, generator=torch.Generator("cuda").manual_seed(1))
    ys = torch.empty(R, M, N_PER_GPU, device="cuda", dtype=torch.float32)
    gathered = torch.empty(world, R, M, N_PER_GPU, device="cuda", dtype=torch.float32) if world > 1 else None

    stream = torch.cuda.Stream()
    y_ptrs = [ys[r].data_ptr() for r in range(R)]
    import ctypes
    gid = None
    if world > 1:
        # the library's own communicator and a gather buffer shared by every
        # rank: the GEMV's merge warps store each output into every GPU
        lib_comm_init(nimf, rank, world)
        # waits between GPUs take microseconds; a short bound makes a broken
        # exchange fail within the warm-up instead of stretching every step
        nimf.check(nimf.lib().nimf_gather_set_timeout_ms(500))
        gid_c, base = ctypes.c_int64(), ctypes.c_void_p()
        nimf.check(nimf.lib().nimf_gather_create(R * M * n_total * 4, ctypes.byref(gid_c),
                                                 ctypes.byref(base)))
        gid = gid_c.value
        g_ptrs = (ctypes.c_void_p * R)(*[base.value + r * M * n_total * 4 for r in range(R)])
        g_handles = (ctypes.c_uint64 * R)(*[w.handle for w in weights])

    def step(st):
        if world > 1:
            # one launch: GEMVs of the 14 shards with the all-gather fused in
            nimf.check(nimf.lib().nimf_matmul_w_group_gather_dev(
                gid, g_handles, R, ctypes.c_void_p(x.data_ptr()), M, g_ptrs,
                ctypes.c_void_p(st.cuda_stream)))
        else:
            nimf.Weight.matmul_group_dev(weights, x.data_ptr(), M, y_ptrs, st.cuda_stream)

    def step_nccl(st):
        nimf.Weight.matmul_group_dev(weights, x.data_ptr(), M, y_ptrs, st.cuda_stream)
        dist.all_gather_into_tensor(gathered.view(-1), ys.view(-1))

    def step_single(st):
        for r in range(R):
            weights[r].matmul_dev(x.data_ptr(), M, ys[r].data_ptr(), st.cuda_stream)
        if world > 1:
            dist.all_gather_into_tensor(gathered.view(-1), ys.view(-1))

    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            step(stream)
            step_single(stream)
    torch.cuda.synchronize()
    if world > 1:
        # every rank learns whether any rank's warm-up exchange timed out
        bad = torch.tensor([float(nimf.lib().nimf_sync() != 0)], device="cuda")
        dist.all_reduce(bad, op=dist.ReduceOp.MAX)
        if bad.item() > 0:
            raise RuntimeError("bench: the fused all-gather's arrival wait expired in the warm-up")
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step(stream)
    graph1 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph1, stream=stream):
        step_single(stream)
    graph_nccl = None
    if world > 1:
        with torch.cuda.stream(stream):
            step_nccl(stream)
        torch.cuda.synchronize()
        graph_nccl = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_nccl, stream=stream):
            step_nccl(stream)
    torch.cuda.synchronize()

    # correctness spot check of one output against a host computation
    if rank == 0:
        y0 = ys[0].cpu().numpy()
        wd = weights[0].dequant()
        ref = wd.astype(np.float64) @ x.cpu().numpy().astype(np.float64).T
        err = float(np.max(np.abs(y0.ravel() - ref.ravel())) / np.max(np.abs(ref)))
        if not err <= 1e-3:
            raise RuntimeError("bench: GEMV output check failed (rel err %.3g)" % err)

    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.2)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        graph.replay()
    end.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    bytes_step = R * algo_bytes(N_PER_GPU, K, M, GS) * world
    value = bytes_step / (ms_per_step * 1e-3) / 1e9

    # the same GEMVs as one launch each (PDL-chained in a graph)
    for _ in range(args.warmup):
        graph1.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s1, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s1.record()
    for _ in range(args.steps):
        graph1.replay()
    e1.record()
    torch.cuda.synchronize()
    ms1 = s1.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms1], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms1 = float(t.item())
    single = {"value": bytes_step / (ms1 / args.steps * 1e-3) / 1e9, "unit": "GB/s",
              "us_per_gemv": ms1 * 1e3 / (args.steps * R),
              "note": "one launch per GEMV, PDL-chained in a CUDA graph"}
    nccl_cmp = None
    if world > 1:
        # the same step with the grouped GEMV followed by an NCCL all-gather
        for _ in range(args.warmup):
            graph_nccl.replay()
        torch.cuda.synchronize()
        dist.barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for _ in range(args.steps):
            graph_nccl.replay()
        e2.record()
        torch.cuda.synchronize()
        t = torch.tensor([s2.elapsed_time(e2)], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms2 = float(t.item()) / args.steps
        nccl_cmp = {"value": bytes_step / (ms2 * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms2,
                    "note": "grouped GEMV launch, then an NCCL all_gather_into_tensor of the "
                            "14 output slices"}
        bad = torch.tensor([float(nimf.lib().nimf_sync() != 0)], device="cuda")
        dist.all_reduce(bad, op=dist.ReduceOp.MAX)
        if bad.item() > 0:
            raise RuntimeError("bench: a gathering GEMV's arrival wait expired on some rank")

    # kernel-level roofline: the grouped GEMV launch (one per step)
    pk, how = peaks()
    per_launch_bytes = R * algo_bytes(N_PER_GPU, K, M, GS)
    launch_s = ms * 1e-3 / args.steps
    achieved = per_launch_bytes / launch_s / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / pk["hbm_gbs"], "traffic": profile_traffic(),
                "peak_source": how, "kernel": "q4g_gemv_kernel<1,2,%d> (grouped, %d weights)" % (1 if M == 1 else 0, R),
                "algorithmic_bytes_per_launch": per_launch_bytes,
                "note": "launch duration = timed region / launches, CUDA events"}

    # end to end through the C ABI with host buffers (pinned), per step R calls
    xh = torch.randn(M, K, dtype=torch.float32).pin_memory()
    yh = torch.empty(R, M, N_PER_GPU, dtype=torch.float32).pin_memory()
    L = nimf.lib()
    import ctypes
    xp = ctypes.c_void_p(xh.data_ptr())
    yps = [ctypes.c_void_p(yh[r].data_ptr()) for r in range(R)]

    hs = (ctypes.c_uint64 * R)(*[w.handle for w in weights])
    ypa = (ctypes.c_void_p * R)(*[yh[r].data_ptr() for r in range(R)])

    def e2e_step():
        nimf.check(L.nimf_matmul_w_group(hs, R, xp, M, ypa))

    for _ in range(max(1, args.warmup)):
        e2e_step()
    e2e_steps = max(5, min(args.steps, 200))
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_s], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = {"value": bytes_step / e2e_s / 1e9, "unit": "GB/s",
           "h2d_bytes_per_step": M * K * 4, "d2h_bytes_per_step": R * M * N_PER_GPU * 4,
           "api": "nimf_matmul_w_group (host buffers, blocking; x copied once for the group, "
                  "the outputs in one copy because their host buffers are contiguous)",
           "note": "per-rank shard outputs; no host all-gather" if world > 1 else ""}

    cpu = None
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        xs = np.random.default_rng(1).standard_normal((M, K)).astype(np.float32)
        rate, desc = cpu_reference_gemv_rate(p[: N_PER_GPU * K // 2], s, z, xs, args.cpu_seconds)
        cpu = {"value": rate, "unit": "GB/s", "cores": 1, "kind": "port", "sample": desc}

    graph.reset()
    graph1.reset()
    if graph_nccl is not None:
        graph_nccl.reset()
    if gid is not None:
        torch.cuda.synchronize()
        nimf.check(nimf.lib().nimf_gather_destroy(gid))
    decode = None
    if args.decode_steps > 0:
        if world == 1:
            decode = run_decode_7b(nimf, torch, args.decode_steps, max(3, args.warmup // 4))
        else:
            # every rank runs the same steps; an error raised on all of them is
            # reported in the line instead of dropping the GEMV measurement
            try:
                decode = run_decode_7b(nimf, torch, args.decode_steps, max(3, args.warmup // 4),
                                       rank, world)
                # the same step with NCCL all-gathers, for comparison
                nccl = run_decode_7b(nimf, torch, args.decode_steps, max(3, args.warmup // 4),
                                     rank, world, exchange="nccl", batches=(1,))
                decode["nccl_batch1"] = nccl["batch1"]
            except Exception as e:  # noqa: BLE001
                decode = {"error": "%s: %s" % (type(e).__name__, e)}
    decode_full = None
    if world == 1 and args.decode_steps > 0:
        decode_full = run_decode_7b_full(nimf, torch, max(5, args.decode_steps // 2), 3)
    elif args.decode_steps > 0:
        try:
            lib_comm_init(nimf, rank, world)
            decode_full = run_decode_7b_sharded(nimf, torch, max(5, args.decode_steps // 2), 3,
                                                rank, world)
        except Exception as e:  # noqa: BLE001
            decode_full = {"error": "%s: %s" % (type(e).__name__, e)}
    prefill = None
    if world == 1 and args.prefill_steps > 0:
        prefill = run_prefill_7b(nimf, torch, args.prefill_steps, 3)
    generate = None
    if world == 1 and args.decode_steps > 0:
        generate = {}
        for gb in (1, 8):
            try:
                generate["batch%d" % gb] = run_generate_7b(nimf, torch, batch=gb)
            except Exception as e:  # noqa: BLE001
                generate["batch%d" % gb] = {"error": "%s: %s" % (type(e).__name__, e)}
    formats = None
    if world == 1 and args.format_steps > 0:
        formats = run_formats(nimf, torch, args.format_steps)
    if rank == 0:
        # the detailed objects go on comment lines first; the one JSON line
        # ends with compact 7B summaries, so a record that keeps only the end
        # of the output still holds them
        detail = {"decode_7b": decode, "decode_7b_full_step": decode_full,
                  "prefill_7b": prefill, "generate_7b": generate, "formats": formats,
                  "single_launch": single}
        for key, val in detail.items():
            if val is not None:
                print("# %s %s" % (key, json.dumps(val)), flush=True)
        line = {"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "u4 weights, f32 activations/accumulate", "data": "synthetic",
                "config": workload_config(world, R),
                "roofline": roofline, "e2e": e2e,
                "gpu_launches": args.steps,
                "clocks": clocks}
        if cpu is not None:
            line["cpu_baseline"] = cpu
        line["pct_of_hbm_peak"] = value / world / pk["hbm_gbs"]
        line["single_launch_gb_s"] = single["value"]
        if nccl_cmp is not None:
            line["nccl_allgather_gb_s"] = nccl_cmp["value"]
            line["exchange"] = ("all-gather fused into the GEMV: merge warps store every output "
                                "into every GPU over NVLink, one arrival per rank per launch")
        line.update(compact_7b(decode, decode_full, prefill, formats, generate))
        print(json.dumps(line), flush=True)
    for wt in weights:
        wt.free()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--copies", type=int, default=14)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--decode-steps", type=int, default=200,
                    help="timed steps of the 7B-shape decode measurement (0: skip)")
    ap.add_argument("--prefill-steps", type=int, default=20,
                    help="timed steps of the 7B-shape prefill measurement (0: skip)")
    ap.add_argument("--format-steps", type=int, default=40,
                    help="timed steps of the FP4/fp8/APF/int8 measurements (0: skip)")
    ap.add_argument("--ncu-case", default=None,
                    help="run one fixed workload for an ncu capture and exit (fw, decode_step, decode_matmul, prefill)")
    args = ap.parse_args()
    if args.ncu_case:
        run_ncu_case(args.ncu_case)
        return
    args.warmup = max(3, args.warmup)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
