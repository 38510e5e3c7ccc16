"""Generate the golden fixtures under tests/golden/ by running the reference's
own Python code (export_to_nimq.py of the Nimformer project).

Usage:  python tests/golden/gen_golden.py --reference <path of the Nimformer source tree>
        (or set NIMF_REFERENCE to that path)

The reference is imported from its source tree (read-only); nothing is copied
from it.  Each fixture stores seeded inputs and the reference's outputs:

  q4g_*.npz     export_to_nimq.py:363-395 quantize_int4_asymmetric_per_group
  i8_*.npz      export_to_nimq.py:353-360 quantize_int8_vectorized
  gptq_*.npz    export_to_nimq.py:219-254 dequantize_gptq_linear
  nimq_small.bin  export_to_nimq.py:580-605 write_string / write_quant_tensor
                  stream with the header export_to_nimq.py:679-682 writes

The numpy version that produced them is recorded in meta.json.
"""
import argparse
import io
import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(path):
    sys.path.insert(0, path)
    import export_to_nimq  # noqa: E402  (reference module, prints a device banner)
    return export_to_nimq


def q4g_cases():
    """(name, W, group_size) cases; W float32 [rows, cols]."""
    rng = np.random.default_rng(0)
    cases = []
    cases.append(("q4g_basic", (rng.standard_normal((8, 256)) * 0.02).astype(np.float32), 128))
    cases.append(("q4g_ragged", (rng.standard_normal((5, 300)) * 0.02).astype(np.float32), 128))
    cases.append(("q4g_oddcols", (rng.standard_normal((3, 129)) * 0.02).astype(np.float32), 128))
    w = (rng.standard_normal((4, 256)) * 0.02).astype(np.float32)
    w[1, :128] = 0.0          # constant group -> scale 1.0, zero 0.0
    w[2, 128:] = 0.37         # constant non-zero group
    cases.append(("q4g_constant", w, 128))
    # exact half-way points on the quantisation grid: 0, 1/15, ..., with
    # midpoints between codes so np.round's half-to-even rule is exercised
    base = np.linspace(-1.0, 1.0, 31, dtype=np.float32)
    w = np.tile(base, (2, 5))[:, :128].astype(np.float32)
    cases.append(("q4g_ties", w, 128))
    w = (rng.standard_normal((16, 512)) * 0.015).astype(np.float32)
    idx = rng.choice(w.size, round(0.001 * w.size) + 4, replace=False)
    w.flat[idx] *= 20.0
    cases.append(("q4g_outliers", w, 128))
    cases.append(("q4g_gs32", (rng.standard_normal((4, 192)) * 0.02).astype(np.float32), 32))
    cases.append(("q4g_gs64", (rng.standard_normal((4, 192)) * 0.02).astype(np.float32), 64))
    cases.append(("q4g_smallk", (rng.standard_normal((6, 40)) * 0.02).astype(np.float32), 40))
    # a slice of the K=4096 decode GEMV weights, W ~ N(0, 0.02), seed 0
    w = (np.random.default_rng(0).standard_normal((8, 4096)) * 0.02).astype(np.float32)
    cases.append(("q4g_k4096", w, 128))
    return cases


def i8_cases():
    rng = np.random.default_rng(1)
    cases = []
    cases.append(("i8_basic", (rng.standard_normal((16, 1024)) * 0.02).astype(np.float32)))
    cases.append(("i8_zeros", np.zeros((4, 16), dtype=np.float32)))
    w = np.array([[-1.0, 1.0, 0.5, -0.5, 0.25, 127.0 / 254.0, 0.0, -0.0]], dtype=np.float32)
    cases.append(("i8_ties", w))
    return cases


def gptq_case(rng, in_features, out_features, group, act_order):
    n_groups = in_features // group
    qweight = rng.integers(0, 2**32, size=(in_features // 8, out_features), dtype=np.uint64)
    qweight = qweight.astype(np.uint32).view(np.int32)
    qzeros = rng.integers(0, 2**32, size=(n_groups, out_features // 8), dtype=np.uint64)
    qzeros = qzeros.astype(np.uint32).view(np.int32)
    scales = (rng.random((n_groups, out_features)) * 0.01 + 1e-4).astype(np.float16)
    g_idx = np.arange(in_features) // group
    if act_order:
        g_idx = rng.permutation(g_idx)
    return qweight, qzeros, scales, g_idx.astype(np.int32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("NIMF_REFERENCE"),
                    help="the Nimformer source tree (default: $NIMF_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set NIMF_REFERENCE")
    ref = load_reference(args.reference)

    for name, w, gs in q4g_cases():
        packed, scales, zeros = ref.quantize_int4_asymmetric_per_group(w, gs)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), w=w, group_size=np.int64(gs),
                            packed=packed, scales=scales, zeros=zeros)

    for name, w in i8_cases():
        q, sc = ref.quantize_int8_vectorized(w)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), w=w, q=q,
                            scale=np.float64(sc))

    rng = np.random.default_rng(2)
    for name, (kin, kout, grp, act) in {"gptq_basic": (256, 64, 128, False),
                                        "gptq_actorder": (256, 32, 64, True)}.items():
        qw, qz, sc, gi = gptq_case(rng, kin, kout, grp, act)
        w = ref.dequantize_gptq_linear(qw, qz, sc, gi)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), qweight=qw, qzeros=qz,
                            scales=sc, g_idx=gi, weight=w)

    # A small .nimq stream written by the exporter's own writer functions.
    rng = np.random.default_rng(3)
    buf = io.BytesIO()
    arch = [256, 2, 4, 64, 512]
    tensors = [
        ("tok_embeddings.weight", (rng.standard_normal((16, 64)) * 0.02).astype(np.float32), ref.QK_FP32_RAW),
        ("layers.0.attention.wq.weight", (rng.standard_normal((64, 256)) * 0.02).astype(np.float32), ref.QK_INT4_ASYMMETRIC),
        ("layers.0.feed_forward.w1.weight", (rng.standard_normal((32, 64)) * 0.02).astype(np.float32), ref.QK_INT8),
        ("norm.weight", np.ones(64, dtype=np.float32), ref.QK_FP32_RAW),
    ]
    ref.write_string(buf, "NIMQ2")
    for v in arch:
        buf.write(struct.pack('<i', v))
    buf.write(struct.pack('<i', len(tensors)))
    for name, arr, kind in tensors:
        ref.write_string(buf, name)
        ref.write_quant_tensor(buf, name, arr, kind)
    with open(os.path.join(HERE, "nimq_small.bin"), "wb") as f:
        f.write(buf.getvalue())
    np.savez_compressed(os.path.join(HERE, "nimq_small_src.npz"),
                        **{n.replace(".", "_"): a for n, a, _ in tensors})

    meta = {"numpy": np.__version__, "generator": "tests/golden/gen_golden.py",
            "reference_module": "export_to_nimq.py"}
    with open(os.path.join(HERE, "meta.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
