"""The library's vectorised host quantiser (nimf.quantize_int4_per_group)
reproduces the reference exporter bit-for-bit (golden fixtures made by
export_to_nimq.py:363-395) and agrees with the oracle on larger inputs."""
import glob
import os

import numpy as np
import pytest

import nimf
import pyoracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "q4g_*.npz"))),
                         ids=lambda p: os.path.basename(p))
def test_matches_exporter_fixtures(path):
    d = np.load(path)
    p, s, z = nimf.quantize_int4_per_group(d["w"], int(d["group_size"]))
    assert np.array_equal(p, d["packed"])
    assert np.array_equal(s.view(np.uint32), d["scales"].view(np.uint32))
    assert np.array_equal(z.view(np.uint32), d["zeros"].view(np.uint32))


@pytest.mark.parametrize("rows,cols,gs", [(64, 4096, 128), (9, 1001, 128), (3, 77, 32)])
def test_matches_oracle(rows, cols, gs):
    w = (np.random.default_rng(rows).standard_normal((rows, cols)) * 0.02).astype(np.float32)
    w[0, :gs] = 0.1
    a = nimf.quantize_int4_per_group(w, gs)
    b = O.quantize_int4_asym_per_group(w, gs)
    for u, v in zip(a, b):
        assert np.array_equal(np.asarray(u).view(np.uint8), np.asarray(v).view(np.uint8))
