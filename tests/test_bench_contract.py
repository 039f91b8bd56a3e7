"""bench.py's roofline numerators against the algorithmic work of the measured configurations: bytes one decode call
must move (every cached cell once, plus q and out) and the exact causal flops of the prefill chunk, as the
configurations define them (c2a 276.8 MB of cache, c4 411.0 MB, c1 138.4 MB, c2b 1107.3 MB; c3 5.785 TFLOP)."""
import json
import os

import pytest

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
QOUT = lambda w: 2 * w["qlen"] * bench.NQ * bench.HS * 2  # q in + out, bf16, per request


@pytest.mark.parametrize("name,cache_mb", [("c2a", 276.8), ("c4", 411.0), ("c1", 138.4), ("c2b", 1107.3)])
def test_decode_bytes(name, cache_mb):
    w = bench.WORKLOADS[name]
    b = bench.algorithmic_bytes(w)
    cache = b - w["seqs"] * QOUT(w)
    assert abs(cache / 1e6 - cache_mb) < 0.1, cache
    assert cache == w["seqs"] * w["ctx"] * bench.NKV * bench.CELL[w["fmt"]]


def test_prefill_flops():
    w = bench.WORKLOADS["c3"]
    f = bench.prefill_flops(w)
    # sum over the chunk's 1024 queries of the keys each sees (229,376 cached + its causal prefix), QK and PV
    ctx0 = w["ctx"] - w["qlen"]
    assert f == sum(4 * bench.NQ * bench.HS * (ctx0 + i + 1) for i in range(w["qlen"]))
    assert abs(f / 1e12 - 5.785) < 1e-3


def test_cells_and_peaks():
    assert bench.CELL == {"int4": 264, "k8v4": 392}
    with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
        hbm = float(json.load(fh)["hbm_gbs"])
    assert bench.peaks() == (hbm, "measured")
