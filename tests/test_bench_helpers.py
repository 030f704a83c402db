"""The bench's JSON-building helpers on synthetic figures (no GPU): the pack
roofline object (algorithmic bytes per launch over the mean launch time,
traffic scaled from the full-chunk ncu figure), the first-chunk object, the
peaks file, the host-thread count, and the command-line surface."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_pack_roofline_object():
    full = bench.PACK_FULL_LAUNCH_BYTES
    r = bench.pack_roofline([0.1] * 14, 14 * full, 6545.6, "measured")
    assert r["bound"] == "hbm" and r["unit"] == "GB/s" and r["launches"] == 14
    assert r["bytes_per_launch"] == full
    assert r["achieved"] == pytest.approx(full / 1e-4 / 1e9, rel=1e-4)
    assert r["frac"] == pytest.approx(r["achieved"] / 6545.6, rel=1e-3)
    assert r["traffic"] == round(bench.PACK_TRAFFIC_PER_FULL_LAUNCH)
    half = bench.pack_roofline([0.05, 0.05], full, 6545.6, "measured")
    assert half["traffic"] == round(bench.PACK_TRAFFIC_PER_FULL_LAUNCH / 2)
    assert bench.pack_roofline([], 0, 6545.6, "measured") is None


def test_first_chunk_object():
    full = bench.PACK_FULL_LAUNCH_BYTES
    fc = bench.pack_first_chunk([0.09, 0.12, 0.12], 3 * full, 3, 6545.6)
    assert fc["ms"] == 0.09 and fc["later_chunks_ms_mean"] == pytest.approx(0.12)
    assert fc["achieved_gbs"] == pytest.approx(full / 0.09 / 1e6, rel=1e-3)
    assert fc["frac"] == pytest.approx(fc["achieved_gbs"] / 6545.6, rel=1e-3)
    assert bench.pack_first_chunk([0.1], full, 1, 6545.6) is None


def test_peaks_and_threads():
    peak, kind = bench.peaks()
    assert peak > 1000 and kind in ("measured", "fallback")
    assert bench.host_threads() >= 1


def test_command_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--help"],
                         capture_output=True, text=True, timeout=120)
    assert out.returncode == 0
    for flag in ("--gpus", "--steps", "--warmup", "--impl"):
        assert flag in out.stdout


def test_sharded_pick_rule_matches_oracle(oracle_mod):
    """The sharded bench's check of the ranks' global picks (numpy: keys of
    the hotness, stable sort by (key, global index)) is the oracle's coldest-k
    over the same concatenated arrays, ties included (values on a 1/16 grid,
    -0.0 beside +0.0)."""
    import numpy as np

    import bench
    rng = np.random.default_rng(7)
    n = 50000
    hot = (rng.integers(-8, 40, n) / 16).astype(np.float32)
    hot[rng.random(n) < 0.01] = -0.0
    elig = rng.random(n) < 0.8
    assert np.array_equal(bench.orderable_u32(hot), oracle_mod.orderable(hot))
    for k in (1, 777, int(elig.sum()) // 2, int(elig.sum())):
        idx = np.nonzero(elig)[0]
        order = np.lexsort((idx, bench.orderable_u32(hot[idx])))[:k]
        got = np.sort(idx[order])
        want = oracle_mod.select_coldest(hot, elig.astype(np.uint8), k).astype(np.int64)
        assert np.array_equal(got, want)
