"""The orchkv_core module as the reference's Python managers use it
(python/orchkv/fast_kvcache_manager.py:106-341, kvcache_manager.py:317-427):
golden op sequences recorded from the reference are replayed through the
pybind names and must give the recorded scores, heats and counters exactly."""
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")


@pytest.fixture(scope="module")
def core(cuda):
    import orchkv_b200
    return orchkv_b200.core()


def _fixtures():
    return sorted(f for f in os.listdir(GOLDEN) if f.startswith("sched_") and f.endswith(".json"))


def f32bits(x):
    return int(np.array([x], np.float32).view(np.uint32)[0])


@pytest.mark.parametrize("name", _fixtures())
def test_core_module_replay(core, name):
    with open(os.path.join(GOLDEN, name)) as fh:
        fx = json.load(fh)
    cfg = dict(fx["config"])
    tm = core.tm_create(cooldown_sec=0.0, **cfg)
    try:
        for op in fx["ops"]:
            k = op[0]
            if k == "reg":
                core.tm_register_block_id(tm, op[1], op[2], op[3])
            elif k == "rep":
                core.tm_report_attn(tm, op[1], op[2])
            elif k == "step":
                core.tm_step_done(tm)
            elif k == "usage":
                core.tm_set_usage(tm, op[1], op[2])
            elif k == "sched":
                core.tm_schedule_once(tm)
            elif k == "tier":
                core.tm_set_block_tier(tm, op[1], op[2])
            elif k == "policy":
                core.tm_set_policy(tm, op[1], op[2], op[3])
        exp = fx["expect"]
        ids = fx["ids"]
        # per-block getters the managers call (fast_kvcache_manager.py:316)
        got_hot = [f32bits(core.tm_get_block_score(tm, i)) for i in ids]
        got_heat = [core.tm_get_block_heat(tm, i) for i in ids]
        assert got_hot == exp["hot"]
        assert got_heat == exp["heat"]
        st = core.tm_get_stats(tm)
        for key in ["schedule_cycles", "prefetches_dispatched", "n_hot", "n_warm", "n_cold",
                    "threshold_adj_up", "threshold_adj_down"]:
            assert st[key] == exp["stat_" + key], key
        assert f32bits(st["threshold_hot"]) == exp["stat_threshold_hot"]
        assert f32bits(st["threshold_warm"]) == exp["stat_threshold_warm"]
        assert set(st) == {"schedule_cycles", "gpu_demotes", "dram_demotes",
                           "prefetches_dispatched", "gpu_used_ratio", "dram_used_ratio",
                           "blocks_migrated", "migration_errors", "prefetch_hits",
                           "prefetch_wasted", "prefetch_hit_rate", "n_hot", "n_warm", "n_cold",
                           "threshold_adj_up", "threshold_adj_down", "threshold_hot",
                           "threshold_warm"}
    finally:
        core.tm_destroy(tm)


def test_core_module_errors_and_data_plane(core, cuda):
    # tm_create raises RuntimeError on failure, like the reference binding
    with pytest.raises(RuntimeError):
        core.tm_create(tracker_cap=0)
    cfg = core.Config()
    cfg.gpu_pool_bytes = 64 * 32768
    cfg.dram_pool_bytes = 64 * 32768
    assert core.init(cfg) == core.OK
    assert core.init(cfg) == -10               # ERR_ALREADY
    try:
        ctx = core.request_create(1, 2, 2)
        k = cuda.randn(2, 100, 128, dtype=cuda.float16, device="cuda")
        assert core.prefill(ctx, 0, k.data_ptr(), k.data_ptr(), 100) == core.OK
        rc, kp, vp = core.get_kv_block(ctx, 0, 1, 1)
        assert rc == core.OK and vp - kp == 16384
        assert core.evict_to_dram(ctx, 0, 1, 1) == core.OK
        assert core.get_stats()["dram_slabs_used"] == 1
        rc, kp2, _ = core.get_kv_block(ctx, 0, 1, 1)      # promotes on access
        assert rc == core.OK and kp2 != 0
        assert core.get_stats()["dram_slabs_used"] == 0
        assert core.evict_to_dram(ctx, 0, 0, 9) == core.ERR_NOT_FOUND
        tok = cuda.randn(2, 128, dtype=cuda.float16, device="cuda")
        assert core.append_token(ctx, 0, tok.data_ptr(), tok.data_ptr()) == core.OK
        s = core.get_stats()
        assert s["gpu_slabs_used"] == 4 and s["transfers_d2h"] == 1
        assert core.request_destroy(ctx) == core.OK
    finally:
        assert core.shutdown() == core.OK
