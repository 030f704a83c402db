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


def test_core_module_staged_report_and_checksums(core, cuda):
    """The module's tm_stage_input_async and block_checksums: a report from a
    host buffer staged ahead of the call scores exactly as the report from
    device memory, and a block's checksum, computed where the block lives,
    is unchanged by an evict to the DRAM tier and the promote back, with tier
    codes 0 (HBM) and 1 (DRAM)."""
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(5)
    R, Hq, Hkv, T, tpb = 2, 4, 2, 128, 64
    n = R * Hkv * (T // tpb)
    probs = torch.softmax(torch.randn(R, Hq, T, generator=g, device="cuda") * 2, -1)
    host = probs.cpu().pin_memory()
    rid = torch.arange(n, dtype=torch.int32, device="cuda")
    scores = []
    for staged in (False, True):
        tm = core.tm_create(tracker_cap=64, cooldown_sec=0.0)
        try:
            for i in range(n):
                core.tm_register_block_id(tm, i)
            src = probs.data_ptr()
            if staged:
                assert core.tm_stage_input_async(tm, host.data_ptr(), host.numel() * 4) == core.OK
                src = host.data_ptr()
            assert core.tm_report_attn_probs(tm, src, R, Hq, Hkv, T, tpb, rid.data_ptr()) == core.OK
            core.tm_step_done(tm)
            core.tm_schedule_once(tm)                   # classifies: the scores are its hotness
            scores.append(np.array([core.tm_get_block_score(tm, i) for i in range(n)], np.float32))
        finally:
            core.tm_destroy(tm)
    assert (scores[0] > 0).all()
    assert np.array_equal(scores[0].view(np.uint32), scores[1].view(np.uint32))

    cfg = core.Config()
    cfg.gpu_pool_bytes = 64 * 32768
    cfg.dram_pool_bytes = 64 * 32768
    assert core.init(cfg) == core.OK
    try:
        ctx = core.request_create(7, 2, 2)                  # 2 layers x 2 KV heads
        for layer in range(2):
            kv = torch.randn(2, 2, 100, 128, generator=g, device="cuda").half()
            assert core.prefill(ctx, layer, kv[0].data_ptr(), kv[1].data_ptr(), 100) == core.OK
        ids = torch.empty(8, dtype=torch.int32, device="cuda")   # [layer][head][block]
        assert core.block_id_table([ctx], 100, ids.data_ptr()) == core.OK
        out = torch.empty(8, dtype=torch.int64, device="cuda")
        tiers = torch.empty(8, dtype=torch.uint8, device="cuda")

        def sums():
            assert core.block_checksums(ids.data_ptr(), 8, out.data_ptr(),
                                        tiers.data_ptr()) == core.OK
            torch.cuda.synchronize()
            return out.cpu().numpy().copy(), tiers.cpu().numpy().copy()

        before, t0 = sums()
        assert (t0 == 0).all() and (before != 0).all()
        assert core.evict_to_dram(ctx, 0, 1, 1) == core.OK    # layer 0, head 1, block 1: entry 3
        mid, t1 = sums()
        assert t1[3] == 1 and (np.delete(t1, 3) == 0).all()
        assert np.array_equal(mid, before)
        assert core.promote_to_gpu(ctx, 0, 1, 1) == core.OK
        after, t2 = sums()
        assert (t2 == 0).all() and np.array_equal(after, before)
        assert core.request_destroy(ctx) == core.OK
    finally:
        assert core.shutdown() == core.OK
