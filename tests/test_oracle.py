"""The oracle restatement pinned against the reference: its own known-answer
tests (values cited by file:line), the committed golden fixtures, and — where
the reference was compiled into oracle/_ref — live random cross-checks."""
import json
import math
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")


def f32(x):
    return float(np.float32(x))


# ---- known answers from the reference's test suite ----------------------------

def test_ema_blend(oracle_mod):
    # test/test_attention_tracker.c:118-150 (lambda 0.8: 0.2 then 0.26)
    s = oracle_mod.OracleSched(capacity=256, ema_lambda=0.8)
    s.register(1)
    s.update(1, 1.0)
    s.step_done()
    st = s.state()
    assert abs(st["ema"][1] - 0.2) < 1e-5 and st["hits"][1] == 1 and st["sum"][1] == 0
    s.update(1, 0.5)
    s.step_done()
    st = s.state()
    assert abs(st["ema"][1] - 0.26) < 1e-5 and st["hits"][1] == 2 and s.step == 2


def test_idle_decay(oracle_mod):
    # test/test_attention_tracker.c:152-181 (0.5 -> 0.25 -> 0.125)
    s = oracle_mod.OracleSched(capacity=256, ema_lambda=0.5)
    s.register(1)
    s.update(1, 1.0)
    s.step_done()
    s.step_done()
    assert abs(s.state()["ema"][1] - 0.25) < 1e-5
    assert s.state()["hits"][1] == 1
    s.step_done()
    assert abs(s.state()["ema"][1] - 0.125) < 1e-5


def test_update_sum_max_and_inactive(oracle_mod):
    # test/test_attention_tracker.c:83-116
    s = oracle_mod.OracleSched(capacity=256)
    s.register(42)
    s.update(42, 0.5)
    s.update(42, 0.3)
    st = s.state()
    assert abs(st["sum"][42] - 0.8) < 1e-5 and abs(st["max"][42] - 0.5) < 1e-5
    assert st["last"][42] == 0
    s.update(99, 1.0)                       # inactive slot ignores reports
    assert s.state()["t_active"][99] == 0 and s.state()["sum"][99] == 0


def test_capacity_rounding(oracle_mod):
    # test/test_attention_tracker.c:44-55 (100 -> 128, 1 -> >= 64)
    assert oracle_mod.OracleSched(capacity=100).cap == 128
    assert oracle_mod.OracleSched(capacity=1).cap == 64


def test_decay_table(oracle_mod):
    # test/test_hotcold_classifier.c:74-93: exp(0)=1, [50]=e^-1, [100]=e^-2
    t = oracle_mod.decay_table(50.0)
    assert abs(t[0] - 1.0) < 1e-5
    assert abs(t[50] - math.exp(-1)) < 1e-4 and abs(t[100] - math.exp(-2)) < 1e-4


def test_hotness_pure_attention(oracle_mod):
    # test/test_hotcold_classifier.c:137-171: 0.08 after one step -> COLD
    s = oracle_mod.OracleSched(capacity=256, alpha=1.0, beta=0.0, gamma=0.0)
    s.register(1)
    s.update(1, 0.8)
    s.step_done()
    s.update_all()
    st = s.state()
    assert abs(st["hot"][1] - 0.08) < 1e-4 and st["heat"][1] == 2
    for _ in range(200):
        s.update(1, 0.8)
        s.step_done()
    s.update_all()
    st = s.state()
    assert abs(st["hot"][1] - 0.8) < 0.05 and st["heat"][1] == 0


def test_hotness_mixed_formula(oracle_mod):
    # test/test_hotcold_classifier.c:418-448: 0.5*0.05 + 0.3*exp(-0.02) + 0.2 = 0.51906
    s = oracle_mod.OracleSched(capacity=256, th_hot=0.4, th_warm=0.15)
    s.register(1)
    s.update(1, 0.5)
    s.step_done()
    s.update_all()
    st = s.state()
    assert abs(st["hot"][1] - 0.51906) < 1e-4
    assert st["heat"][1] == 0


def test_recency_and_frequency(oracle_mod):
    # test/test_hotcold_classifier.c:173-235
    s = oracle_mod.OracleSched(capacity=256, alpha=0, beta=1, gamma=0, recency_tau=10)
    s.register(1)
    s.update(1, 0.1)
    s.step_done()
    s.update_all()
    assert s.state()["heat"][1] == 0
    for _ in range(50):
        s.step_done()
    s.update_all()
    assert s.state()["heat"][1] == 2
    s = oracle_mod.OracleSched(capacity=256, alpha=0, beta=0, gamma=1)
    s.register(1)
    for _ in range(10):
        s.update(1, 0.1)
        s.step_done()
    s.update_all()
    assert abs(s.state()["hot"][1] - 1.0) < 0.01
    for _ in range(90):
        s.step_done()
    s.update_all()
    assert abs(s.state()["hot"][1] - 0.1) < 0.01 and s.state()["heat"][1] == 2


def test_sink_always_hot(oracle_mod):
    # test/test_hotcold_classifier.c:116-135
    s = oracle_mod.OracleSched(capacity=256)
    s.register(1, 0x08)
    s.update_all()
    assert s.state()["heat"][1] == 0
    for _ in range(100):
        s.step_done()
    s.update_all()
    assert s.state()["heat"][1] == 0


def test_threshold_controller(oracle_mod):
    # test/test_adaptive_threshold.c:54-176 (raise above HWM, lower below LWM, clamp)
    a = oracle_mod.Athresh()
    assert a.update(0.95, 0.5) and abs(a.th_hot - 0.52) < 1e-6
    a2 = oracle_mod.Athresh()
    assert a2.update(0.5, 0.5) and abs(a2.th_hot - 0.48) < 1e-6
    a3 = oracle_mod.Athresh()
    for _ in range(100):
        a3.update(0.99, 0.99)
    assert abs(a3.th_hot - 0.9) < 1e-6 and abs(a3.th_warm - 0.5) < 1e-6
    a4 = oracle_mod.Athresh()
    assert not a4.update(0.8, 0.8)        # midrange: no change


def test_select_coldest_ties_by_id(oracle_mod):
    hot = np.array([0.5, 0.1, 0.1, 0.3, 0.1, -0.0, 0.0, 0.2], np.float32)
    el = np.array([1, 1, 1, 1, 1, 1, 1, 0], np.uint8)
    # order: 5(-0), 6(+0) tie -> by id; then 1, 2, 4 (0.1) ...
    assert oracle_mod.select_coldest(hot, el, 3).tolist() == [1, 5, 6]
    assert oracle_mod.select_coldest(hot, el, 4).tolist() == [1, 2, 5, 6]
    assert oracle_mod.select_coldest(hot, el, 100).tolist() == [0, 1, 2, 3, 4, 5, 6]
    assert oracle_mod.select_coldest(hot, el, 0).tolist() == []


def test_prefetch_rules(oracle_mod):
    # src/scheduler/prefetch_scheduler.c:131-172 rules
    ema = np.array([0.9, 0.9, 0.3, 0.3, 0.6, 0.1], np.float32)
    act = np.ones(6, np.uint8)
    tier = np.array([0, 1, 1, 2, 2, 2], np.uint8)
    got = oracle_mod.select_prefetch(ema, act, tier, 0.5, 0.2, 10)
    assert got.tolist() == [1, 3, 4]      # 0 on GPU, 2 DRAM below th_gpu, 5 below th_dram
    assert oracle_mod.select_prefetch(ema, act, tier, 0.5, 0.2, 2).tolist() == [1, 4]


def test_score_blocks_order(oracle_mod):
    rng = np.random.default_rng(0)
    p = rng.random((3, 8, 40), dtype=np.float32)
    out = oracle_mod.score_blocks(p, Hq=8, Hkv=2, tpb=16, lens=np.array([40, 33, 17], np.uint32))
    assert out.shape == (3, 2, 3)
    exp = np.float32(0)
    for g in range(4):
        for t in range(16, 32):
            exp = np.float32(exp + p[1, 4 + g, t])
    assert out[1, 1, 1] == exp
    assert out[2, 0, 2] == 0.0            # block beyond the row's length
    assert out[1, 0, 2] == np.float32(sum(np.float64(p[1, g, 32]) for g in range(4))) or \
        abs(out[1, 0, 2] - p[1, :4, 32].sum()) < 1e-6


def test_pool_lifo_order(oracle_mod):
    # src/tiered_store/gpu_tier.cu:36-42: first pops are 0,1,2...
    p = oracle_mod.Pool(5)
    assert [p.pop() for _ in range(3)] == [0, 1, 2]
    p.push(1)
    assert p.pop() == 1 and p.pop() == 3


# ---- committed golden fixtures (generated from the compiled reference) --------

def _fixtures():
    if not os.path.isdir(GOLDEN):
        return []
    return sorted(f for f in os.listdir(GOLDEN) if f.startswith("sched_") and f.endswith(".json"))


@pytest.mark.parametrize("name", _fixtures())
def test_golden_fixture(oracle_mod, name):
    with open(os.path.join(GOLDEN, name)) as fh:
        fx = json.load(fh)
    from tests.golden.replay import replay_oracle
    got = replay_oracle(oracle_mod, fx)
    for key, want in fx["expect"].items():
        g = got[key]
        if isinstance(want, list):
            assert list(g) == want, key
        else:
            assert g == want, key


def test_fixtures_present():
    assert len(_fixtures()) >= 3, "tests/golden fixtures missing (run tests/golden/gen_golden.py)"
    assert os.path.exists(os.path.join(GOLDEN, "c4_demote_callbacks.json"))


@pytest.mark.ref
@pytest.mark.parametrize("name", ["c4_demote_callbacks", "c4_demote_callbacks_failing"])
def test_c4_fixture_regenerates(oracle_mod, name):
    """The callback-path fixtures are what the compiled reference produces now."""
    if not oracle_mod.ref_available():
        pytest.skip("reference not compiled into oracle/_ref on this machine")
    from tests.golden.gen_golden import run_ref_c4
    with open(os.path.join(GOLDEN, name + ".json")) as fh:
        fx = json.load(fh)
    assert run_ref_c4(fx["case"]) == fx["expect"]


# ---- live cross-check against the reference compiled from its sources --------

@pytest.mark.ref
def test_oracle_vs_reference_random(oracle_mod):
    if not oracle_mod.ref_available():
        pytest.skip("reference not compiled into oracle/_ref on this machine")
    rng = np.random.default_rng(7)
    kw = dict(tracker_cap=1024, max_blocks=900, ema_lambda=0.87, alpha=0.55, beta=0.3,
              gamma=0.15, recency_tau=9.0, threshold_to_gpu=0.4, threshold_to_dram=0.15)
    ref = oracle_mod.RefTM(cooldown_sec=0.0, **kw)
    orc = oracle_mod.OracleTM(**kw)
    ids = rng.choice(50000, 800, replace=False)
    for i in ids:
        f, t = int(rng.choice([0, 0, 8, 1])), int(rng.choice([0, 0, 1, 2, 4]))
        assert ref.register(int(i), t, f) == orc.register(int(i), t, f)
    for step in range(60):
        for r in rng.choice(ids, 300):
            w = float(rng.random())
            ref.report(int(r), w)
            orc.report(int(r), w)
        ref.step_done()
        orc.step_done()
        g, d = float(rng.random()), float(rng.random())
        ref.set_usage(g, d)
        orc.set_usage(g, d)
        ref.schedule_once()
        orc.schedule_once()
    a, b = ref.state(), orc.s.state()
    for k in ["sum", "ema", "hits", "last", "t_active", "hot", "heat", "c_active"]:
        assert np.array_equal(a[k].view(np.uint8), b[k].view(np.uint8)), k
    rs, os_ = ref.stats(), orc.stats()
    for k in os_:
        assert rs[k] == os_[k], k


@pytest.mark.ref
def test_pool_vs_reference_dram_tier(oracle_mod):
    if not oracle_mod.ref_available():
        pytest.skip("reference not compiled into oracle/_ref on this machine")
    rng = np.random.default_rng(3)
    ref = oracle_mod.RefDramPool(37)
    orc = oracle_mod.Pool(37)
    held = []
    for _ in range(400):
        if held and rng.random() < 0.45:
            i = held.pop(int(rng.integers(len(held))))
            assert ref.free(i) == 0
            orc.push(i)
        else:
            a, b = ref.alloc(), orc.pop()
            assert a == b
            if a is not None:
                held.append(a)
    ref.close()
