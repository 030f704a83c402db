"""GPU scheduler parity through the C ABI (liborchkv_b200.so) against the
oracle: exact for the per-block API (same inputs, same float op order),
1e-5 relative for the tensor-level reduction (different summation order),
exact for selection given the GPU's own hotness."""
import ctypes as C
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
NOBLK = 0xFFFFFFFF
REL_TOL = 1e-5     # per-block attention mass: fp32, reduction order differs


@pytest.fixture(scope="module")
def okv(cuda):
    import orchkv_b200
    orchkv_b200.lib()
    return orchkv_b200


def _fixtures():
    return sorted(f for f in os.listdir(GOLDEN) if f.startswith("sched_") and f.endswith(".json"))


@pytest.mark.parametrize("name", _fixtures())
def test_golden_replay_bit_exact(okv, name):
    from tests.golden.replay import replay_gpu
    with open(os.path.join(GOLDEN, name)) as fh:
        fx = json.load(fh)
    got = replay_gpu(okv, fx)
    for key, want in fx["expect"].items():
        assert got[key] == want, key


def test_known_answers_gpu(okv):
    # test/test_attention_tracker.c:118-150 and test/test_hotcold_classifier.c:418-448
    m = okv.Manager(tracker_cap=256, ema_lambda=0.8)
    m.register_id(1)
    m.report(1, 1.0)
    m.step_done()
    st = m.state()
    assert st["ema"][1] == np.float32(0.2) or abs(st["ema"][1] - 0.2) < 1e-7
    m.report(1, 0.5)
    m.step_done()
    assert abs(m.state()["ema"][1] - 0.26) < 1e-6
    m.close()
    m = okv.Manager(tracker_cap=256)
    m.register_id(1)
    m.report(1, 0.5)
    m.step_done()
    m.set_usage(0.8, 0.8)
    m.schedule_once()
    assert abs(m.score(1) - 0.51906) < 1e-4
    assert m.heat(1) == 0          # 0.519 >= th_hot 0.5 (thresholds move after classifying)
    m.close()


@pytest.mark.parametrize("where", ["pinned", "pageable"])
def test_tensor_scoring_host_inputs(okv, cuda, where):
    """tm_report_attn_probs reading host buffers (probabilities, lengths and
    ids, pinned or pageable) records exactly what it records from device
    copies of the same arrays, over two calls (the second grows nothing)."""
    rng = np.random.default_rng(77)
    R, Hq, Hkv, T, tpb = 5, 8, 2, 1024, 16
    nb = T // tpb
    ids = np.arange(R * Hkv * nb, dtype=np.uint32)
    states = []
    for mode in ("device", where):
        m = okv.Manager(tracker_cap=R * Hkv * nb, max_blocks=1 << 20)
        for i in range(R * Hkv * nb):
            m.register_id(i)
        for call in range(2):
            r2 = np.random.default_rng(call)
            probs = _mk_probs(r2, R, Hq, T)
            lens = r2.integers(1, T + 1, R).astype(np.uint32)
            if mode == "device":
                bufs = [_dev(cuda, a) for a in (probs, lens, ids)]
            else:
                bufs = [cuda.from_numpy(a.copy()) for a in (probs, lens, ids)]
                if where == "pinned":
                    bufs = [b.pin_memory() for b in bufs]
            assert okv.lib().tm_report_attn_probs(m.ref, bufs[0].data_ptr(), R, Hq, Hkv, T, tpb,
                                                  bufs[1].data_ptr(), bufs[2].data_ptr()) == 0
            m.step_done()
        states.append(m.state())
        m.close()
    for key in ("sum", "ema", "hits", "last"):
        assert np.array_equal(states[0][key], states[1][key]), key
    assert np.count_nonzero(states[0]["hits"]) > R * Hkv * 8


def test_concurrent_reports_from_threads(okv):
    """The reference's concurrency case (test/test_attention_tracker.c:309-343):
    4 threads each report weight 0.01 to one block 10,000 times; the sum ends
    within 0.1 of 400.  ctypes drops the GIL for each call, so the threads run
    the library's report path at the same time; a second block fed by the
    same threads with weight 1.0 must end at exactly 40,000 hits of mass."""
    import threading
    L = okv.lib()
    m = okv.Manager(tracker_cap=256, ema_lambda=0.9)
    m.register_id(1)
    m.register_id(2)

    def worker():
        for _ in range(10000):
            L.tm_notify_attn(m.ref, 1, C.c_float(0.01))
            L.tm_notify_attn(m.ref, 2, C.c_float(1.0))

    threads = [threading.Thread(target=worker) for _ in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    st = m.state()
    # all addends equal, so any interleaving gives the sequential fp32 sum
    want = np.float32(0.0)
    for _ in range(40000):
        want = np.float32(want + np.float32(0.01))
    assert st["sum"][1] == want and abs(float(want) - 400.0) < 0.1
    assert float(st["sum"][2]) == 40000.0                # exact in fp32
    assert st["hits"][1] == 0 and st["t_active"][1] == 1
    m.close()


def _dev(cuda, arr):
    return cuda.from_numpy(np.ascontiguousarray(arr)).cuda()


def _mk_probs(rng, R, Hq, T):
    logits = rng.normal(0, 2, (R, Hq, T)).astype(np.float32)
    logits -= logits.max(-1, keepdims=True)
    p = np.exp(logits)
    return (p / p.sum(-1, keepdims=True)).astype(np.float32)


@pytest.mark.parametrize("tpb,T,lens_mode", [(16, 1024, "full"), (64, 2048, "ragged"),
                                             (4, 256, "full"), (128, 1536, "ragged"),
                                             (12, 300, "ragged"), (16, 1030, "full")])
def test_tensor_scoring_vs_oracle(okv, oracle_mod, cuda, tpb, T, lens_mode):
    rng = np.random.default_rng(tpb * 1000 + T)
    R, Hq, Hkv = 6, 14, 2
    nb = (T + tpb - 1) // tpb
    probs = _mk_probs(rng, R, Hq, T)
    lens = np.full(R, T, np.uint32) if lens_mode == "full" else \
        rng.integers(1, T + 1, R).astype(np.uint32)
    ids = np.arange(R * Hkv * nb, dtype=np.uint32).reshape(R, Hkv, nb)
    ids[0, 1, 3] = NOBLK
    m = okv.Manager(tracker_cap=R * Hkv * nb, max_blocks=1 << 20)
    for i in range(R * Hkv * nb):
        if i % 17 != 5:                        # some blocks unregistered: reports ignored
            m.register_id(i)
    dp, di, dl = _dev(cuda, probs), _dev(cuda, ids), _dev(cuda, lens)
    rc = okv.lib().tm_report_attn_probs(m.ref, dp.data_ptr(), R, Hq, Hkv, T, tpb,
                                        dl.data_ptr(), di.data_ptr())
    assert rc == 0
    st = m.state()
    want = oracle_mod.score_blocks(probs, Hq, Hkv, tpb, lens)
    exact_path = not ((tpb & (tpb - 1)) == 0 and tpb <= 128 and T % 4 == 0)
    for r in range(R):
        for h in range(Hkv):
            for b in range(nb):
                i = ids[r, h, b]
                if i == NOBLK:
                    continue
                got_sum, hit = st["sum"][i], st["last"][i] == 0
                has_tokens = b * tpb < lens[r]
                if i % 17 == 5:
                    assert got_sum == 0 and st["t_active"][i] == 0
                    continue
                if not has_tokens:
                    assert got_sum == 0 and not hit
                    continue
                assert hit
                w = want[r, h, b]
                if exact_path:
                    assert got_sum == w
                else:
                    assert abs(got_sum - w) <= REL_TOL * max(abs(w), 1e-30)
    m.close()


def test_step_and_classify_bit_exact(okv, oracle_mod, cuda):
    rng = np.random.default_rng(5)
    n = 4096
    m = okv.Manager(tracker_cap=n, ema_lambda=0.85, alpha=0.6, beta=0.25, gamma=0.15,
                    recency_tau=11.0)
    o = oracle_mod.OracleSched(n, 0.85, 0.6, 0.25, 0.15, 11.0)
    flags = rng.choice([0, 0, 0, 8], n)
    for i in range(n):
        m.register_id(i, 0, int(flags[i]))
        o.register(i, int(flags[i]))
    for step in range(12):
        ids = rng.choice(n, n // 3, replace=False).astype(np.uint32)
        w = rng.random(len(ids)).astype(np.float32)
        di, dw = _dev(cuda, ids), _dev(cuda, w)
        assert okv.lib().tm_report_attn_batch_dev(m.ref, di.data_ptr(), dw.data_ptr(), len(ids)) == 0
        assert okv.lib().tm_step_and_classify(m.ref) == 0
        o.update_batch(ids.astype(np.uint64), w)
        o.step_done()
        o.update_all()
    a, b = m.state(), o.state()
    for k in ["ema", "hits", "last", "hot", "heat"]:
        assert np.array_equal(a[k].view(np.uint8), b[k].view(np.uint8)), k
    m.close()


def _select(okv, cuda, m, k, mode="victims", thg=0.0, thd=0.0):
    out = cuda.zeros(max(k, 1), dtype=cuda.int32, device="cuda")
    cnt = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    if mode == "victims":
        rc = okv.lib().tm_select_victims(m.ref, k, out.data_ptr(), cnt.data_ptr())
    else:
        rc = okv.lib().tm_select_prefetch(m.ref, k, thg, thd, out.data_ptr(), cnt.data_ptr())
    assert rc == 0
    assert okv.lib().tm_sync(m.ref) == 0
    c = int(cnt.item())
    return out[:c].cpu().numpy().view(np.uint32).copy()


@pytest.mark.parametrize("n,k", [(5000, 0), (5000, 1), (5000, 1250), (5000, 4999),
                                 (5000, 99999), (70000, 17000)])
def test_select_victims_vs_oracle(okv, oracle_mod, cuda, n, k):
    rng = np.random.default_rng(n + k)
    m = okv.Manager(tracker_cap=n, max_blocks=1 << 20)
    tiers = rng.choice([0, 0, 0, 1], n)
    flags = rng.choice([0, 0, 0, 0, 1, 8], n)
    for i in range(n):
        m.register_id(i, int(tiers[i]), int(flags[i]))
    # quantised weights produce many exact hotness ties
    ids = rng.choice(n, n // 2, replace=False).astype(np.uint32)
    w = (rng.integers(0, 7, len(ids)) / 8).astype(np.float32)
    ids_d, w_d = _dev(cuda, ids), _dev(cuda, w)        # held until the launch has run
    okv.lib().tm_report_attn_batch_dev(m.ref, ids_d.data_ptr(), w_d.data_ptr(), len(ids))
    okv.lib().tm_step_and_classify(m.ref)
    st = m.state()
    cap = m.cap
    elig = np.zeros(cap, np.uint8)
    elig[:n] = (tiers == 0) & ((flags & 9) == 0)
    want = oracle_mod.select_coldest(st["hot"], elig & st["c_active"], k)
    got = _select(okv, cuda, m, k)
    assert np.array_equal(got, want)
    m.close()


def test_select_prefetch_vs_oracle(okv, oracle_mod, cuda):
    rng = np.random.default_rng(11)
    n = 20000
    m = okv.Manager(tracker_cap=n, max_blocks=1 << 20)
    tiers = rng.choice([0, 1, 2, 4], n)
    for i in range(n):
        m.register_id(i, int(tiers[i]), 0)
    for _ in range(3):
        ids = rng.choice(n, n // 2, replace=False).astype(np.uint32)
        w = (rng.integers(0, 9, len(ids)) / 4).astype(np.float32)
        ids_d, w_d = _dev(cuda, ids), _dev(cuda, w)
        okv.lib().tm_report_attn_batch_dev(m.ref, ids_d.data_ptr(), w_d.data_ptr(), len(ids))
        okv.lib().tm_step_and_classify(m.ref)
    st = m.state()
    tier_full = np.full(m.cap, 4, np.uint8)
    tier_full[:n] = tiers
    for thg, thd, k in [(0.5, 0.2, 300), (0.0, 0.0, 1000), (0.9, 0.1, 50000), (0.3, 0.3, 0)]:
        want = oracle_mod.select_prefetch(st["ema"], st["t_active"], tier_full, thg, thd, k)
        got = _select(okv, cuda, m, k, "prefetch", thg, thd)
        assert np.array_equal(got, want), (thg, thd, k)
    m.close()


@pytest.mark.parametrize("where", ["device", "host"])
def test_range_mass_vs_oracle(okv, oracle_mod, cuda, where):
    """tm_report_attn_ranges: block i gets the sum over heads and tokens
    [start_i, min(end_i, kv_len)) of avg; ranges clipped by kv_len, empty
    ranges and ranges wholly past kv_len report nothing; unregistered ids are
    ignored.  Against the oracle tracker fed the same per-block sums (summed
    in another order: 1e-5)."""
    rng = np.random.default_rng(31)
    heads, kv_len, n = 6, 700, 60
    avg = rng.random((heads, kv_len)).astype(np.float32) / kv_len
    starts = rng.integers(0, 760, n).astype(np.uint32)
    ends = (starts + rng.integers(0, 40, n)).astype(np.uint32)
    starts[:3], ends[:3] = [5, 690, 720], [5, 740, 760]       # empty, clipped, past the end
    ids = rng.permutation(4000)[:n].astype(np.uint32)
    m = okv.Manager(tracker_cap=4096, max_blocks=1 << 20)
    orc = oracle_mod.OracleSched(4096, 0.9, 0.5, 0.3, 0.2, 50.0)
    for i in ids[::2]:                                         # every other id registered
        m.register_id(int(i))
        orc.register(int(i))
    if where == "device":
        bufs = [_dev(cuda, a) for a in (avg, starts, ends, ids)]
    else:
        bufs = [cuda.from_numpy(a.copy()) for a in (avg, starts, ends, ids)]
    assert okv.lib().tm_report_attn_ranges(m.ref, bufs[0].data_ptr(), heads, kv_len,
                                           bufs[1].data_ptr(), bufs[2].data_ptr(),
                                           bufs[3].data_ptr(), n) == 0
    reported = 0
    for i in range(n):
        s, e = int(starts[i]), min(int(ends[i]), kv_len)
        if s < e:
            orc.update(int(ids[i]), float(avg[:, s:e].astype(np.float64).sum()))
            reported += int(i % 2 == 0)
    m.step_done()
    orc.step_done()
    got, want = m.state(), orc.state()
    sl = ids.astype(np.int64) & 4095
    for key in ("hits", "last", "t_active"):
        assert np.array_equal(got[key][sl], want[key][sl]), key
    a, b = got["ema"][sl], want["ema"][sl]
    assert np.all(np.abs(a - b) <= REL_TOL * np.maximum(np.abs(b), 1e-30))
    assert int(np.count_nonzero(got["hits"][sl])) == reported > 10
    assert okv.lib().tm_report_attn_ranges(m.ref, 0, heads, kv_len, bufs[1].data_ptr(),
                                           bufs[2].data_ptr(), bufs[3].data_ptr(), n) == -2
    m.close()
