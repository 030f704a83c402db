"""The CPU-runnable scheduler step end to end on the GPU: 1 request, 8 layers
x 4 KV heads, d_head 128 fp16, 64-token blocks, 4096-token context (2,048
slabs of 32 KB).  Attention probabilities per (layer, 28 q-heads, token) are
softmax(N(0,2) logits + 0.002 * position); every slab has Poisson(3) hits
spread over a 16-step history; alpha, beta, gamma = 0.5, 0.3, 0.2, EMA decay
0.9, tau 50; seed 0.  The step scores all slabs with one launch, classifies,
selects the coldest 50% (1,024 slabs), evicts them to pinned DRAM and
promotes them back.

Checked against the oracle (always) and, where oracle/_ref is built, the
reference itself: its C scheduler fed the same reports
(src/scheduler/attention_tracker.c, hotcold_classifier.c) and its data plane
(src/api/orchkv_api.cu:353-428) evicting and promoting the same blocks one by
one.  Hits and last-hit steps exact; EMA and hotness within 1e-5 relative
(the per-block mass is summed in another order); victims identical to the
oracle's selection on the GPU's hotness and, against the reference's
hotness, differing only between blocks tied within that tolerance; DRAM and
GPU slab indices and all slab bytes bit-exact, before and after the round
trip."""
import ctypes as C

import numpy as np
import pytest

from tests.test_gpu_pool import read_dev, read_host

pytestmark = pytest.mark.gpu

LY, HQ, HKV, D, TPB, T = 8, 28, 4, 128, 64, 4096
NB = T // TPB
N = LY * HKV * NB
ROW = D * 2
SLAB = TPB * ROW * 2
HALF = SLAB // 2
HIST = 16
REL = 1e-5


def make_inputs():
    rng = np.random.default_rng(0)
    logits = (rng.normal(0, 2, (LY, HQ, T)).astype(np.float32)
              + (0.002 * np.arange(T)).astype(np.float32))
    logits -= logits.max(-1, keepdims=True)
    p = np.exp(logits)
    probs = (p / p.sum(-1, keepdims=True)).astype(np.float32)
    kv = rng.standard_normal((LY, 2, HKV, T, D)).astype(np.float16)
    hits = np.minimum(rng.poisson(3, N), HIST)
    history = [[] for _ in range(HIST)]           # per step: (slab index, weight)
    for i in range(N):
        steps = rng.choice(HIST, hits[i], replace=False)
        w = rng.random(hits[i]).astype(np.float32)
        for s, x in zip(steps, w):
            history[int(s)].append((i, float(x)))
    for h in history:
        h.sort()
    return probs, kv, history


def slab_bytes(kv, l, h, b):
    """[K tpb x d | V tpb x d] of block b (src/api/orchkv_api.cu:8-18)."""
    k = kv[l, 0, h, b * TPB:(b + 1) * TPB].view(np.uint8).reshape(-1)
    v = kv[l, 1, h, b * TPB:(b + 1) * TPB].view(np.uint8).reshape(-1)
    return np.concatenate([k, v])


def lhb_of(i):
    """slab index i <-> (layer, head, block), the id table's order."""
    return i // (HKV * NB), (i // NB) % HKV, i % NB


def _dev(cuda, a):
    return cuda.from_numpy(np.ascontiguousarray(a)).cuda()


def test_cpu_step_end_to_end(cuda, oracle_mod):
    import orchkv_b200 as o
    O = oracle_mod
    L = o.lib()
    probs, kv, history = make_inputs()
    cfg = o.make_config(gpu_pool_bytes=(N + 64) * SLAB, dram_pool_bytes=N * SLAB,
                        tokens_per_block=TPB, d_head=D, dtype=0, max_blocks_per_head=NB + 8)
    ext = o.OrchkvConfigExt()
    ext.max_blocks = 4096
    assert L.orchkv_init_ext(C.byref(cfg), C.byref(ext)) == 0
    tm = o.Manager(tracker_cap=4096, max_blocks=8192, ema_lambda=0.9, alpha=0.5, beta=0.3,
                   gamma=0.2, recency_tau=50.0, cooldown_sec=0.0)
    ref_tm = ref_api = None
    try:
        assert L.orchkv_attach_scheduler(tm.ref) == 0
        ctx = L.orchkv_request_create(0, LY, HKV)
        assert ctx
        for l in range(LY):
            assert L.orchkv_prefill(ctx, l, kv[l, 0].ctypes.data, kv[l, 1].ctypes.data, T) == 0
        arr = (C.c_void_p * 1)(ctx)
        ids_d = cuda.empty(N, dtype=cuda.int32, device="cuda")
        assert L.orchkv_block_id_table(arr, 1, T, C.c_void_p(ids_d.data_ptr())) == 0
        assert L.orchkv_sync() == 0
        ids = ids_d.cpu().numpy().view(np.uint32).astype(np.uint64)
        assert len(set(ids.tolist())) == N

        orc = O.OracleSched(4096, 0.9, 0.5, 0.3, 0.2, 50.0)
        for i in ids:
            orc.register(int(i))
        if O.ref_available():
            ref_tm = O.RefTM(tracker_cap=4096, max_blocks=8192, recency_tau=50.0,
                             cooldown_sec=0.0)
            for i in ids:
                assert ref_tm.register(int(i), 0, 0) == 0

        # 16-step hit history, per-block reports
        for step in history:
            for i, w in step:
                tm.report(int(ids[i]), w)
                orc.update(int(ids[i]), w)
                if ref_tm:
                    ref_tm.report(int(ids[i]), w)
            tm.step_done()
            orc.step_done()
            if ref_tm:
                ref_tm.step_done()

        # the measured step: one scoring launch over all slabs, step + classify
        probs_d = _dev(cuda, probs)
        assert L.tm_report_attn_probs(tm.ref, probs_d.data_ptr(), LY, HQ, HKV, T, TPB, None,
                                      ids_d.data_ptr()) == 0
        assert L.tm_step_and_classify(tm.ref) == 0
        mass = O.score_blocks(probs, HQ, HKV, TPB).reshape(-1)   # [layer][head][block]
        orc.update_batch(ids, mass)
        orc.step_done()
        orc.update_all()
        if ref_tm:
            ref_tm.report_batch(ids, mass)
            ref_tm.step_done()
            ref_tm.update_all()

        got = tm.state()
        sl = (ids & (tm.cap - 1)).astype(np.int64)
        want = orc.state()
        osl = (ids & (len(want["ema"]) - 1)).astype(np.int64)
        for key in ("hits", "last"):
            assert np.array_equal(got[key][sl], want[key][osl]), key
        for key in ("ema", "hot"):
            a, b = got[key][sl], want[key][osl]
            assert np.all(np.abs(a - b) <= REL * np.maximum(np.abs(b), 1e-30)), key
        if ref_tm:
            rs = ref_tm.state()
            rsl = (ids & (ref_tm.cap - 1)).astype(np.int64)
            for key in ("ema", "hot", "hits", "last", "heat"):
                # the oracle is the reference bit for bit on the same reports
                assert np.array_equal(want[key][osl].view(np.uint8),
                                      rs[key][rsl].view(np.uint8)), key

        # coldest 50%
        k = N // 2
        out = cuda.zeros(N, dtype=cuda.int32, device="cuda")
        cnt = cuda.zeros(1, dtype=cuda.int32, device="cuda")
        assert L.tm_select_victims(tm.ref, k, out.data_ptr(), cnt.data_ptr()) == 0
        assert L.orchkv_sync() == 0
        assert int(cnt.item()) == k
        victims = out[:k].cpu().numpy().view(np.uint32).copy()
        elig = got["c_active"].copy()
        assert np.array_equal(victims, O.select_coldest(got["hot"], elig, k))
        # against the reference's own hotness: only near-ties may swap
        h_ref = want["hot"][osl]
        order = np.lexsort((ids, h_ref))
        ref_sel = set(ids[order[:k]].tolist())
        kth = h_ref[order[k - 1]]
        pos = {int(b): j for j, b in enumerate(ids.tolist())}
        for b in ref_sel.symmetric_difference(victims.tolist()):
            assert abs(h_ref[pos[b]] - kth) <= 4 * REL * abs(kth), b

        # evict the victims, then promote them back
        vic_d = _dev(cuda, victims.view(np.int32))
        res = cuda.zeros(2, dtype=cuda.int32, device="cuda")
        assert L.orchkv_evict_batch_to_dram(vic_d.data_ptr(), None, k, res.data_ptr()) == 0
        assert L.orchkv_sync() == 0
        assert res.cpu().tolist() == [k, 0]
        dram = read_host(L.orchkv_dram_pool_base(), N * SLAB)
        vic_slab = [pos[int(b)] for b in victims]            # slab index in [l][h][b] order
        d_slabs = []
        for i in vic_slab:
            l, h, b = lhb_of(i)
            rc, bid, tier, s, st, tok = _info(L, ctx, l, h, b)
            assert rc == 0 and tier == 1 and st == 3
            d_slabs.append(s)
            assert np.array_equal(dram[s * SLAB:(s + 1) * SLAB], slab_bytes(kv, l, h, b)), i
        assert L.orchkv_promote_batch_to_gpu(vic_d.data_ptr(), None, k, res.data_ptr()) == 0
        assert L.orchkv_sync() == 0
        assert res.cpu().tolist() == [k, 0]
        gpu = read_dev(L.orchkv_gpu_pool_base(), (N + 64) * SLAB)
        g_slabs = []
        for i in range(N):
            l, h, b = lhb_of(i)
            rc, bid, tier, s, st, tok = _info(L, ctx, l, h, b)
            assert rc == 0 and tier == 0
            g_slabs.append(s)
            assert np.array_equal(gpu[s * SLAB:(s + 1) * SLAB], slab_bytes(kv, l, h, b)), i

        if O.ref_available():
            # the reference data plane, block by block in the same order
            R = O.ref()
            assert R.ref_api_init(0, (N + 64) * SLAB, N * SLAB, TPB, D, 0, 1, NB + 8,
                                  b"/tmp/orchkv_ref_cpu_step") == 0
            ref_api = R
            rc_ = R.ref_api_request_create(0, LY, HKV)
            assert rc_
            for l in range(LY):
                assert R.ref_api_prefill(rc_, l, kv[l, 0].ctypes.data, kv[l, 1].ctypes.data,
                                         T) == 0
            tier, data = C.c_int(), C.c_void_p()
            dbase = R.ref_api_dram_base()
            for i, s in zip(vic_slab, d_slabs):
                l, h, b = lhb_of(i)
                assert R.ref_api_evict(rc_, l, h, b) == 0
                assert R.ref_api_block(rc_, l, h, b, C.byref(tier), C.byref(data)) == 0
                assert tier.value == 1 and (data.value - dbase) // SLAB == s
            ref_dram = read_host(dbase, N * SLAB)
            for s in d_slabs:
                assert np.array_equal(ref_dram[s * SLAB:(s + 1) * SLAB],
                                      dram[s * SLAB:(s + 1) * SLAB]), s
            for i in vic_slab:
                assert R.ref_api_promote(rc_, *lhb_of(i)) == 0
            gbase = R.ref_api_gpu_base()
            ref_gpu = read_dev(gbase, (N + 64) * SLAB)
            for i in range(N):
                l, h, b = lhb_of(i)
                assert R.ref_api_block(rc_, l, h, b, C.byref(tier), C.byref(data)) == 0
                assert tier.value == 0
                s = (data.value - gbase) // SLAB
                assert s == g_slabs[i], i
                assert np.array_equal(ref_gpu[s * SLAB:(s + 1) * SLAB],
                                      gpu[s * SLAB:(s + 1) * SLAB]), i
            assert R.ref_api_request_destroy(rc_) == 0
        assert L.orchkv_request_destroy(ctx) == 0
    finally:
        if ref_api is not None:
            ref_api.ref_api_shutdown()
        if ref_tm:
            ref_tm.close()
        L.orchkv_shutdown()
        tm.close()


def _info(L, ctx, l, h, b):
    bid, tier, slab, st, tok = C.c_uint64(), C.c_int(), C.c_uint32(), C.c_int(), C.c_uint32()
    rc = L.orchkv_block_info(ctx, l, h, b, C.byref(bid), C.byref(tier), C.byref(slab),
                             C.byref(st), C.byref(tok))
    return rc, bid.value, tier.value, slab.value, st.value, tok.value
