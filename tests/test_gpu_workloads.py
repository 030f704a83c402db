"""Parity cases shaped like the path's three multi-request workloads, each
cut to a size the oracle checks in seconds, run through the C ABI on one GPU:

* Llama-3-8B-shaped (32 layers, 32 q-heads / 8 KV heads, d 128, fp16,
  64-token blocks): Zipf(1.1) block attention mass over each (request,
  layer, KV head)'s blocks in a seeded order, three steps, GPU capacity 40%
  (the coldest 60% evicted to DRAM, then promoted back).
* Mistral-7B-shaped time-multiplexed pool (32 layers, 32 q-heads / 8 KV
  heads, d 128, bf16, 16-token blocks): four sub-batches of requests, two
  resident; every step scores the resident ones (logits N(0, 1.5)) and one
  orchkv_swap_batch evicts a resident sub-batch while promoting the next,
  so half of the GPU's blocks move each way.
* Llama-3-70B-shaped three tiers (80 layers, 64 q-heads / 8 KV heads, d 128,
  fp16, 64-token blocks): GPU keeps 20%, DRAM takes 50%, the coldest 30%
  go two hops to the POSIX file tier; then everything comes back.

Checked against the oracle and, where oracle/_ref is built, the reference:
tracker and classifier state (bit-exact where the per-block mass is given,
1e-5 relative where the kernel sums probabilities in another order),
victim sets, free stacks, block locations, and every slab's bytes against
the data each request was filled with, in HBM, in DRAM and in the file at
the reference's offsets (src/tiered_store/orchfs_tier.h:89-97)."""
import ctypes as C
import os

import numpy as np
import pytest

from tests.test_gpu_pool import locs, pool_state, read_dev, read_host

pytestmark = pytest.mark.gpu

MASK = 0x1FFFFFFF
REL = 1e-5


def _dev(cuda, a):
    return cuda.from_numpy(np.ascontiguousarray(a)).cuda()


def _ids_dev(cuda, ids):
    return _dev(cuda, np.asarray(ids, np.uint32).view(np.int32))


class Geometry:
    def __init__(self, ly, hq, hkv, d, tpb, t, b, elem=2):
        self.ly, self.hq, self.hkv, self.d, self.tpb, self.t, self.b = ly, hq, hkv, d, tpb, t, b
        self.nb = t // tpb
        self.rows = b * ly
        self.n = b * ly * hkv * self.nb
        self.slab = tpb * d * elem * 2
        self.half = self.slab // 2

    def lhb(self, idx):
        """table index -> (request, layer, head, block)"""
        r, rem = divmod(int(idx), self.ly * self.hkv * self.nb)
        l, rem = divmod(rem, self.hkv * self.nb)
        h, b = divmod(rem, self.nb)
        return r, l, h, b


def kv_row(rng, g, bf16):
    """K and V of one (request, layer): [kv head][token][d], N(0, 1) values
    as fp16, or as bf16 (the top half of each fp32)."""
    shape = (g.hkv, g.t, g.d)
    out = []
    for _ in range(2):
        x = rng.standard_normal(shape, dtype=np.float32)
        out.append((x.view(np.uint32) >> 16).astype(np.uint16) if bf16 else x.astype(np.float16))
    return out


def fill(L, g, rng, ctxs, expect, bf16, rows=None):
    """Prefill every (request, layer) of `ctxs` and record each slab's bytes,
    [K tpb x d | V tpb x d] (src/api/orchkv_api.cu:8-18), in `expect`."""
    if rows is None:
        rows = list(enumerate(ctxs))
    for ri, ctx in rows:
        for layer in range(g.ly):
            k, v = kv_row(rng, g, bf16)
            assert L.orchkv_prefill(ctx, layer, k.ctypes.data, v.ctypes.data, g.t) == 0
            e = expect[ri * g.ly + layer]
            e[:, :, :g.half] = k.reshape(g.hkv, g.nb, -1).view(np.uint8)
            e[:, :, g.half:] = v.reshape(g.hkv, g.nb, -1).view(np.uint8)


def id_table(L, cuda, g, ctxs):
    arr = (C.c_void_p * len(ctxs))(*ctxs)
    ids_d = cuda.empty(len(ctxs) * g.ly * g.hkv * g.nb, dtype=cuda.int32, device="cuda")
    assert L.orchkv_block_id_table(arr, len(ctxs), g.t, C.c_void_p(ids_d.data_ptr())) == 0
    assert L.orchkv_sync() == 0
    ids = ids_d.cpu().numpy().view(np.uint32).astype(np.int64)
    assert len(np.unique(ids)) == len(ids)
    return ids, ids_d


def check_bytes(L, g, ids, expect, n_gpu, n_dram, max_blocks):
    """Every block's bytes where it lives (HBM or DRAM) == what it was filled
    with; returns each block's tier."""
    loc, _ = locs(L, max_blocks)
    w = loc[ids].astype(np.int64)
    tier, slab = w >> 29, w & MASK
    exp = expect.reshape(-1, g.slab)
    gb = read_dev(L.orchkv_gpu_pool_base(), n_gpu * g.slab).reshape(n_gpu, g.slab)
    on = tier == 0
    assert np.array_equal(gb[slab[on]], exp[on])
    del gb
    on = tier == 1
    if on.any():
        db = read_host(L.orchkv_dram_pool_base(), n_dram * g.slab).reshape(n_dram, g.slab)
        assert np.array_equal(db[slab[on]], exp[on])
    return tier


class PoolModel:
    """The oracle's per-block model of the pools (src/api/orchkv_api.cu:353-428,
    in list order), loaded from the device's current state."""

    def __init__(self, L, g, n_gpu, n_dram, max_blocks):
        from oracle import oracle as O
        self.O, self.g, self.n_gpu, self.n_dram, self.maxb = O, g, n_gpu, n_dram, max_blocks
        self.gp, self.dp = O.Pool(n_gpu), O.Pool(n_dram)
        self.gp.stack = pool_state(L, 0, n_gpu)
        self.dp.stack = pool_state(L, 1, n_dram)
        loc, state = locs(L, max_blocks)
        self.loc = loc.astype(np.int64).tolist()
        self.state = state.tolist()
        self.gb = read_dev(L.orchkv_gpu_pool_base(), n_gpu * g.slab)
        self.db = read_host(L.orchkv_dram_pool_base(), n_dram * g.slab)

    def evict(self, ids):
        return self.O.evict_batch(self.gp, self.dp, self.loc, self.state, None,
                                  [int(x) for x in ids], self.gb, self.db, self.g.slab)

    def promote(self, ids):
        return self.O.promote_batch(self.gp, self.dp, self.loc, self.state,
                                    [int(x) for x in ids], self.gb, self.db, self.g.slab)

    def check(self, L, evicted=()):
        """Device == model: free stacks and tiers exactly; a block's slab index
        exactly, except that a staged evict hands the popped DRAM slabs to its
        victims in ascending order, so those are compared as a set."""
        assert pool_state(L, 0, self.n_gpu) == self.gp.stack
        assert pool_state(L, 1, self.n_dram) == self.dp.stack
        loc, _ = locs(L, self.maxb)
        loc = loc.astype(np.int64)
        mloc = np.asarray(self.loc, np.int64)
        assert np.array_equal(loc >> 29, mloc >> 29)
        ev = np.zeros(self.maxb, bool)
        ev[np.asarray(evicted, np.int64).reshape(-1)] = True
        free = ~(ev & ((loc >> 29) == 1))
        bad = np.nonzero(free & (loc != mloc))[0]
        assert len(bad) == 0, (len(bad), [(int(i), bool(ev[i]), int(loc[i] >> 29),
                                           int(loc[i] & MASK), int(mloc[i] & MASK))
                                          for i in bad[:6]])
        assert sorted((loc[~free] & MASK).tolist()) == sorted((mloc[~free] & MASK).tolist())


def init(o, L, g, n_gpu, n_dram, dtype, max_blocks, mbph=None, base=None, staging_mb=0):
    cfg = o.make_config(gpu_pool_bytes=n_gpu * g.slab, dram_pool_bytes=n_dram * g.slab,
                        tokens_per_block=g.tpb, d_head=g.d, dtype=dtype,
                        max_blocks_per_head=mbph or g.nb + 8)
    if base:
        cfg.orchfs_base_dir = base.encode()
    ext = o.OrchkvConfigExt()
    ext.max_blocks = max_blocks
    ext.staging_mb = staging_mb
    assert L.orchkv_init_ext(C.byref(cfg), C.byref(ext)) == 0


def compare_sched(got, want, cap, ids, exact, thresholds=(0.5, 0.2)):
    """Device tracker/classifier state == oracle's for these ids.  When the
    per-block mass was summed in another order (exact=False), EMA and hotness
    agree within REL and the heat class is compared away from the hot and
    warm thresholds only."""
    sl = (np.asarray(ids, np.int64) & (cap - 1))
    for key in ("hits", "last", "c_active"):
        assert np.array_equal(got[key][sl], want[key][sl]), key
    for key in ("ema", "hot"):
        a, b = got[key][sl], want[key][sl]
        if exact:
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), key
        else:
            assert np.all(np.abs(a - b) <= REL * np.maximum(np.abs(b), 1e-30)), key
    far = np.ones(len(sl), bool)
    if not exact:
        h = want["hot"][sl]
        for th in thresholds:
            far &= np.abs(h - th) > REL * th
    assert np.array_equal(got["heat"][sl][far], want["heat"][sl][far])


def select(L, cuda, tm, k, n):
    out = cuda.zeros(max(n, 1), dtype=cuda.int32, device="cuda")
    cnt = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    assert L.tm_select_victims(tm.ref, k, out.data_ptr(), cnt.data_ptr()) == 0
    assert L.orchkv_sync() == 0
    c = int(cnt.item())
    return out[:c].cpu().numpy().view(np.uint32).astype(np.int64)


# ---------------------------------------------------------------------------
# Llama-3-8B-shaped: Zipf(1.1) block mass, GPU capacity 40%
# ---------------------------------------------------------------------------

def test_llama3_8b_zipf_capacity_40pct(cuda, oracle_mod):
    import orchkv_b200 as o
    O = oracle_mod
    L = o.lib()
    g = Geometry(ly=32, hq=32, hkv=8, d=128, tpb=64, t=1024, b=2)      # 8,192 slabs of 32 KB
    n_gpu, n_dram, maxb, cap = g.n + 64, g.n, 16384, 16384
    init(o, L, g, n_gpu, n_dram, dtype=0, max_blocks=maxb)
    tm = o.Manager(tracker_cap=cap, max_blocks=2 * maxb, ema_lambda=0.9, alpha=0.5, beta=0.3,
                   gamma=0.2, recency_tau=50.0, cooldown_sec=0.0)
    ref_tm = None
    try:
        assert L.orchkv_attach_scheduler(tm.ref) == 0
        rng = np.random.default_rng(3)
        ctxs = [L.orchkv_request_create(r, g.ly, g.hkv) for r in range(g.b)]
        assert all(ctxs)
        expect = np.empty((g.rows, g.hkv, g.nb, g.slab), np.uint8)
        fill(L, g, rng, ctxs, expect, bf16=False)
        ids, ids_d = id_table(L, cuda, g, ctxs)
        assert ids.max() < cap
        orc = O.OracleSched(cap, 0.9, 0.5, 0.3, 0.2, 50.0)
        for i in ids:
            orc.register(int(i))
        if O.ref_available():
            ref_tm = O.RefTM(tracker_cap=cap, max_blocks=2 * maxb, recency_tau=50.0,
                             cooldown_sec=0.0)
            for i in ids:
                assert ref_tm.register(int(i), 0, 0) == 0

        zipf = (np.arange(1, g.nb + 1, dtype=np.float64) ** -1.1)
        zipf = (zipf / zipf.sum()).astype(np.float32)
        for _ in range(3):
            mass = np.empty((g.rows * g.hkv, g.nb), np.float32)
            for j in range(g.rows * g.hkv):
                mass[j, rng.permutation(g.nb)] = zipf
            m = mass.reshape(-1)
            w_d = _dev(cuda, m)
            assert L.tm_report_attn_batch_dev(tm.ref, C.c_void_p(ids_d.data_ptr()),
                                              C.c_void_p(w_d.data_ptr()), g.n) == 0
            assert L.tm_step_and_classify(tm.ref) == 0
            orc.update_batch(ids, m)
            orc.step_done()
            orc.update_all()
            if ref_tm:
                ref_tm.report_batch(ids, m)
                ref_tm.step_done()
                ref_tm.update_all()
        got, want = tm.state(), orc.state()
        compare_sched(got, want, cap, ids, exact=True)
        if ref_tm:
            rs = ref_tm.state()
            rsl = ids & (ref_tm.cap - 1)
            osl = ids & (cap - 1)
            for key in ("ema", "hot", "hits", "last", "heat"):
                assert np.array_equal(want[key][osl].view(np.uint8), rs[key][rsl].view(np.uint8))

        # GPU capacity 40%: the coldest 60% leave
        k = g.n - int(0.4 * g.n)
        victims = select(L, cuda, tm, k, g.n)
        assert len(victims) == k
        assert np.array_equal(victims, O.select_coldest(got["hot"], got["c_active"], k))
        order = np.lexsort((ids, want["hot"][ids & (cap - 1)]))
        assert np.array_equal(victims, np.sort(ids[order[:k]]))

        m = PoolModel(L, g, n_gpu, n_dram, maxb)
        res = cuda.zeros(2, dtype=cuda.int32, device="cuda")
        vd = _ids_dev(cuda, victims)
        assert L.orchkv_evict_batch_to_dram(vd.data_ptr(), None, k, res.data_ptr()) == 0
        assert L.orchkv_sync() == 0
        assert res.cpu().tolist() == list(m.evict(victims)) == [k, 0]
        m.check(L, evicted=victims)
        tier = check_bytes(L, g, ids, expect, n_gpu, n_dram, maxb)
        assert int((tier == 1).sum()) == k

        assert L.orchkv_promote_batch_to_gpu(vd.data_ptr(), None, k, res.data_ptr()) == 0
        assert L.orchkv_sync() == 0
        assert res.cpu().tolist() == list(m.promote(victims)) == [k, 0]
        m.check(L, evicted=victims)
        tier = check_bytes(L, g, ids, expect, n_gpu, n_dram, maxb)
        assert (tier == 0).all()
        for c in ctxs:
            assert L.orchkv_request_destroy(c) == 0
    finally:
        if ref_tm:
            ref_tm.close()
        L.orchkv_shutdown()
        tm.close()


# ---------------------------------------------------------------------------
# Mistral-7B-shaped time-multiplexed pool: four sub-batches, two resident
# ---------------------------------------------------------------------------

def test_mistral_time_multiplexed_rotation(cuda, oracle_mod):
    import orchkv_b200 as o
    O = oracle_mod
    L = o.lib()
    g = Geometry(ly=32, hq=32, hkv=8, d=128, tpb=16, t=128, b=8)       # 16,384 slabs of 8 KB
    per_req = g.ly * g.hkv * g.nb
    sb_n = 2 * per_req                                                 # 4,096 slabs
    n_gpu, n_dram, maxb, cap = 3 * sb_n + 64, 3 * sb_n + 64, 32768, 32768
    init(o, L, g, n_gpu, n_dram, dtype=1, max_blocks=maxb, staging_mb=64)
    tm = o.Manager(tracker_cap=cap, max_blocks=maxb, ema_lambda=0.9, alpha=0.5, beta=0.3,
                   gamma=0.2, recency_tau=50.0, cooldown_sec=0.0)
    try:
        assert L.orchkv_attach_scheduler(tm.ref) == 0
        rng = np.random.default_rng(4)
        ctxs = [L.orchkv_request_create(r, g.ly, g.hkv) for r in range(g.b)]
        assert all(ctxs)
        expect = np.empty((g.rows, g.hkv, g.nb, g.slab), np.uint8)
        res = cuda.zeros(4, dtype=cuda.int32, device="cuda")
        sb_ids = [None] * 4
        for sb in range(4):                      # sub-batches 2 and 3 start in DRAM
            fill(L, g, rng, ctxs, expect, bf16=True,
                 rows=[(2 * sb + j, ctxs[2 * sb + j]) for j in range(2)])
            sb_ids[sb], _ = id_table(L, cuda, g, ctxs[2 * sb:2 * sb + 2])
            if sb >= 2:
                sd = _ids_dev(cuda, sb_ids[sb])
                assert L.orchkv_evict_batch_to_dram(sd.data_ptr(), None, sb_n, res.data_ptr()) == 0
                assert L.orchkv_sync() == 0
                assert res.cpu().tolist()[:2] == [sb_n, 0]
        all_ids, _ = id_table(L, cuda, g, ctxs)
        assert all_ids.max() < cap
        orc = O.OracleSched(cap, 0.9, 0.5, 0.3, 0.2, 50.0)
        for i in all_ids:
            orc.register(int(i))
        resident = [0, 1]
        for step in range(8):
            # score the resident sub-batches: logits N(0, 1.5), softmax per (row, q-head)
            reqs = [2 * sb + j for sb in resident for j in range(2)]
            ids_r, ids_rd = id_table(L, cuda, g, [ctxs[r] for r in reqs])
            logits = rng.normal(0, 1.5, (len(reqs) * g.ly, g.hq, g.t)).astype(np.float32)
            logits -= logits.max(-1, keepdims=True)
            p = np.exp(logits)
            probs = (p / p.sum(-1, keepdims=True)).astype(np.float32)
            pd = _dev(cuda, probs)
            assert L.tm_report_attn_probs(tm.ref, pd.data_ptr(), len(reqs) * g.ly, g.hq, g.hkv,
                                          g.t, g.tpb, None, ids_rd.data_ptr()) == 0
            assert L.tm_step_and_classify(tm.ref) == 0
            orc.update_batch(ids_r, O.score_blocks(probs, g.hq, g.hkv, g.tpb).reshape(-1))
            orc.step_done()
            orc.update_all()
            compare_sched(tm.state(), orc.state(), cap, all_ids, exact=False)

            # rotate: the older resident sub-batch out, the next one in
            out_sb, in_sb = step % 4, (step + 2) % 4
            assert resident[0] == out_sb
            ev, pr = np.sort(sb_ids[out_sb]), np.sort(sb_ids[in_sb])
            # the model starts from the device's state: earlier evicts may
            # have placed their victims on DRAM slabs in another (checked) order
            m = PoolModel(L, g, n_gpu, n_dram, maxb)
            ed, pd_ = _ids_dev(cuda, ev), _ids_dev(cuda, pr)
            assert L.orchkv_swap_batch(ed.data_ptr(), None, sb_n, pd_.data_ptr(), None, sb_n,
                                       res.data_ptr()) == 0
            assert L.orchkv_sync() == 0
            de, se = m.evict(ev)
            dp, sp = m.promote(pr)
            assert res.cpu().tolist() == [de, se, dp, sp] == [sb_n, 0, sb_n, 0]
            m.check(L, evicted=ev)
            runs, ce, zc, ov = C.c_uint32(), C.c_uint32(), C.c_uint32(), C.c_int()
            assert L.orchkv_last_promote_layout(C.byref(runs), C.byref(ce), C.byref(zc),
                                                C.byref(ov)) == 0
            assert ov.value == 1              # both directions of the host link at once
            resident = [resident[1], in_sb]
            if step % 4 == 3:
                tier = check_bytes(L, g, all_ids, expect, n_gpu, n_dram, maxb)
                assert int((tier == 0).sum()) == 2 * sb_n and int((tier == 1).sum()) == 2 * sb_n
        for c in ctxs:
            assert L.orchkv_request_destroy(c) == 0
    finally:
        L.orchkv_shutdown()
        tm.close()


# ---------------------------------------------------------------------------
# Llama-3-70B-shaped three tiers: GPU 20%, DRAM 50%, file 30%
# ---------------------------------------------------------------------------

def test_llama3_70b_three_tier_round_trip(cuda, oracle_mod, tmp_path):
    import orchkv_b200 as o
    O = oracle_mod
    L = o.lib()
    g = Geometry(ly=80, hq=64, hkv=8, d=128, tpb=64, t=2048, b=1)      # 20,480 slabs of 32 KB
    mbph, rid = g.nb, 7070                       # one (layer, head) = 1 MiB of the file
    n_gpu, n_dram, maxb, cap = g.n + 64, g.n // 2 + 64, 32768, 32768
    base = str(tmp_path / "orchkv_tiers")
    init(o, L, g, n_gpu, n_dram, dtype=0, max_blocks=maxb, mbph=mbph, base=base)
    tm = o.Manager(tracker_cap=cap, max_blocks=maxb, ema_lambda=0.9, alpha=0.5, beta=0.3,
                   gamma=0.2, recency_tau=50.0, cooldown_sec=0.0)
    try:
        assert L.orchkv_attach_scheduler(tm.ref) == 0
        rng = np.random.default_rng(5)
        ctx = L.orchkv_request_create(rid, g.ly, g.hkv)
        assert ctx
        expect = np.empty((g.rows, g.hkv, g.nb, g.slab), np.uint8)
        fill(L, g, rng, [ctx], expect, bf16=False)
        ids, ids_d = id_table(L, cuda, g, [ctx])
        assert ids.max() < cap
        pos = {int(b): j for j, b in enumerate(ids.tolist())}
        orc = O.OracleSched(cap, 0.9, 0.5, 0.3, 0.2, 50.0)
        for i in ids:
            orc.register(int(i))

        # one step: logits N(0, 2) + 0.002 * position, so older blocks run colder
        logits = (rng.normal(0, 2, (g.rows, g.hq, g.t)).astype(np.float32)
                  + (0.002 * np.arange(g.t)).astype(np.float32))
        logits -= logits.max(-1, keepdims=True)
        p = np.exp(logits)
        probs = (p / p.sum(-1, keepdims=True)).astype(np.float32)
        del logits, p
        pd = _dev(cuda, probs)
        assert L.tm_report_attn_probs(tm.ref, pd.data_ptr(), g.rows, g.hq, g.hkv, g.t, g.tpb,
                                      None, ids_d.data_ptr()) == 0
        assert L.tm_step_and_classify(tm.ref) == 0
        orc.update_batch(ids, O.score_blocks(probs, g.hq, g.hkv, g.tpb).reshape(-1))
        orc.step_done()
        orc.update_all()
        got = tm.state()
        compare_sched(got, orc.state(), cap, ids, exact=False)

        k_file, k_off = int(0.3 * g.n), g.n - int(0.2 * g.n)
        cold = select(L, cuda, tm, k_file, g.n)
        off = select(L, cuda, tm, k_off, g.n)
        assert np.array_equal(cold, O.select_coldest(got["hot"], got["c_active"], k_file))
        assert np.array_equal(off, O.select_coldest(got["hot"], got["c_active"], k_off))
        assert np.isin(cold, off).all()
        warm = np.setdiff1d(off, cold)

        def lhb(id_list):
            return np.array([g.lhb(pos[int(b)])[1:] for b in id_list], np.uint32).reshape(-1)

        # the coldest 30%: GPU -> DRAM -> file in one batch
        hres = (C.c_uint32 * 2)()
        cold_lhb = lhb(cold)
        assert L.orchkv_evict_cold_batch(ctx, cold_lhb.ctypes.data, len(cold), hres) == 0
        assert [hres[0], hres[1]] == [len(cold), 0]
        # the next 50%: GPU -> DRAM
        res = cuda.zeros(2, dtype=cuda.int32, device="cuda")
        wd, cd = _ids_dev(cuda, warm), _ids_dev(cuda, cold)
        assert L.orchkv_evict_batch_to_dram(wd.data_ptr(), None, len(warm), res.data_ptr()) == 0
        assert L.orchkv_sync() == 0
        assert res.cpu().tolist() == [len(warm), 0]
        tier = check_bytes(L, g, ids, expect, n_gpu, n_dram, maxb)
        assert [int((tier == t).sum()) for t in range(3)] == [g.n - k_off, len(warm), k_file]
        assert set(ids[tier == 2].tolist()) == set(cold.tolist())

        # the file: each cold slab at the reference's offset
        exp = expect.reshape(-1, g.slab)
        with open(os.path.join(base, f"req_{rid}"), "rb") as fh:
            data = np.frombuffer(fh.read(), np.uint8)
        for b in cold:
            j = pos[int(b)]
            _, l, h, bi = g.lhb(j)
            offset = ((l * g.hkv + h) * mbph + bi) * g.slab
            assert np.array_equal(data[offset:offset + g.slab], exp[j]), (l, h, bi)
        if O.ref_available():
            buf = np.zeros(g.slab, np.uint8)
            for b in cold[::61]:
                j = pos[int(b)]
                _, l, h, bi = g.lhb(j)
                assert O.ref().ref_storage_read(base.encode(), rid, g.ly, g.hkv, mbph, g.slab,
                                                l, h, bi, buf.ctypes.data) == 0
                assert np.array_equal(buf, exp[j])

        # back: DRAM -> GPU, then file -> DRAM -> GPU
        assert L.orchkv_promote_batch_to_gpu(wd.data_ptr(), None, len(warm), res.data_ptr()) == 0
        assert L.orchkv_sync() == 0
        assert res.cpu().tolist() == [len(warm), 0]
        assert L.orchkv_promote_batch_from_storage(ctx, cold_lhb.ctypes.data, len(cold),
                                                   hres) == 0
        assert [hres[0], hres[1]] == [len(cold), 0]
        tier = check_bytes(L, g, ids, expect, n_gpu, n_dram, maxb)
        assert int((tier == 1).sum()) == len(cold)
        assert L.orchkv_promote_batch_to_gpu(cd.data_ptr(), None, len(cold), res.data_ptr()) == 0
        assert L.orchkv_sync() == 0
        assert res.cpu().tolist() == [len(cold), 0]
        tier = check_bytes(L, g, ids, expect, n_gpu, n_dram, maxb)
        assert (tier == 0).all()
        assert L.orchkv_request_destroy(ctx) == 0
        assert not os.path.exists(os.path.join(base, f"req_{rid}"))
    finally:
        L.orchkv_shutdown()
        tm.close()
