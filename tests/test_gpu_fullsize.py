"""The benchmark's own decode step at its full size, checked.

bench.py's Workload is the Qwen2.5-7B-shaped GQA batch on one GPU: 32
requests x 8192 tokens, 28 layers, 28 query / 4 KV heads, d_head 128, bf16,
16-token blocks -- 1,835,008 slabs of 8 KB, 14 GiB, with the coldest 5% held
in the pinned DRAM tier.  One step appends a token per (request, layer),
scores, classifies, selects the coldest 25% of the HBM-resident blocks
(458,752) and the 5% prefetch set (91,750), and swaps them.  Here that step
runs through the same code and is checked at that size:

* tracker sums of 64 seeded rows (64 x 4 KV heads x 512 blocks) within
  1e-5 of the oracle's reduction of the same probabilities;
* the victim list equal to the oracle's coldest-k, and the prefetch list to
  the oracle's prefetch rule, both fed the GPU's own hotness / EMA;
* every evicted block's DRAM bytes equal its GPU bytes before the step, and
  every promoted block's GPU bytes its DRAM bytes before the step, compared
  as per-slab 64-bit checksums: a device kernel (orchkv_block_checksums) on
  one side, numpy over the pinned DRAM pool on the other;
* the round trip back (the victims promoted, the prefetch set evicted again)
  bit-exact by the same checksums.

It runs twice: with the bench's staging (a whole evict packed up front, the
swap overlapping both copy directions) and with the library's default
three-slot staging ring, where the 14-chunk evict reuses slots and the
restore's 14-chunk promote reuses the three promote-ring slots -- the slot
waits of both staged paths.  (The reference checks migrated bytes with
seed^i words, test/test_gpu_dram.cu:40-55; selection and scoring follow
python/orchkv/fast_kvcache_manager.py:221-341.)"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL = 1e-5
SAMPLE_ROWS = 64
KV_STATE_MIGRATING = 5


def _mults(words):
    """m_i = splitmix64 output(i) | 1, the checksum's word multipliers."""
    z = np.arange(words, dtype=np.uint64) + np.uint64(0x9E3779B97F4A7C15)
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    z = z ^ (z >> np.uint64(31))
    return z | np.uint64(1)


def host_checksums(base, slab, n_slabs, slabs, chunk=8192):
    """The device kernel's checksum, recomputed on the host for slabs of a
    pool in host memory (the pinned DRAM tier)."""
    words = slab // 8
    m = _mults(words)
    raw = (C.c_char * (n_slabs * slab)).from_address(base)
    pool = np.frombuffer(raw, dtype=np.uint64).reshape(n_slabs, words)
    out = np.empty(len(slabs), np.uint64)
    slabs = np.asarray(slabs, np.int64)
    for i in range(0, len(slabs), chunk):
        rows = pool[slabs[i:i + chunk]]
        out[i:i + chunk] = (rows * m).sum(axis=1, dtype=np.uint64)
    return out


def dev_checksums(torch, L, ids_dev):
    n = ids_dev.numel()
    out = torch.empty(n, dtype=torch.int64, device="cuda")
    tier = torch.empty(n, dtype=torch.uint8, device="cuda")
    assert L.orchkv_block_checksums(C.c_void_p(ids_dev.data_ptr()), n,
                                    C.c_void_p(out.data_ptr()), C.c_void_p(tier.data_ptr())) == 0
    assert L.orchkv_sync() == 0
    return out.cpu().numpy().view(np.uint64), tier.cpu().numpy()


def block_locs(L, max_blocks):
    loc = np.zeros(max_blocks, np.uint32)
    state = np.zeros(max_blocks, np.uint8)
    assert L.orchkv_read_block_locs(loc.ctypes.data, state.ctypes.data) == 0
    return loc.astype(np.int64), state


def test_checksum_matches_host_definition(cuda):
    """The device checksum equals the host restatement on a small pool, for
    blocks in HBM and in the DRAM tier; blocks in neither give 0 / tier 7."""
    import orchkv_b200 as okv
    torch = cuda
    L = okv.lib()
    tpb, d = 16, 128
    slab = tpb * d * 2 * 2
    cfg = okv.make_config(gpu_pool_bytes=64 * slab, dram_pool_bytes=64 * slab,
                          tokens_per_block=tpb, d_head=d, dtype=1, max_blocks_per_head=16)
    ext = okv.OrchkvConfigExt()
    ext.max_blocks = 256
    assert L.orchkv_init_ext(C.byref(cfg), C.byref(ext)) == 0
    try:
        c = L.orchkv_request_create(1, 2, 2)
        g = torch.Generator(device="cuda").manual_seed(5)
        for layer in range(2):
            kv = torch.randn(2, 2, 8 * tpb, d, generator=g, device="cuda", dtype=torch.bfloat16)
            assert L.orchkv_prefill(c, layer, kv[0].data_ptr(), kv[1].data_ptr(), 8 * tpb) == 0
        n = 2 * 2 * 8
        ids = torch.arange(n, dtype=torch.int32, device="cuda")
        gpu_sum, tier = dev_checksums(torch, L, ids)
        assert (tier == 0).all()
        ev = ids[::3].contiguous()
        res = torch.zeros(2, dtype=torch.int32, device="cuda")
        assert L.orchkv_evict_batch_to_dram(C.c_void_p(ev.data_ptr()), None, ev.numel(),
                                            C.c_void_p(res.data_ptr())) == 0
        assert L.orchkv_sync() == 0
        loc, _ = block_locs(L, 256)
        got, tier = dev_checksums(torch, L, ids)
        assert np.array_equal(got, gpu_sum)
        on_dram = np.nonzero(tier == 1)[0]
        assert len(on_dram) == ev.numel()
        host = host_checksums(L.orchkv_dram_pool_base(), slab, 64, loc[on_dram] & 0x1FFFFFFF)
        assert np.array_equal(host, gpu_sum[on_dram])
        # a flipped bit in the DRAM copy changes the checksum
        p = L.orchkv_dram_pool_base() + int(loc[on_dram[0]] & 0x1FFFFFFF) * slab + 1000
        C.c_uint8.from_address(p).value ^= 0x10
        got2, _ = dev_checksums(torch, L, ids)
        assert got2[on_dram[0]] != gpu_sum[on_dram[0]]
        C.c_uint8.from_address(p).value ^= 0x10
        bogus = torch.tensor([n + 5, 1 << 30], dtype=torch.int32, device="cuda")
        z, t = dev_checksums(torch, L, bogus)
        assert z.tolist() == [0, 0] and t.tolist() == [7, 7]
        assert L.orchkv_request_destroy(c) == 0
    finally:
        L.orchkv_shutdown()


@pytest.mark.parametrize("staging", ["whole", "ring"])
def test_full_size_decode_step(cuda, oracle_mod, staging):
    import bench
    import orchkv_b200 as okv
    torch = cuda
    O = oracle_mod
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    wl = bench.Workload(torch, okv, 0, 1, staging=staging)
    L = wl.L
    cap = wl.tm.cap
    maxb = L.orchkv_max_blocks()
    rng = np.random.default_rng(11)
    rows = np.sort(rng.choice(wl.rows, SAMPLE_ROWS, replace=False))
    seen = {}

    def check(phase):
        torch.cuda.synchronize()
        if phase == "scored":
            st = wl.tm.state()
            ids = wl.ids.view(wl.rows, wl.Hkv, wl.nb)[torch.as_tensor(rows, device="cuda")]
            ids = ids.cpu().numpy().view(np.uint32).astype(np.int64)
            mass = O.score_blocks(wl.probs[torch.as_tensor(rows, device="cuda")].cpu().numpy(),
                                  wl.Hq, wl.Hkv, wl.tpb)
            got = st["sum"][ids & (cap - 1)]
            assert ids.size == SAMPLE_ROWS * wl.Hkv * wl.nb
            assert np.all(np.abs(got - mass) <= REL * np.abs(mass)), \
                float(np.max(np.abs(got - mass) / np.abs(mass)))
            seen["scored"] = ids.size
            return
        assert phase == "selected"
        st = wl.tm.state()
        loc, state = block_locs(L, maxb)
        n = min(cap, maxb)
        tier = (loc[:n] >> 29).astype(np.uint8)
        tier[tier > 3] = 4                                   # no block: TIER_NONE
        cnt = wl.counts.cpu().numpy().view(np.uint32)
        victims = wl.victims[:int(cnt[0])].cpu().numpy().view(np.uint32).astype(np.int64)
        pref = wl.pref[:int(cnt[1])].cpu().numpy().view(np.uint32).astype(np.int64)
        elig = (st["t_active"][:n] & st["c_active"][:n] & (tier == 0) &
                (state[:n] != KV_STATE_MIGRATING)).astype(np.uint8)
        want_v = O.select_coldest(st["hot"][:n], elig, wl.k_evict)
        assert len(victims) == wl.k_evict == len(want_v)
        assert np.array_equal(victims, want_v)
        want_p = O.select_prefetch(st["ema"][:n], st["t_active"][:n], tier, 0.0, 0.0,
                                   wl.k_promote)
        assert len(pref) == len(want_p) > 0
        assert np.array_equal(pref, want_p)
        # bytes before the move: victims from HBM (device), the prefetch set
        # from the DRAM tier (host)
        assert (tier[victims] == 0).all() and (tier[pref] == 1).all()
        seen["v_ids"] = torch.as_tensor(victims.astype(np.int32), device="cuda")
        seen["p_ids"] = torch.as_tensor(pref.astype(np.int32), device="cuda")
        seen["v_sum"], t = dev_checksums(torch, L, seen["v_ids"])
        assert (t == 0).all()
        seen["p_sum"] = host_checksums(L.orchkv_dram_pool_base(), wl.slab, _dram_total(L),
                                       loc[pref] & 0x1FFFFFFF)
        seen["victims"], seen["pref"] = victims, pref

    try:
        wl.step(check=check)
        torch.cuda.synchronize()
        assert "scored" in seen and "v_sum" in seen
        c = wl.counts.cpu().numpy().view(np.uint32)
        victims, pref = seen["victims"], seen["pref"]
        assert c[2] == len(victims) and c[3] == 0 and c[4] == len(pref) and c[5] == 0
        # which staged path ran
        play = [C.c_uint32() for _ in range(3)] + [C.c_int()]
        L.orchkv_last_promote_layout(*[C.byref(x) for x in play])
        chunks = C.c_uint32()
        L.orchkv_last_pack_chunks(None, 0, C.byref(chunks))
        ring_slabs = (256 << 20) // wl.slab
        assert chunks.value == (len(victims) + ring_slabs - 1) // ring_slabs
        assert chunks.value > 3
        assert bool(play[3].value) == (staging == "whole")
        # evicted: DRAM bytes (host) == GPU bytes before (device)
        loc, _ = block_locs(L, maxb)
        assert (loc[victims] >> 29 == 1).all() and (loc[pref] >> 29 == 0).all()
        d_total = _dram_total(L)
        got_v = host_checksums(L.orchkv_dram_pool_base(), wl.slab, d_total,
                               loc[victims] & 0x1FFFFFFF)
        bad = np.nonzero(got_v != seen["v_sum"])[0]
        assert len(bad) == 0, (len(bad), victims[bad[:8]].tolist())
        # promoted: GPU bytes (device) == DRAM bytes before (host)
        got_p, t = dev_checksums(torch, L, seen["p_ids"])
        assert (t == 0).all()
        assert np.array_equal(got_p, seen["p_sum"])

        # the way back: every off-GPU block promoted (14 chunks through the
        # three promote-ring slots), then the prefetch set evicted again
        tm = wl.tm.ref
        assert L.tm_select_prefetch(tm, 1 << 21, 0.0, 0.0, wl._ptr(wl.pref),
                                    wl._ptr(wl.counts, 32)) == 0
        assert L.orchkv_promote_batch_to_gpu(wl._ptr(wl.pref), wl._ptr(wl.counts, 32), 1 << 21,
                                             wl._ptr(wl.counts, 36)) == 0
        assert L.orchkv_sync() == 0
        c = wl.counts.cpu().numpy().view(np.uint32)
        assert c[8] == c[9] == len(victims)
        n_up = C.c_uint32()
        L.orchkv_last_unpack_chunks(None, None, 0, C.byref(n_up))
        assert n_up.value > 3
        back, t = dev_checksums(torch, L, seen["v_ids"])
        assert (t == 0).all()
        assert np.array_equal(back, seen["v_sum"])
        wl._evict_reserve()
        assert L.orchkv_sync() == 0
        loc, _ = block_locs(L, maxb)
        again = host_checksums(L.orchkv_dram_pool_base(), wl.slab, d_total,
                               loc[pref] & 0x1FFFFFFF)
        assert np.array_equal(again, seen["p_sum"])
    finally:
        wl.close()
        torch.cuda.set_stream(torch.cuda.default_stream())


def _dram_total(L):
    import orchkv_b200 as okv
    st = okv.OrchkvStats()
    assert L.orchkv_get_stats(C.byref(st)) == 0
    return int(st.dram_slabs_total)
