"""Large batched promotes take the staged path: the promoted blocks' DRAM
slabs are sorted, runs of at least 1 MiB are copied host-to-device by the
copy engine and scattered by an unpack kernel, shorter runs are read
zero-copy.  orchkv_swap_batch evicts one list and promotes another with the
effect of the two batched calls in sequence, overlapping the two directions
of the host link when it can.

Every case is checked against the oracle's sequential per-block model
(src/api/orchkv_api.cu:353-428 in list order), started from the device's own
state: free stacks, every block's tier, and every block's bytes where it
now lives.  Only a staged evict's choice of which popped DRAM slab each
victim gets may differ from the model (ascending assignment), so DRAM slab
indices of evicted blocks are compared as the same set."""
import ctypes as C

import numpy as np
import pytest

from tests.test_gpu_pool import ROW, SLAB, TPB, kv_data, locs, pool_state, read_dev, read_host

pytestmark = pytest.mark.gpu

G_SLABS, D_SLABS, MAXB = 7000, 6000, 8192
MASK = 0x1FFFFFFF


@pytest.fixture
def sysm(cuda):
    import orchkv_b200 as o
    L = o.lib()
    cfg = o.make_config(gpu_pool_bytes=G_SLABS * SLAB, dram_pool_bytes=D_SLABS * SLAB,
                        tokens_per_block=TPB, d_head=128, dtype=1, max_blocks_per_head=512)
    ext = o.OrchkvConfigExt()
    ext.max_blocks = MAXB
    ext.staging_mb = 64               # > 4200 slabs of 8 KB: a whole evict fits
    assert L.orchkv_init_ext(C.byref(cfg), C.byref(ext)) == 0
    rng = np.random.default_rng(31)
    reqs = []
    for r in range(4):                                     # 6400 blocks of 8 KB
        k, v = kv_data(rng, 4, 16 * 400)
        c = L.orchkv_request_create(r, 1, 4)
        assert L.orchkv_prefill(c, 0, k.ctypes.data, v.ctypes.data, 16 * 400) == 0
        reqs.append(c)
    yield o, L, rng
    for c in reqs:
        assert L.orchkv_request_destroy(c) == 0
    assert L.orchkv_shutdown() == 0


class Model:
    """The oracle's pools, locations and bytes, loaded from the device."""

    def __init__(self, L):
        from oracle import oracle as O
        self.O = O
        self.g = O.Pool(G_SLABS)
        self.d = O.Pool(D_SLABS)
        self.g.stack = pool_state(L, 0, G_SLABS)
        self.d.stack = pool_state(L, 1, D_SLABS)
        loc, state = locs(L, MAXB)
        self.loc = loc.astype(np.int64).tolist()
        self.state = state.tolist()
        self.gb = read_dev(L.orchkv_gpu_pool_base(), G_SLABS * SLAB)
        self.db = read_host(L.orchkv_dram_pool_base(), D_SLABS * SLAB)

    def evict(self, ids):
        return self.O.evict_batch(self.g, self.d, self.loc, self.state, None, list(ids),
                                  self.gb, self.db, SLAB)

    def promote(self, ids):
        return self.O.promote_batch(self.g, self.d, self.loc, self.state, list(ids), self.gb,
                                    self.db, SLAB)


def check(L, m, evicted=(), exact_dram_stack=True):
    """Device == model: stacks, tiers, bytes; evicted blocks' DRAM slabs as a set."""
    g2, d2 = pool_state(L, 0, G_SLABS), pool_state(L, 1, D_SLABS)
    assert g2 == m.g.stack
    if exact_dram_stack:
        assert d2 == m.d.stack
    else:
        assert sorted(d2) == sorted(m.d.stack)
    loc, _ = locs(L, MAXB)
    gb = read_dev(L.orchkv_gpu_pool_base(), G_SLABS * SLAB)
    db = read_host(L.orchkv_dram_pool_base(), D_SLABS * SLAB)
    ev = set(int(x) for x in evicted)
    dev_set, mod_set = [], []
    for i in range(MAXB):
        w, mw = int(loc[i]), m.loc[i]
        t, mt = w >> 29, mw >> 29
        assert t == mt, i
        if t not in (0, 1):
            continue
        s, ms = w & MASK, mw & MASK
        pool, mpool = (gb, m.gb) if t == 0 else (db, m.db)
        assert np.array_equal(pool[s * SLAB:(s + 1) * SLAB], mpool[ms * SLAB:(ms + 1) * SLAB]), i
        if t == 1 and i in ev:
            dev_set.append(s)
            mod_set.append(ms)
        else:
            assert s == ms, i
    assert sorted(dev_set) == sorted(mod_set)


def on_tier(L, tier):
    loc, _ = locs(L, MAXB)
    return [i for i in range(MAXB) if (int(loc[i]) >> 29) == tier]


def dev_ids(cuda, ids):
    return cuda.from_numpy(np.asarray(ids, np.uint32).view(np.int32).copy()).cuda()


def promote_layout(L):
    runs, ce, zc, ov = C.c_uint32(), C.c_uint32(), C.c_uint32(), C.c_int()
    assert L.orchkv_last_promote_layout(C.byref(runs), C.byref(ce), C.byref(zc),
                                        C.byref(ov)) == 0
    return runs.value, ce.value, zc.value, ov.value


@pytest.mark.parametrize("order", ["same", "random_subset"])
def test_staged_promote_matches_sequential_model(sysm, cuda, order):
    o, L, rng = sysm
    victims = sorted(rng.choice(on_tier(L, 0), 4200, replace=False).tolist())
    vd = dev_ids(cuda, victims)
    assert L.orchkv_evict_batch_to_dram(vd.data_ptr(), None, 4200, None) == 0
    assert L.orchkv_sync() == 0
    m = Model(L)
    if order == "same":           # evicted together, promoted together: long source runs
        back = victims
    else:                         # a scattered subset in random order: short runs
        back = rng.permutation(victims)[:2600].tolist()
    res = cuda.zeros(2, dtype=cuda.int32, device="cuda")
    bd = dev_ids(cuda, back)
    assert L.orchkv_promote_batch_to_gpu(bd.data_ptr(), None, len(back),
                                         res.data_ptr()) == 0
    assert L.orchkv_sync() == 0
    done, skipped = m.promote(back)
    assert res.cpu().tolist() == [done, skipped] and done == len(back)
    check(L, m)
    runs, ce, zc, _ = promote_layout(L)
    if order == "same":
        assert ce >= 1 and zc == 0
    else:
        assert runs > 100 and zc > 0


@pytest.mark.parametrize("case", ["disjoint", "overlapping", "small"])
def test_swap_equals_evict_then_promote(sysm, cuda, case):
    o, L, rng = sysm
    # blocks evicted earlier, to be promoted by the swap
    first = sorted(rng.choice(on_tier(L, 0), 2500, replace=False).tolist())
    fd = dev_ids(cuda, first)
    assert L.orchkv_evict_batch_to_dram(fd.data_ptr(), None, len(first),
                                        None) == 0
    assert L.orchkv_sync() == 0
    m = Model(L)
    gpu_now = on_tier(L, 0)
    if case == "small":
        ev = sorted(rng.choice(gpu_now, 500, replace=False).tolist())
        pr = first[:300]
    else:
        ev = sorted(rng.choice(gpu_now, 3000, replace=False).tolist())
        pr = list(first)
        if case == "overlapping":   # some blocks evicted and promoted in the same call
            pr = pr[:2000] + ev[:300]
    res = cuda.zeros(4, dtype=cuda.int32, device="cuda")
    # both lists held in their own tensors: a temporary freed after
    # data_ptr() could hand its memory to the next list before the call reads it
    ed, pd = dev_ids(cuda, ev), dev_ids(cuda, pr)
    assert L.orchkv_swap_batch(ed.data_ptr(), None, len(ev), pd.data_ptr(), None, len(pr),
                               res.data_ptr()) == 0
    assert L.orchkv_sync() == 0
    de, se = m.evict(ev)
    dp, sp = m.promote(pr)
    assert res.cpu().tolist() == [de, se, dp, sp]
    # a staged evict's assignment changes which slabs its overlap blocks
    # return to the DRAM stack, not which set
    check(L, m, evicted=ev, exact_dram_stack=case != "overlapping")
    ov = promote_layout(L)[3]
    assert ov == (1 if case == "disjoint" else 0)
