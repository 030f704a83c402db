"""Large batched evicts take the staged path (HBM pack into a device ring +
copy-engine drain).  On a fragmented DRAM pool the popped slabs are sorted
and handed out in ascending order; runs of at least 1 MiB are drained by the
copy engine, shorter ones written zero-copy.  Checked against the
oracle's sequential per-block model: both free stacks identical, the set of
DRAM slabs used identical, each victim's slab = the sorted assignment, and
every slab's bytes identical to what it held on the GPU."""
import ctypes as C

import numpy as np
import pytest

from tests.test_gpu_pool import (ROW, SLAB, TPB, info, kv_data, locs, pool_state, read_dev,
                                 read_host)

pytestmark = pytest.mark.gpu

G_SLABS, D_SLABS = 7000, 6000


@pytest.fixture
def big(cuda):
    import orchkv_b200 as o
    L = o.lib()
    cfg = o.make_config(gpu_pool_bytes=G_SLABS * SLAB, dram_pool_bytes=D_SLABS * SLAB,
                        tokens_per_block=TPB, d_head=128, dtype=1, max_blocks_per_head=512)
    ext = o.OrchkvConfigExt()
    ext.max_blocks = 8192
    assert L.orchkv_init_ext(C.byref(cfg), C.byref(ext)) == 0
    yield o, L
    assert L.orchkv_shutdown() == 0


@pytest.mark.parametrize("fragment", [False, True])
def test_staged_evict_matches_sequential_model(big, cuda, fragment):
    from oracle import oracle as O
    o, L = big
    rng = np.random.default_rng(5 + fragment)
    H, n = 4, 16 * 400                                     # 1600 blocks per request
    reqs = []
    for r in range(4):                                     # 6400 blocks
        k, v = kv_data(rng, H, n)
        c = L.orchkv_request_create(r, 1, H)
        assert L.orchkv_prefill(c, 0, k.ctypes.data, v.ctypes.data, n) == 0
        reqs.append(c)
    loc, _ = locs(L, 8192)
    live = [i for i in range(8192) if (int(loc[i]) >> 29) == 0]
    if fragment:
        # scatter the DRAM free stack: per-block evicts of random blocks, then
        # promotes of a random subset, in random order
        ids = rng.choice(live, 1500, replace=False).astype(np.uint32)
        d = cuda.from_numpy(ids.view(np.int32)).cuda()
        assert L.orchkv_evict_batch_to_dram(d.data_ptr(), None, 1500, None) == 0
        back = rng.permutation(ids)[:1100].astype(np.uint32)
        d2 = cuda.from_numpy(back.view(np.int32)).cuda()
        assert L.orchkv_promote_batch_to_gpu(d2.data_ptr(), None, 1100, None) == 0
        assert L.orchkv_sync() == 0
    gpool = O.Pool(G_SLABS)
    dpool = O.Pool(D_SLABS)
    gpool.stack = pool_state(L, 0, G_SLABS)
    dpool.stack = pool_state(L, 1, D_SLABS)
    loc, state = locs(L, 8192)
    loc = loc.astype(np.int64).tolist()
    state = state.tolist()
    gbytes = read_dev(L.orchkv_gpu_pool_base(), G_SLABS * SLAB)
    dbytes = read_host(L.orchkv_dram_pool_base(), D_SLABS * SLAB)
    on_gpu = [i for i in range(8192) if (loc[i] >> 29) == 0]
    victims = np.sort(rng.choice(on_gpu, 4200, replace=False)).astype(np.uint32)
    dv = cuda.from_numpy(victims.view(np.int32)).cuda()
    res = cuda.zeros(2, dtype=cuda.int32, device="cuda")
    assert L.orchkv_evict_batch_to_dram(dv.data_ptr(), None, len(victims), res.data_ptr()) == 0
    assert L.orchkv_sync() == 0
    chunks = C.c_uint32()
    assert L.orchkv_last_migration_profile(None, None, C.byref(chunks), None) == 0
    assert chunks.value >= 1, "staged copy-engine path was not taken"
    runs, ce, zc = C.c_uint32(), C.c_uint32(), C.c_uint32()
    assert L.orchkv_last_evict_layout(C.byref(runs), C.byref(ce), C.byref(zc)) == 0
    assert ce.value >= 1
    if fragment:            # scattered slabs: short runs go zero-copy, long ones by copy engine
        assert runs.value > 100 and 0 < zc.value < len(victims)
    else:
        assert runs.value == 1 and zc.value == 0
    # sequential per-block model (src/api/orchkv_api.cu:353-389 in list order)
    d_before = list(dpool.stack)
    done, skipped = O.evict_batch(gpool, dpool, loc, state, None, victims.tolist(), gbytes,
                                  dbytes, SLAB)
    assert res.cpu().tolist() == [done, skipped]
    g2 = pool_state(L, 0, G_SLABS)
    dst2 = pool_state(L, 1, D_SLABS)
    assert g2 == gpool.stack and dst2 == dpool.stack
    popped = sorted(d_before[len(d_before) - done:])
    loc2, _ = locs(L, 8192)
    got = [int(loc2[v]) for v in victims[:done]]
    assert all(w >> 29 == 1 for w in got)
    assert [w & 0x1FFFFFFF for w in got] == popped          # ascending in list order
    dnow = read_host(L.orchkv_dram_pool_base(), D_SLABS * SLAB)
    for v, w in zip(victims[:done].tolist(), got):
        s = loc[v] & 0x1FFFFFFF                             # model: slab bytes by content
        want = dbytes[s * SLAB:(s + 1) * SLAB]
        ds = w & 0x1FFFFFFF
        assert np.array_equal(dnow[ds * SLAB:(ds + 1) * SLAB], want), v
    for c in reqs:
        assert L.orchkv_request_destroy(c) == 0
