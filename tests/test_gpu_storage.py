"""Storage tier through the C ABI: two-hop orchkv_evict_cold and
orchkv_promote_from_storage round trips bit-exact, files in the reference's
layout (offset = ((layer*H + head)*max_blocks_per_head + block)*slab,
src/tiered_store/orchfs_tier.h:89-97) — read back with the reference's own
orchfs_tier_read where oracle/_ref is present — and the reference's error
codes (src/api/orchkv_api.cu:432-516)."""
import ctypes as C
import os

import numpy as np
import pytest

from tests.test_gpu_pool import (DRAM_SLABS, GPU_SLABS, HALF, ROW, SLAB, TPB, expected_slab,
                                 info, kv_data, read_dev, read_host)

pytestmark = pytest.mark.gpu

BASE = "/dev/shm/orchkv_b200_test_storage"
MBPH = 32


@pytest.fixture
def sp(cuda):
    import orchkv_b200 as o
    L = o.lib()
    cfg = o.make_config(gpu_pool_bytes=GPU_SLABS * SLAB, dram_pool_bytes=DRAM_SLABS * SLAB,
                        tokens_per_block=TPB, d_head=128, dtype=1, max_blocks_per_head=MBPH)
    cfg.orchfs_base_dir = BASE.encode()
    ext = o.OrchkvConfigExt()
    ext.max_blocks = 512
    assert L.orchkv_init_ext(C.byref(cfg), C.byref(ext)) == 0
    yield o, L
    assert L.orchkv_shutdown() == 0


def _file_tier_counts(L):
    """(total_writes, total_reads) of the orchkv_orchfs_tier() snapshot, read
    at the reference's field offsets (src/tiered_store/orchfs_tier.h:40-51)."""
    p = L.orchkv_orchfs_tier()
    assert p
    w = (C.c_uint64 * 2).from_address(p + 272)
    return int(w[0]), int(w[1])


def test_two_hop_round_trip_and_file_layout(sp, cuda):
    o, L = sp
    from oracle import oracle as O
    rng = np.random.default_rng(21)
    H, n, rid = 2, 64, 4242
    k, v = kv_data(rng, H, n)
    ctx = L.orchkv_request_create(rid, 2, H)
    assert L.orchkv_prefill(ctx, 1, k.ctypes.data, v.ctypes.data, n) == 0
    path = os.path.join(BASE, f"req_{rid}")
    assert os.path.exists(path)
    cold = [(1, 0, 1), (1, 1, 3), (1, 1, 0)]
    for (l, h, b) in cold:
        assert L.orchkv_evict_cold(ctx, l, h, b) == 0            # GPU -> DRAM -> file
        rc, bid, tier, slab, st, tok = info(L, ctx, l, h, b)
        assert tier == 2 and st == 4                             # TIER_NVM, KV_STATE_COLD
    s = o.OrchkvStats()
    L.orchkv_get_stats(C.byref(s))
    assert s.dram_slabs_used == 0 and s.gpu_slabs_used == 2 * 4 - 3
    assert _file_tier_counts(L) == (3, 0)            # one write per slab, as the reference
    # the file holds each slab at the reference offset
    with open(path, "rb") as fh:
        data = fh.read()
    for (l, h, b) in cold:
        off = ((l * H + h) * MBPH + b) * SLAB
        assert data[off:off + SLAB] == expected_slab(k, v, h, b).tobytes()
        if O.ref_available():
            buf = np.zeros(SLAB, np.uint8)
            assert O.ref().ref_storage_read(BASE.encode(), rid, 2, H, MBPH, SLAB, l, h, b,
                                            buf.ctypes.data) == 0
            assert np.array_equal(buf, expected_slab(k, v, h, b))
    # storage -> DRAM, then get_kv_block brings the other ones straight to GPU
    l, h, b = cold[0]
    assert L.orchkv_promote_from_storage(ctx, l, h, b) == 0
    rc, bid, tier, slab, st, tok = info(L, ctx, l, h, b)
    assert tier == 1 and st == 3
    assert np.array_equal(read_host(L.orchkv_dram_pool_base() + slab * SLAB, SLAB),
                          expected_slab(k, v, h, b))
    assert _file_tier_counts(L) == (3, 1)
    for (l, h, b) in cold:
        kp, vp = C.c_void_p(), C.c_void_p()
        assert L.orchkv_get_kv_block(ctx, l, h, b, C.byref(kp), C.byref(vp)) == 0
        assert vp.value - kp.value == HALF
        assert np.array_equal(read_dev(kp.value, SLAB), expected_slab(k, v, h, b))
    L.orchkv_get_stats(C.byref(s))
    assert s.gpu_slabs_used == 8 and s.dram_slabs_used == 0
    assert _file_tier_counts(L) == (3, 3)            # get_kv_block read the other two
    assert L.orchkv_request_destroy(ctx) == 0
    assert not os.path.exists(path)                             # removed with the request


def test_storage_error_codes(sp, cuda):
    o, L = sp
    rng = np.random.default_rng(3)
    H = 2
    k, v = kv_data(rng, H, 32)
    ctx = L.orchkv_request_create(77, 1, H)
    assert L.orchkv_prefill(ctx, 0, k.ctypes.data, v.ctypes.data, 32) == 0
    assert L.orchkv_evict_to_storage(ctx, 0, 0, 0) == -8       # on GPU: ERR_STATE
    assert L.orchkv_promote_from_storage(ctx, 0, 0, 0) == -8   # not on storage
    assert L.orchkv_evict_to_storage(ctx, 0, 0, 7) == -3       # ERR_NOT_FOUND
    assert L.orchkv_evict_to_dram(ctx, 0, 1, 1) == 0
    assert L.orchkv_set_block_flags(ctx, 0, 1, 1, 0x01) == 0
    assert L.orchkv_evict_to_storage(ctx, 0, 1, 1) == -7       # pinned: ERR_LOCKED
    assert L.orchkv_set_block_flags(ctx, 0, 1, 1, 0x00) == 0
    assert L.orchkv_evict_to_storage(ctx, 0, 1, 1) == 0
    assert L.orchkv_evict_cold(ctx, 0, 1, 1) == -8             # already cold
    assert L.orchkv_request_destroy(ctx) == 0


def test_storage_io_failures_leave_state_unchanged(sp, cuda):
    """Host-side fault injection (no GPU fault): the request's file is a link
    to /dev/full (every write fails with ENOSPC), then a truncated file
    (every read comes up short).  The failed calls return ORCHKV_ERR_IO and
    leave the blocks, the stacks and the counters as they were
    (src/api/orchkv_api.cu:432-504 restores the same way)."""
    o, L = sp
    rng = np.random.default_rng(8)
    H, rid = 2, 9191
    os.makedirs(BASE, exist_ok=True)
    path = os.path.join(BASE, f"req_{rid}")
    if os.path.lexists(path):
        os.unlink(path)
    os.symlink("/dev/full", path)
    k, v = kv_data(rng, H, 64)
    ctx = L.orchkv_request_create(rid, 1, H)
    assert ctx
    assert L.orchkv_prefill(ctx, 0, k.ctypes.data, v.ctypes.data, 64) == 0
    assert L.orchkv_evict_to_dram(ctx, 0, 0, 1) == 0
    assert L.orchkv_evict_to_dram(ctx, 0, 1, 2) == 0

    def snap():
        g = np.zeros(GPU_SLABS, np.uint32)
        d = np.zeros(DRAM_SLABS, np.uint32)
        tg, td = C.c_uint32(), C.c_uint32()
        assert L.orchkv_read_pool(0, g.ctypes.data, C.byref(tg)) == 0
        assert L.orchkv_read_pool(1, d.ctypes.data, C.byref(td)) == 0
        return (g[:tg.value].tolist(), d[:td.value].tolist(),
                [info(L, ctx, 0, h, b) for h in range(H) for b in range(4)])

    before = snap()
    assert L.orchkv_evict_to_storage(ctx, 0, 0, 1) == -6          # ERR_IO
    lhb = np.array([0, 0, 1, 0, 1, 2], np.uint32)
    res = (C.c_uint32 * 2)()
    assert L.orchkv_evict_batch_to_storage(ctx, lhb.ctypes.data, 2, res) == -6
    cold = np.array([0, 0, 3], np.uint32)
    assert L.orchkv_evict_cold_batch(ctx, cold.ctypes.data, 1, res) == -6
    assert snap() == before
    assert L.orchkv_request_destroy(ctx) == 0

    # reads: a real file, evicted, then cut short under the library
    ctx = L.orchkv_request_create(rid + 1, 1, H)
    assert L.orchkv_prefill(ctx, 0, k.ctypes.data, v.ctypes.data, 64) == 0
    assert L.orchkv_evict_cold(ctx, 0, 0, 1) == 0
    assert L.orchkv_evict_cold(ctx, 0, 1, 3) == 0
    before = snap()
    os.truncate(os.path.join(BASE, f"req_{rid + 1}"), 0)
    assert L.orchkv_promote_from_storage(ctx, 0, 0, 1) == -6
    lhb = np.array([0, 0, 1, 0, 1, 3], np.uint32)
    assert L.orchkv_promote_batch_from_storage(ctx, lhb.ctypes.data, 2, res) == -6
    assert snap() == before
    assert L.orchkv_request_destroy(ctx) == 0


def _storage_scenario(o, L, batched):
    """One run of evict-to-storage / evict_cold / promote-from-storage lists,
    as batches or as the per-block calls in list order; returns everything
    observable."""
    rng = np.random.default_rng(31)
    H, n, rid = 2, 16 * 12, 777
    ctx = L.orchkv_request_create(rid, 2, H)
    for layer in range(2):
        k, v = kv_data(rng, H, n)
        assert L.orchkv_prefill(ctx, layer, k.ctypes.data, v.ctypes.data, n) == 0
    for (l, h, b) in [(0, 0, 3), (0, 0, 4), (1, 1, 7), (1, 0, 2), (0, 1, 9)]:
        assert L.orchkv_evict_to_dram(ctx, l, h, b) == 0
    assert L.orchkv_set_block_flags(ctx, 1, 0, 2, 1) == 0          # pinned, on DRAM

    def run(fn_batch, fn_one, triples):
        if batched:
            arr = np.array(triples, np.uint32).reshape(-1)
            res = (C.c_uint32 * 2)()
            assert fn_batch(ctx, arr.ctypes.data, len(triples), res) == 0
            return [res[0], res[1]]
        ok = sum(1 for t in triples if fn_one(ctx, *t) == 0)
        return [ok, len(triples) - ok]

    out = []
    # DRAM blocks go; a GPU block, a repeat, a missing block, a pinned one do not
    out.append(run(L.orchkv_evict_batch_to_storage, L.orchkv_evict_to_storage,
                   [(0, 0, 4), (1, 1, 7), (0, 0, 5), (0, 0, 4), (1, 1, 30), (1, 0, 2),
                    (0, 0, 3), (0, 1, 9)]))
    # two hops for GPU blocks, 8 consecutive ones of (0, 1) among them
    out.append(run(L.orchkv_evict_cold_batch, L.orchkv_evict_cold,
                   [(0, 1, i) for i in range(8)] + [(1, 0, 2), (0, 0, 3), (1, 1, 11),
                                                    (0, 1, 3)]))
    # back from storage: some of them, a repeat, a DRAM block, a GPU block
    out.append(run(L.orchkv_promote_batch_from_storage, L.orchkv_promote_from_storage,
                   [(0, 1, 5), (0, 0, 4), (0, 1, 2), (0, 1, 5), (1, 0, 2), (0, 0, 0),
                    (1, 1, 7), (0, 1, 0)]))
    g = np.zeros(GPU_SLABS, np.uint32)
    d = np.zeros(DRAM_SLABS, np.uint32)
    tg, td = C.c_uint32(), C.c_uint32()
    assert L.orchkv_read_pool(0, g.ctypes.data, C.byref(tg)) == 0
    assert L.orchkv_read_pool(1, d.ctypes.data, C.byref(td)) == 0
    blocks = [info(L, ctx, l, h, b) for l in range(2) for h in range(H) for b in range(12)]
    dram = read_host(L.orchkv_dram_pool_base(), DRAM_SLABS * SLAB)
    dram_used = {s: dram[s * SLAB:(s + 1) * SLAB].tobytes() for (_, _, t, s, _, _) in blocks
                 if t == 1}
    with open(os.path.join(BASE, f"req_{rid}"), "rb") as fh:
        data = fh.read()
    files = {(l, h, b): data[((l * H + h) * MBPH + b) * SLAB:((l * H + h) * MBPH + b + 1) * SLAB]
             for l in range(2) for h in range(H) for b in range(12)
             if blocks[(l * H + h) * 12 + b][2] == 2}
    counts = _file_tier_counts(L)
    assert L.orchkv_request_destroy(ctx) == 0
    return out, g[:tg.value].tolist(), d[:td.value].tolist(), blocks, dram_used, files, counts


def test_storage_batches_equal_per_block_calls(cuda):
    import orchkv_b200 as o
    L = o.lib()
    results = []
    for batched in (True, False):
        cfg = o.make_config(gpu_pool_bytes=GPU_SLABS * SLAB, dram_pool_bytes=DRAM_SLABS * SLAB,
                            tokens_per_block=TPB, d_head=128, dtype=1, max_blocks_per_head=MBPH)
        cfg.orchfs_base_dir = BASE.encode()
        ext = o.OrchkvConfigExt()
        ext.max_blocks = 512
        assert L.orchkv_init_ext(C.byref(cfg), C.byref(ext)) == 0
        try:
            results.append(_storage_scenario(o, L, batched))
        finally:
            assert L.orchkv_shutdown() == 0
    b, p = results
    assert b[0] == p[0]
    assert b[0] == [[4, 4], [9, 3], [5, 3]]
    assert b[-1] == (4 + 9, 5)               # file-tier counters: one per slab moved
    for x, y in zip(b[1:], p[1:]):
        assert x == y


def test_two_hop_batch_spanning_staging_chunks(cuda):
    """One orchkv_evict_cold_batch of 78,643 blocks of 8 KB (614 MB, three
    256 MB staging chunks: the next chunk is gathered while the IO workers
    write the current one), listed in a shuffled order, then
    orchkv_promote_batch_from_storage and a promote back to HBM: every
    block's checksum equals its checksum before, and the counts and tiers
    are those of the per-block calls."""
    import orchkv_b200 as o
    torch = cuda
    L = o.lib()
    Ly, H, T, tpb, d = 48, 8, 4096, 16, 128
    nb = T // tpb
    n = Ly * H * nb
    slab = tpb * d * 2 * 2
    cfg = o.make_config(gpu_pool_bytes=(n + 64) * slab, dram_pool_bytes=(n + 64) * slab,
                        tokens_per_block=tpb, d_head=d, dtype=1, max_blocks_per_head=nb + 8)
    cfg.orchfs_base_dir = (BASE + "_chunks").encode()
    cfg.orchfs_io_workers = 8
    ext = o.OrchkvConfigExt()
    ext.max_blocks = 1 << 17
    assert L.orchkv_init_ext(C.byref(cfg), C.byref(ext)) == 0
    try:
        ctx = L.orchkv_request_create(777, Ly, H)
        g = torch.Generator(device="cuda").manual_seed(31)
        for layer in range(Ly):
            kv = torch.randn(2, H, T, d, generator=g, device="cuda", dtype=torch.bfloat16)
            assert L.orchkv_prefill(ctx, layer, kv[0].data_ptr(), kv[1].data_ptr(), T) == 0
        arr = (C.c_void_p * 1)(ctx)
        ids = torch.empty(n, dtype=torch.int32, device="cuda")
        assert L.orchkv_block_id_table(arr, 1, T, C.c_void_p(ids.data_ptr())) == 0
        sums = torch.empty(n, dtype=torch.int64, device="cuda")
        tier = torch.empty(n, dtype=torch.uint8, device="cuda")

        def checksums():
            assert L.orchkv_block_checksums(C.c_void_p(ids.data_ptr()), n,
                                            C.c_void_p(sums.data_ptr()),
                                            C.c_void_p(tier.data_ptr())) == 0
            assert L.orchkv_sync() == 0
            return sums.cpu().numpy().copy(), tier.cpu().numpy().copy()

        before, t0 = checksums()
        assert (t0 == 0).all()
        rng = np.random.default_rng(5)
        pick = rng.permutation(n)[: n * 4 // 5]                 # 78,643 blocks, shuffled
        lay, rem = np.divmod(pick, H * nb)
        head, blk = np.divmod(rem, nb)
        lhb = np.ascontiguousarray(np.stack([lay, head, blk], 1).astype(np.uint32).reshape(-1))
        res = (C.c_uint32 * 2)()
        assert L.orchkv_evict_cold_batch(ctx, lhb.ctypes.data, len(pick), res) == 0
        assert list(res) == [len(pick), 0]
        _, t1 = checksums()
        assert (t1[pick] == 7).all()                            # in no GPU or DRAM slab
        assert int((t1 == 0).sum()) == n - len(pick)
        assert L.orchkv_promote_batch_from_storage(ctx, lhb.ctypes.data, len(pick), res) == 0
        assert list(res) == [len(pick), 0]
        mid, t2 = checksums()
        assert (t2[pick] == 1).all()
        assert np.array_equal(mid[pick], before[pick])
        dp = ids[torch.as_tensor(pick, device="cuda")].contiguous()
        cnt = torch.zeros(2, dtype=torch.int32, device="cuda")
        assert L.orchkv_promote_batch_to_gpu(C.c_void_p(dp.data_ptr()), None, len(pick),
                                             C.c_void_p(cnt.data_ptr())) == 0
        after, t3 = checksums()
        assert cnt.tolist() == [len(pick), 0]
        assert (t3 == 0).all()
        assert np.array_equal(after, before)
        assert L.orchkv_request_destroy(ctx) == 0
    finally:
        L.orchkv_shutdown()
