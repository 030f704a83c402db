"""Data-plane parity on the GPU through the C ABI: slab layout after prefill
and append, per-block and batched evict/promote against the oracle's
sequential per-block model (free stacks, block locations and slab bytes
bit-exact), the GPU -> DRAM -> GPU round trip, and error codes."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TPB, D, E = 16, 128, 2
ROW = D * E
SLAB = TPB * ROW * 2
HALF = SLAB // 2


GPU_SLABS, DRAM_SLABS = 160, 64


@pytest.fixture
def dp(cuda):
    import orchkv_b200 as o
    L = o.lib()
    cfg = o.make_config(gpu_pool_bytes=GPU_SLABS * SLAB, dram_pool_bytes=DRAM_SLABS * SLAB,
                        tokens_per_block=TPB, d_head=D, dtype=1, max_blocks_per_head=32)
    ext = o.OrchkvConfigExt()
    ext.max_blocks = 512
    assert L.orchkv_init_ext(C.byref(cfg), C.byref(ext)) == 0
    yield o, L
    assert L.orchkv_shutdown() == 0


def pool_state(L, which, total):
    st = np.zeros(total, np.uint32)
    top = C.c_uint32()
    assert L.orchkv_read_pool(which, st.ctypes.data, C.byref(top)) == 0
    return st[: top.value].tolist()


def locs(L, n):
    loc = np.zeros(n, np.uint32)
    state = np.zeros(n, np.uint8)
    assert L.orchkv_read_block_locs(loc.ctypes.data, state.ctypes.data) == 0
    return loc, state


_CUDART = None


def _cudart():
    global _CUDART
    if _CUDART is None:
        import glob
        import os
        import torch
        cands = glob.glob(os.path.join(os.path.dirname(torch.__file__), "..", "nvidia",
                                       "cuda_runtime", "lib", "libcudart.so*"))
        cands += ["libcudart.so.12", "/usr/local/cuda/lib64/libcudart.so"]
        for c in cands:
            try:
                _CUDART = C.CDLL(c)
                break
            except OSError:
                continue
        _CUDART.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
    return _CUDART


def read_dev(ptr, nbytes):
    out = np.empty(nbytes, np.uint8)
    assert _cudart().cudaMemcpy(out.ctypes.data, ptr, nbytes, 2) == 0
    return out


def read_host(ptr, nbytes):
    return np.ctypeslib.as_array((C.c_uint8 * nbytes).from_address(ptr)).copy()


def kv_data(rng, H, n):
    k = rng.integers(0, 255, (H, n, ROW), dtype=np.uint8)
    v = rng.integers(0, 255, (H, n, ROW), dtype=np.uint8)
    return k, v


def expected_slab(k, v, h, b):
    """Slab bytes of block b of head h: [K rows | V rows] (src/api/orchkv_api.cu:8-18)."""
    out = np.zeros(SLAB, np.uint8)
    n = k.shape[1]
    rows = range(b * TPB, min((b + 1) * TPB, n))
    for j, t in enumerate(rows):
        out[j * ROW:(j + 1) * ROW] = k[h, t]
        out[HALF + j * ROW:HALF + (j + 1) * ROW] = v[h, t]
    return out


def info(L, ctx, l, h, b):
    bid, tier, slab, st, tok = C.c_uint64(), C.c_int(), C.c_uint32(), C.c_int(), C.c_uint32()
    rc = L.orchkv_block_info(ctx, l, h, b, C.byref(bid), C.byref(tier), C.byref(slab),
                             C.byref(st), C.byref(tok))
    return rc, bid.value, tier.value, slab.value, st.value, tok.value


@pytest.mark.parametrize("src", ["pageable", "device", "pinned"])
def test_prefill_layout_and_ids(dp, cuda, src):
    o, L = dp
    rng = np.random.default_rng(1)
    H, n = 2, 40                      # 3 blocks per head, last one partial
    k, v = kv_data(rng, H, n)
    ctx = L.orchkv_request_create(7, 2, H)
    assert ctx
    if src == "pageable":
        kp, vp = k.ctypes.data, v.ctypes.data
        keep = (k, v)
    elif src == "device":
        kt, vt = cuda.from_numpy(k).cuda(), cuda.from_numpy(v).cuda()
        kp, vp, keep = kt.data_ptr(), vt.data_ptr(), (kt, vt)
    else:
        kt, vt = cuda.from_numpy(k).pin_memory(), cuda.from_numpy(v).pin_memory()
        kp, vp, keep = kt.data_ptr(), vt.data_ptr(), (kt, vt)
    assert L.orchkv_prefill(ctx, 0, kp, vp, n) == 0
    del keep
    # block ids follow the reference counter order: block-major, then head
    # (src/core/kv_request.c:177-204); slabs are popped head-major
    # (src/api/orchkv_api.cu:219-226): head 0 gets slabs 0,1,2
    base = L.orchkv_gpu_pool_base()
    for h in range(H):
        for b in range(3):
            rc, bid, tier, slab, st, tok = info(L, ctx, 0, h, b)
            assert rc == 0 and tier == 0 and st == 2
            assert bid == b * H + h
            assert slab == h * 3 + b
            assert tok == (TPB if b < 2 else n - 2 * TPB)
            got = read_dev(base + slab * SLAB, SLAB)
            want = expected_slab(k, v, h, b)
            used = tok * ROW
            assert np.array_equal(got[:used], want[:used])
            assert np.array_equal(got[HALF:HALF + used], want[HALF:HALF + used])
    assert info(L, ctx, 0, 0, 3)[0] == -3       # NOT_FOUND
    assert info(L, ctx, 1, 0, 0)[0] == -3
    s = o.OrchkvStats()
    L.orchkv_get_stats(C.byref(s))
    assert s.gpu_slabs_used == 6 and s.total_blocks == 6
    assert L.orchkv_request_destroy(ctx) == 0
    L.orchkv_get_stats(C.byref(s))
    assert s.gpu_slabs_used == 0


def _model_from_device(L, total_g, total_d, max_blocks):
    from oracle import oracle as O
    gp, dp_ = O.Pool(total_g), O.Pool(total_d)
    gp.stack = pool_state(L, 0, total_g)
    dp_.stack = pool_state(L, 1, total_d)
    loc, state = locs(L, max_blocks)
    return gp, dp_, loc.astype(np.int64).tolist(), state.tolist()


def test_per_block_evict_promote_vs_oracle(dp, cuda):
    from oracle import oracle as O
    o, L = dp
    rng = np.random.default_rng(2)
    H, n = 4, 64
    k, v = kv_data(rng, H, n)
    ctx = L.orchkv_request_create(1, 1, H)
    assert L.orchkv_prefill(ctx, 0, k.ctypes.data, v.ctypes.data, n) == 0
    gtot, dtot = GPU_SLABS, DRAM_SLABS
    gpool, dpool, loc, state = _model_from_device(L, gtot, dtot, 512)
    gbytes = read_dev(L.orchkv_gpu_pool_base(), gtot * SLAB)
    dbytes = np.zeros(dtot * SLAB, np.uint8)
    ops = [("e", 1, 2), ("e", 0, 0), ("e", 3, 3), ("p", 0, 0), ("e", 2, 1), ("p", 3, 3),
           ("p", 1, 2), ("e", 1, 2), ("e", 0, 0)]
    for kind, h, b in ops:
        bid = info(L, ctx, 0, h, b)[1]
        if kind == "e":
            assert L.orchkv_evict_to_dram(ctx, 0, h, b) == 0
            O.evict_batch(gpool, dpool, loc, state, None, [bid], gbytes, dbytes, SLAB)
        else:
            assert L.orchkv_promote_to_gpu(ctx, 0, h, b) == 0
            O.promote_batch(gpool, dpool, loc, state, [bid], gbytes, dbytes, SLAB)
    g2, d2, loc2, state2 = _model_from_device(L, gtot, dtot, 512)
    assert g2.stack == gpool.stack and d2.stack == dpool.stack
    assert loc2 == loc
    # every block's bytes, wherever it lives, equal the prefilled data
    dbase = L.orchkv_dram_pool_base()
    for h in range(H):
        for b in range(4):
            _, bid, tier, slab, _, _ = info(L, ctx, 0, h, b)
            got = read_dev(L.orchkv_gpu_pool_base() + slab * SLAB, SLAB) if tier == 0 else \
                read_host(dbase + slab * SLAB, SLAB)
            assert np.array_equal(got, expected_slab(k, v, h, b))
    # error codes (src/api/orchkv_api.cu:353-428)
    h, b = 0, 0
    t = info(L, ctx, 0, h, b)[2]
    if t == 1:
        assert L.orchkv_evict_to_dram(ctx, 0, h, b) == -8       # ERR_STATE
    else:
        assert L.orchkv_promote_to_gpu(ctx, 0, h, b) == -8
    assert L.orchkv_evict_to_dram(ctx, 0, 0, 9) == -3           # ERR_NOT_FOUND
    assert L.orchkv_set_block_flags(ctx, 0, 2, 2, 0x01) == 0
    assert L.orchkv_evict_to_dram(ctx, 0, 2, 2) == -7           # ERR_LOCKED
    kp, vp = C.c_void_p(), C.c_void_p()
    _, _, tier, _, _, _ = info(L, ctx, 0, 1, 2)
    assert L.orchkv_get_kv_block(ctx, 0, 1, 2, C.byref(kp), C.byref(vp)) == 0
    assert info(L, ctx, 0, 1, 2)[2] == 0 and vp.value - kp.value == HALF
    assert L.orchkv_request_destroy(ctx) == 0


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_batched_migration_equals_sequential(dp, cuda, seed):
    from oracle import oracle as O
    o, L = dp
    rng = np.random.default_rng(seed)
    H, n = 4, 16 * 12
    k, v = kv_data(rng, H, n)
    ctxs = [L.orchkv_request_create(i, 1, H) for i in range(2)]
    for c in ctxs:
        assert L.orchkv_prefill(c, 0, k.ctypes.data, v.ctypes.data, n) == 0
    gtot, dtot = GPU_SLABS, DRAM_SLABS
    # a few single evictions first so the DRAM free stack is not in order
    for h, b in [(0, 1), (2, 5), (1, 7)]:
        assert L.orchkv_evict_to_dram(ctxs[0], 0, h, b) == 0
    gpool, dpool, loc, state = _model_from_device(L, gtot, dtot, 512)
    gbytes = read_dev(L.orchkv_gpu_pool_base(), gtot * SLAB)
    dbytes = read_host(L.orchkv_dram_pool_base(), dtot * SLAB)
    live = [i for i, w in enumerate(loc) if (w >> 29) in (0, 1)]
    for rnd in range(4):
        ids = rng.choice(live, int(rng.integers(10, 80)), replace=False).astype(np.uint32)
        ids = np.concatenate([ids, np.array([511], np.uint32)])     # an id with no block
        if seed == 2:                                               # repeated ids
            ids = np.concatenate([ids, rng.choice(ids, 12)]).astype(np.uint32)
            rng.shuffle(ids)
        dev_ids = cuda.from_numpy(ids.view(np.int32)).cuda()
        res = cuda.zeros(2, dtype=cuda.int32, device="cuda")
        if rnd % 2 == 0:
            assert L.orchkv_evict_batch_to_dram(dev_ids.data_ptr(), None, len(ids), res.data_ptr()) == 0
            done, skipped = O.evict_batch(gpool, dpool, loc, state, None, ids.tolist(),
                                          gbytes, dbytes, SLAB)
        else:
            assert L.orchkv_promote_batch_to_gpu(dev_ids.data_ptr(), None, len(ids), res.data_ptr()) == 0
            done, skipped = O.promote_batch(gpool, dpool, loc, state, ids.tolist(), gbytes,
                                            dbytes, SLAB)
        r = res.cpu().numpy()
        assert (int(r[0]), int(r[1])) == (done, skipped)
    g2, d2, loc2, _ = _model_from_device(L, gtot, dtot, 512)
    assert g2.stack == gpool.stack and d2.stack == dpool.stack and loc2 == loc
    for bid, w in enumerate(loc):
        t, s = w >> 29, w & 0x1FFFFFFF
        if t == 0:
            assert np.array_equal(read_dev(L.orchkv_gpu_pool_base() + s * SLAB, SLAB),
                                  gbytes[s * SLAB:(s + 1) * SLAB]), bid
        elif t == 1:
            assert np.array_equal(read_host(L.orchkv_dram_pool_base() + s * SLAB, SLAB),
                                  dbytes[s * SLAB:(s + 1) * SLAB]), bid
    for c in ctxs:
        assert L.orchkv_request_destroy(c) == 0


def test_batch_pool_exhaustion(dp, cuda):
    from oracle import oracle as O
    o, L = dp
    rng = np.random.default_rng(9)
    H, n = 4, 16 * 20        # 80 GPU slabs; DRAM holds 64
    k, v = kv_data(rng, H, n)
    ctx = L.orchkv_request_create(3, 1, H)
    assert L.orchkv_prefill(ctx, 0, k.ctypes.data, v.ctypes.data, n) == 0
    gpool, dpool, loc, state = _model_from_device(L, GPU_SLABS, DRAM_SLABS, 512)
    ids = np.arange(80, dtype=np.uint32)[::-1].copy()
    dev_ids = cuda.from_numpy(ids.view(np.int32)).cuda()
    cnt = cuda.tensor([75], dtype=cuda.int32, device="cuda")
    res = cuda.zeros(2, dtype=cuda.int32, device="cuda")
    assert L.orchkv_evict_batch_to_dram(dev_ids.data_ptr(), cnt.data_ptr(), 80, res.data_ptr()) == 0
    gb = read_dev(L.orchkv_gpu_pool_base(), GPU_SLABS * SLAB)
    db = np.zeros(DRAM_SLABS * SLAB, np.uint8)
    done, skipped = O.evict_batch(gpool, dpool, loc, state, None, ids[:75].tolist(), gb, db, SLAB)
    assert (done, skipped) == (64, 11)
    assert res.cpu().tolist() == [64, 11]
    g2, d2, loc2, _ = _model_from_device(L, GPU_SLABS, DRAM_SLABS, 512)
    assert g2.stack == gpool.stack and d2.stack == dpool.stack and loc2 == loc
    assert L.orchkv_request_destroy(ctx) == 0


def test_append_one_and_batch_agree(dp, cuda):
    o, L = dp
    rng = np.random.default_rng(4)
    H, Lr, n0 = 2, 3, 30
    reqs = []
    for _ in range(2):                       # two identical systems: per-call vs batch
        reqs.append([L.orchkv_request_create(i, Lr, H) for i in range(3)])
    k0, v0 = kv_data(rng, H, n0)
    for group in reqs:
        for c in group:
            for layer in range(Lr):
                assert L.orchkv_prefill(c, layer, k0.ctypes.data, v0.ctypes.data, n0) == 0
    for step in range(5):
        kt = rng.integers(0, 255, (3, Lr, H, ROW), dtype=np.uint8)
        vt = rng.integers(0, 255, (3, Lr, H, ROW), dtype=np.uint8)
        # reference call order: for request, for layer (src/api/orchkv_api.cu:263-317)
        for i, c in enumerate(reqs[0]):
            for layer in range(Lr):
                assert L.orchkv_append_token(c, layer, kt[i, layer].ctypes.data,
                                             vt[i, layer].ctypes.data) == 0
        arr = (C.c_void_p * 3)(*reqs[1])
        kd, vd = cuda.from_numpy(kt).cuda(), cuda.from_numpy(vt).cuda()
        assert L.orchkv_append_token_batch(arr, 3, kd.data_ptr(), vd.data_ptr()) == 0
    base = L.orchkv_gpu_pool_base()
    for i in range(3):
        for layer in range(Lr):
            for h in range(H):
                for b in range(3):
                    a = info(L, reqs[0][i], layer, h, b)
                    bb = info(L, reqs[1][i], layer, h, b)
                    assert a[0] == 0 and bb[0] == 0 and a[5] == bb[5]
                    ga = read_dev(base + a[3] * SLAB, SLAB)
                    gb = read_dev(base + bb[3] * SLAB, SLAB)
                    used = a[5] * ROW
                    assert np.array_equal(ga[:used], gb[:used])
                    assert np.array_equal(ga[HALF:HALF + used], gb[HALF:HALF + used])
    s = o.OrchkvStats()
    L.orchkv_get_stats(C.byref(s))
    assert s.gpu_slabs_used == 2 * 3 * Lr * H * 3
    for group in reqs:
        for c in group:
            assert L.orchkv_request_destroy(c) == 0


def test_append_state_error(dp, cuda):
    o, L = dp
    rng = np.random.default_rng(8)
    H = 2
    k, v = kv_data(rng, H, 20)                  # last block partial (4 of 16)
    ctx = L.orchkv_request_create(1, 1, H)
    assert L.orchkv_prefill(ctx, 0, k.ctypes.data, v.ctypes.data, 20) == 0
    assert L.orchkv_evict_to_dram(ctx, 0, 1, 1) == 0
    row = np.zeros((H, ROW), np.uint8)
    assert L.orchkv_append_token(ctx, 0, row.ctypes.data, row.ctypes.data) == -8
    arr = (C.c_void_p * 1)(ctx)
    kd = cuda.zeros(H * ROW, dtype=cuda.uint8, device="cuda")
    assert L.orchkv_append_token_batch(arr, 1, kd.data_ptr(), kd.data_ptr()) == -8
    assert L.orchkv_request_destroy(ctx) == 0


def test_attached_manager_lifetimes(cuda):
    """A manager attached to the data plane may be destroyed first (the data
    plane stops touching its slots) or last (it gets its own stream back when
    the data plane shuts down); both orders leave every call valid."""
    import orchkv_b200 as o
    L = o.lib()
    rng = np.random.default_rng(9)
    for destroy_manager_first in (True, False):
        cfg = o.make_config(gpu_pool_bytes=GPU_SLABS * SLAB, dram_pool_bytes=DRAM_SLABS * SLAB,
                            tokens_per_block=TPB, d_head=D, dtype=1, max_blocks_per_head=32)
        ext = o.OrchkvConfigExt()
        ext.max_blocks = 512
        assert L.orchkv_init_ext(C.byref(cfg), C.byref(ext)) == 0
        m = o.Manager(tracker_cap=512, max_blocks=4096)
        assert L.orchkv_attach_scheduler(m.ref) == 0
        k, v = kv_data(rng, 2, 40)
        c1 = L.orchkv_request_create(1, 2, 2)
        assert L.orchkv_prefill(c1, 0, k.ctypes.data, v.ctypes.data, 40) == 0
        assert L.orchkv_sync() == 0
        assert m.state()["c_active"].sum() == 6              # 2 heads x 3 blocks registered
        if destroy_manager_first:
            m.close()
            # data-plane work after the manager is gone
            c2 = L.orchkv_request_create(2, 2, 2)
            assert L.orchkv_prefill(c2, 1, k.ctypes.data, v.ctypes.data, 40) == 0
            assert L.orchkv_evict_to_dram(c2, 1, 0, 0) == 0
            assert L.orchkv_request_destroy(c2) == 0
            assert L.orchkv_request_destroy(c1) == 0
            assert L.orchkv_sync() == 0
            assert L.orchkv_shutdown() == 0
        else:
            assert L.orchkv_request_destroy(c1) == 0
            assert L.orchkv_shutdown() == 0
            # the manager keeps working on its own stream, then goes away
            m.report(0, 0.5)
            m.step_done()
            assert m.state()["t_active"].sum() == 0          # request teardown unregistered
            m.close()


@pytest.mark.parametrize("kv_src", ["pageable", "pageable_k_device_v"])
def test_prefill_stages_large_host_inputs(cuda, kv_src):
    """Pageable K and V larger than the staging buffer of a fresh system: both
    are staged before the buffer can move (K bytes used to be lost when the
    buffer grew for V)."""
    import orchkv_b200 as o
    L = o.lib()
    H, n = 4, 16 * 100                                # 1.6 MB each of K and V
    cfg = o.make_config(gpu_pool_bytes=(H * 100 + 8) * SLAB, dram_pool_bytes=8 * SLAB,
                        tokens_per_block=TPB, d_head=D, dtype=1, max_blocks_per_head=128)
    ext = o.OrchkvConfigExt()
    ext.max_blocks = 512
    assert L.orchkv_init_ext(C.byref(cfg), C.byref(ext)) == 0
    try:
        rng = np.random.default_rng(21)
        k, v = kv_data(rng, H, n)
        ctx = L.orchkv_request_create(1, 1, H)
        vt = cuda.from_numpy(v).cuda() if kv_src == "pageable_k_device_v" else None
        vp = vt.data_ptr() if vt is not None else v.ctypes.data
        assert L.orchkv_prefill(ctx, 0, k.ctypes.data, vp, n) == 0
        base = L.orchkv_gpu_pool_base()
        for h in range(H):
            for b in (0, 57, 99):
                rc, bid, tier, slab, st, tok = info(L, ctx, 0, h, b)
                assert rc == 0 and tier == 0
                assert np.array_equal(read_dev(base + slab * SLAB, SLAB),
                                      expected_slab(k, v, h, b)), (h, b)
        assert L.orchkv_request_destroy(ctx) == 0
    finally:
        assert L.orchkv_shutdown() == 0


def test_request_destroy_returns_slabs_in_table_order(dp, cuda):
    """Teardown (src/api/orchkv_api.cu:149-183) pushes each existing block's
    slab onto its tier's stack and its id onto the id stack in (layer, head,
    block) order; blocks on both tiers, two layers, a partial last block."""
    o, L = dp
    rng = np.random.default_rng(17)
    H, n = 2, 16 * 5 + 7                       # 6 blocks per head, the last partial
    ctxs = []
    for r in range(2):
        c = L.orchkv_request_create(r, 2, H)
        for layer in range(2):
            k, v = kv_data(rng, H, n)
            assert L.orchkv_prefill(c, layer, k.ctypes.data, v.ctypes.data, n) == 0
        ctxs.append(c)
    c = ctxs[0]
    for (l, h, b) in [(0, 1, 2), (1, 0, 0), (1, 1, 5), (0, 0, 4)]:
        assert L.orchkv_evict_to_dram(c, l, h, b) == 0
    g0, d0 = pool_state(L, 0, GPU_SLABS), pool_state(L, 1, DRAM_SLABS)
    want_g, want_d, want_i = list(g0), list(d0), []
    for l in range(2):
        for h in range(H):
            for b in range(6):
                rc, bid, tier, slab, st, tok = info(L, c, l, h, b)
                assert rc == 0
                (want_g if tier == 0 else want_d).append(slab)
                want_i.append(bid)
    st = o.OrchkvStats()
    L.orchkv_get_stats(C.byref(st))
    blocks_before = st.total_blocks
    assert L.orchkv_request_destroy(c) == 0
    assert pool_state(L, 0, GPU_SLABS) == want_g
    assert pool_state(L, 1, DRAM_SLABS) == want_d
    ids_top = pool_state(L, 2, 512)
    assert ids_top[-len(want_i):] == want_i
    L.orchkv_get_stats(C.byref(st))
    assert st.total_blocks == blocks_before - 24
    assert L.orchkv_request_destroy(ctxs[1]) == 0


def test_batched_edge_cases(dp, cuda):
    """Empty lists, a device count below max_n, ids past the block-id space
    and repeated ids: skipped exactly as the per-block calls would skip them
    (unknown id -> not on the tier), nothing else moves."""
    o, L = dp
    rng = np.random.default_rng(23)
    H, n = 2, 16 * 4
    k, v = kv_data(rng, H, n)
    c = L.orchkv_request_create(1, 1, H)
    assert L.orchkv_prefill(c, 0, k.ctypes.data, v.ctypes.data, n) == 0
    g0, d0 = pool_state(L, 0, GPU_SLABS), pool_state(L, 1, DRAM_SLABS)
    res = cuda.full((4,), -1, dtype=cuda.int32, device="cuda")
    empty = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    assert L.orchkv_evict_batch_to_dram(empty.data_ptr(), None, 0, res.data_ptr()) == 0
    assert L.orchkv_promote_batch_to_gpu(empty.data_ptr(), None, 0, res.data_ptr()) == 0
    assert L.orchkv_swap_batch(empty.data_ptr(), None, 0, empty.data_ptr(), None, 0,
                               res.data_ptr()) == 0
    assert L.orchkv_sync() == 0
    assert res.cpu().tolist() == [0, 0, 0, 0]
    assert pool_state(L, 0, GPU_SLABS) == g0 and pool_state(L, 1, DRAM_SLABS) == d0
    # count 2 of a 5-entry list; then unknown and repeated ids
    ids = cuda.tensor([0, 1, 2, 3, 4], dtype=cuda.int32, device="cuda")
    cnt = cuda.tensor([2], dtype=cuda.int32, device="cuda")
    assert L.orchkv_evict_batch_to_dram(ids.data_ptr(), cnt.data_ptr(), 5, res.data_ptr()) == 0
    assert L.orchkv_sync() == 0
    assert res.cpu().tolist()[:2] == [2, 0]
    odd = cuda.tensor([1 << 30, 0, 0, 511, 5], dtype=cuda.int32, device="cuda")
    assert L.orchkv_promote_batch_to_gpu(odd.data_ptr(), None, 5, res.data_ptr()) == 0
    assert L.orchkv_sync() == 0
    # id 0 (on DRAM) comes back once; its repeat, the unknown ids and id 5
    # (on the GPU) are skipped
    assert res.cpu().tolist()[:2] == [1, 4]
    rc, bid, tier, slab, st, tok = info(L, c, 0, 0, 0)
    assert bid == 0 and tier == 0
    assert L.orchkv_request_destroy(c) == 0


@pytest.mark.parametrize("tpb,seed", [(64, 0xCAFEBABE), (8192, 0xDEADBEEF)])
def test_seed_pattern_round_trips(cuda, tpb, seed):
    """The reference's data-integrity known answers (test/test_gpu_dram.cu:40-55,
    151-243): slabs of 32 KB and 4 MB (fp16, d_head 128, 64- and 8192-token
    blocks) holding u32 words seed ^ i, GPU -> DRAM -> GPU by the batched and
    by the per-block calls, every word checked after each hop."""
    import orchkv_b200 as o
    L = o.lib()
    d, e = 128, 2
    slab = tpb * d * e * 2
    half, H, nblk = slab // 2, 2, 2
    cfg = o.make_config(gpu_pool_bytes=8 * slab, dram_pool_bytes=8 * slab, tokens_per_block=tpb,
                        d_head=d, dtype=0, max_blocks_per_head=4)
    ext = o.OrchkvConfigExt()
    ext.max_blocks = 64
    assert L.orchkv_init_ext(C.byref(cfg), C.byref(ext)) == 0
    try:
        # slab (h, b) holds seed' ^ i with seed' = seed + 16 * h + b: K half
        # first, V half second, as the slab layout puts them
        pats = {(h, b): (np.uint32(seed + 16 * h + b) ^
                         np.arange(slab // 4, dtype=np.uint32)).view(np.uint8)
                for h in range(H) for b in range(nblk)}
        k = np.empty((H, nblk * tpb, d * e), np.uint8)
        v = np.empty_like(k)
        for (h, b), p in pats.items():
            k[h, b * tpb:(b + 1) * tpb] = p[:half].reshape(tpb, d * e)
            v[h, b * tpb:(b + 1) * tpb] = p[half:].reshape(tpb, d * e)
        c = L.orchkv_request_create(9, 1, H)
        assert L.orchkv_prefill(c, 0, k.ctypes.data, v.ctypes.data, nblk * tpb) == 0

        def check(tier_want):
            for (h, b), p in pats.items():
                rc, bid, tier, s, st, tok = info(L, c, 0, h, b)
                assert rc == 0 and tier == tier_want
                got = (read_dev(L.orchkv_gpu_pool_base() + s * slab, slab) if tier == 0 else
                       read_host(L.orchkv_dram_pool_base() + s * slab, slab))
                assert np.array_equal(got, p), (h, b)

        check(0)
        bids = cuda.tensor([info(L, c, 0, h, b)[1] for h in range(H) for b in range(nblk)],
                           dtype=cuda.int32, device="cuda")
        res = cuda.zeros(2, dtype=cuda.int32, device="cuda")
        assert L.orchkv_evict_batch_to_dram(bids.data_ptr(), None, len(bids), res.data_ptr()) == 0
        assert L.orchkv_sync() == 0
        assert res.cpu().tolist() == [len(bids), 0]
        check(1)
        assert L.orchkv_promote_batch_to_gpu(bids.data_ptr(), None, len(bids), res.data_ptr()) == 0
        assert L.orchkv_sync() == 0
        check(0)
        for h in range(H):
            for b in range(nblk):
                assert L.orchkv_evict_to_dram(c, 0, h, b) == 0
        check(1)
        for h in range(H):
            for b in range(nblk):
                assert L.orchkv_promote_to_gpu(c, 0, h, b) == 0
        check(0)
        assert L.orchkv_request_destroy(c) == 0
    finally:
        L.orchkv_shutdown()


def test_concurrent_batches_from_threads(dp, cuda):
    """Batched evicts and promotes issued from two host threads at once (two
    requests, each thread its own): whichever order the library serialises
    them in, every block moves once, its bytes are intact where it lands, and
    the free stacks hold exactly the slabs not in use."""
    import threading
    o, L = dp
    rng = np.random.default_rng(41)
    H, n = 2, 16 * 8                                  # 16 blocks per request
    data, ctxs, ids = [], [], []
    for r in range(2):
        k, v = kv_data(rng, H, n)
        c = L.orchkv_request_create(50 + r, 1, H)
        assert L.orchkv_prefill(c, 0, k.ctypes.data, v.ctypes.data, n) == 0
        data.append((k, v))
        ctxs.append(c)
        ids.append([info(L, c, 0, h, b)[1] for h in range(H) for b in range(8)])
    g_free0 = len(pool_state(L, 0, GPU_SLABS))
    dev = [cuda.tensor(i, dtype=cuda.int32, device="cuda") for i in ids]
    res = [cuda.zeros(2, dtype=cuda.int32, device="cuda") for _ in range(2)]
    errors = []

    def worker(r, fn):
        try:
            for _ in range(3):
                rc = fn(dev[r].data_ptr(), None, len(ids[r]), res[r].data_ptr())
                if rc != 0:
                    errors.append(rc)
        except Exception as e:                         # pragma: no cover - reported below
            errors.append(repr(e))

    for fn, tier in ((L.orchkv_evict_batch_to_dram, 1), (L.orchkv_promote_batch_to_gpu, 0)):
        ts = [threading.Thread(target=worker, args=(r, fn)) for r in range(2)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        assert L.orchkv_sync() == 0 and not errors
        for r in range(2):
            k, v = data[r]
            for h in range(H):
                for b in range(8):
                    rc, bid, t_, slab, st, tok = info(L, ctxs[r], 0, h, b)
                    assert rc == 0 and t_ == tier
                    base = L.orchkv_dram_pool_base() if tier == 1 else L.orchkv_gpu_pool_base()
                    got = (read_host if tier == 1 else read_dev)(base + slab * SLAB, SLAB)
                    assert np.array_equal(got, expected_slab(k, v, h, b)), (r, h, b)
        g_free, d_free = len(pool_state(L, 0, GPU_SLABS)), len(pool_state(L, 1, DRAM_SLABS))
        if tier == 1:
            assert g_free == g_free0 + 32 and d_free == DRAM_SLABS - 32
        else:
            assert g_free == g_free0 and d_free == DRAM_SLABS
    for c in ctxs:
        assert L.orchkv_request_destroy(c) == 0
