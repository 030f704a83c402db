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
    for (l, h, b) in cold:
        kp, vp = C.c_void_p(), C.c_void_p()
        assert L.orchkv_get_kv_block(ctx, l, h, b, C.byref(kp), C.byref(vp)) == 0
        assert vp.value - kp.value == HALF
        assert np.array_equal(read_dev(kp.value, SLAB), expected_slab(k, v, h, b))
    L.orchkv_get_stats(C.byref(s))
    assert s.gpu_slabs_used == 8 and s.dram_slabs_used == 0
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
