"""Demotion through the caller's callbacks (tm_schedule_once with transfer_fn,
alloc_fn and free_fn set): victim choice by the LRU-tail scan
(src/scheduler/eviction_policy.c:55-143), the migration bookkeeping
(src/scheduler/migration_engine.c:111-190) and the demote loops
(src/scheduler/tiered_manager.c:215-281), compared with the reference run on
the same scenarios (tests/golden/c4_demote_callbacks*.json, one with every
third transfer failing like test/test_migration_engine.c's failing mock):
final tier, state and payload of every block, and every demotion/migration
counter."""
import ctypes as C
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
PAYLOAD = 64

_libc = C.CDLL(None)
_libc.calloc.restype = C.c_void_p
_libc.calloc.argtypes = [C.c_size_t, C.c_size_t]
_libc.free.argtypes = [C.c_void_p]
_libc.memmove.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t]
_libc.memmove.restype = C.c_void_p


def run_b200(c):
    import orchkv_b200 as o
    from orchkv_b200 import _lib as Lb
    L = o.lib()
    XFER = C.CFUNCTYPE(C.c_int, C.POINTER(Lb.KvBlock), C.c_void_p, C.c_size_t, C.c_int,
                       C.c_void_p)
    ALLOC = C.CFUNCTYPE(C.c_void_p, C.c_size_t, C.c_int, C.c_void_p)
    FREE = C.CFUNCTYPE(None, C.c_void_p, C.c_int, C.c_void_p)

    calls = [0]
    fail_every = c.get("fail_every", 0)

    def transfer(blk, dst, size, op, ctx):
        calls[0] += 1
        if fail_every and calls[0] % fail_every == 0:
            return -6                                    # ORCHKV_ERR_IO
        if blk.contents.data_ptr and dst:
            _libc.memmove(dst, blk.contents.data_ptr, size)
        return 0

    def alloc(size, tier, ctx):
        return _libc.calloc(1, size)

    def free(p, tier, ctx):
        _libc.free(p)

    cb = (XFER(transfer), ALLOC(alloc), FREE(free))      # kept alive for the run
    cfg = Lb.TmConfig()
    L.tm_config_default(C.byref(cfg))
    cfg.tracker_capacity = 4096
    cfg.max_blocks = 4096
    cfg.hcc_params.alpha, cfg.hcc_params.beta, cfg.hcc_params.gamma = (
        c["alpha"], c["beta"], c["gamma"])
    cfg.transfer_fn = C.cast(cb[0], C.c_void_p)
    cfg.alloc_fn = C.cast(cb[1], C.c_void_p)
    cfg.free_fn = C.cast(cb[2], C.c_void_p)
    cfg.block_data_size = PAYLOAD
    cfg.demote_batch_size = c["demote_batch"]
    cfg.athresh_params.cooldown_sec = 0.0
    m = Lb.TieredManager()
    assert L.tm_init(C.byref(m), C.byref(cfg)) == 0
    n = len(c["ids"])
    blocks = (Lb.KvBlock * n)()
    for i in range(n):
        b = blocks[i]
        b.block_id = c["ids"][i]
        b.tier = c["tiers"][i]
        b.flags = c["flags"][i]
        b.state = 2 if c["tiers"][i] == 0 else 3
        b.data_ptr = _libc.calloc(1, PAYLOAD)
        C.memset(b.data_ptr, i & 0xFF, PAYLOAD)
        assert L.tm_register_block(C.byref(m), C.byref(b)) == 0
    for t in c["touch"]:
        L.tm_notify_access(C.byref(m), C.byref(blocks[t]))
    off = c["rep_off"]
    for s in range(c["steps"]):
        for r in range(off[s], off[s + 1]):
            L.tm_notify_attn(C.byref(m), c["rep_ids"][r], c["rep_w"][r])
        L.tm_step_done(C.byref(m))
        L.tm_set_usage(C.byref(m), c["gpu_ratio"][s], c["dram_ratio"][s])
        L.tm_schedule_once(C.byref(m))
    st = Lb.TmStats()
    L.tm_get_stats(C.byref(m), C.byref(st))
    ms = st.migration_stats
    stats = ([st.gpu_demotes, st.dram_demotes, ms.blocks_migrated, ms.op_errors]
             + list(ms.op_count) + [x // PAYLOAD for x in ms.op_bytes])
    tier, state, byte = [], [], []
    for i in range(n):
        b = blocks[i]
        tier.append(int(b.tier))
        state.append(int(b.state))
        byte.append(C.cast(b.data_ptr, C.POINTER(C.c_ubyte))[PAYLOAD - 1]
                    if b.data_ptr else -1)
    L.tm_destroy(C.byref(m))
    for i in range(n):
        if blocks[i].data_ptr:
            _libc.free(blocks[i].data_ptr)
    return dict(tier=tier, state=state, byte=byte, stats=[int(x) for x in stats])


@pytest.mark.parametrize("name", ["c4_demote_callbacks", "c4_demote_callbacks_failing"])
def test_c4_demotion_matches_reference(cuda, name):
    with open(os.path.join(HERE, "golden", name + ".json")) as fh:
        fx = json.load(fh)
    got = run_b200(fx["case"])
    exp = fx["expect"]
    assert got["stats"] == exp["stats"]
    assert got["tier"] == exp["tier"]
    assert got["state"] == exp["state"]
    assert got["byte"] == exp["byte"]
    assert exp["stats"][0] > 0 and exp["stats"][1] > 0     # both demote loops exercised
    assert np.count_nonzero(np.asarray(exp["tier"]) == 2) > 0
    if fx["case"].get("fail_every"):
        assert exp["stats"][3] > 0                         # failed transfers rolled back
