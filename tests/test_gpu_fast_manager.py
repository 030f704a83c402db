"""orchkv_b200.fast_manager.FastKVCacheManager against a CPU restatement of
the reference's python/orchkv/fast_kvcache_manager.py (oracle/
fast_manager_model.py, its scheduler the oracle's OracleTM) over a decode
run: prefill, then per step one appended token, attention reported for every
layer, step_done and schedule under a GPU byte budget that forces evictions,
with build_past_kv (which restores every evicted block) every few steps.

Attention weights are multiples of 2**-12, so every per-block sum is exact
in any summation order: tracker and classifier state must then be
bit-identical, the evicted block sets identical, and the KV buffers
byte-identical.  The QK-norm proxy is checked separately (1e-5 relative: the
block sums of |q.K| are added in another order)."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LY, HKV, HQ, D, BS = 4, 2, 4, 64, 16


def tm_state(o, mgr):
    n = mgr._cap
    out = {"sum": np.zeros(n, np.float32), "ema": np.zeros(n, np.float32),
           "hits": np.zeros(n, np.uint32), "last": np.zeros(n, np.uint64),
           "t_active": np.zeros(n, np.uint8), "hot": np.zeros(n, np.float32),
           "heat": np.zeros(n, np.uint8), "c_active": np.zeros(n, np.uint8)}
    assert o.lib().tm_read_state(mgr.tm_ref(), *(out[k].ctypes.data for k in (
        "sum", "ema", "hits", "last", "t_active", "hot", "heat", "c_active"))) == 0
    return out


def test_fast_manager_matches_reference_model(cuda):
    import orchkv_b200 as o
    from orchkv_b200.fast_manager import FastKVCacheManager
    from oracle.fast_manager_model import FastManagerModel
    torch = cuda
    rng = np.random.default_rng(3)
    block_bytes = 2 * HKV * BS * D * 2
    budget = 40 * LY * block_bytes                    # evictions start around 47 blocks
    mgr = FastKVCacheManager(LY, HKV, D, block_size=BS, dtype=torch.float16,
                             gpu_budget_bytes=budget, max_seq_len=1024, sink_tokens=4)
    mod = FastManagerModel(LY, HKV, D, block_size=BS, dtype=np.float16,
                           gpu_budget_bytes=budget, max_seq_len=1024, sink_tokens=4)
    try:
        t0 = 700
        k = [rng.standard_normal((HKV, t0, D)).astype(np.float16) for _ in range(LY)]
        v = [rng.standard_normal((HKV, t0, D)).astype(np.float16) for _ in range(LY)]
        mgr.ingest_step(tuple((torch.from_numpy(k[i])[None].cuda(),
                               torch.from_numpy(v[i])[None].cuda()) for i in range(LY)))
        mod.ingest(k, v)
        evictions = 0
        for step in range(40):
            kt = [rng.standard_normal((HKV, D)).astype(np.float16) for _ in range(LY)]
            vt = [rng.standard_normal((HKV, D)).astype(np.float16) for _ in range(LY)]
            mgr.append_token(tuple((torch.from_numpy(kt[i])[None, :, None].cuda(),
                                    torch.from_numpy(vt[i])[None, :, None].cuda())
                                   for i in range(LY)))
            mod.append(kt, vt)
            T = mod._total_tokens
            for li in range(LY):
                attn = (rng.integers(0, 16, (1, HQ, 1, T)) / 4096.0).astype(np.float32)
                mgr.report_attention(li, torch.from_numpy(attn).cuda())
                mod.report_attention(attn[0, :, 0, :])
            mgr.step_done()
            mod.step_done()
            assert mgr.schedule() == mod.schedule()
            assert sorted(mgr._evicted) == mod.evicted_blocks(), step
            assert mgr.get_stats() == mod.get_stats(), step
            evictions += mgr.get_stats()["migrations"]["evictions_this_step"]
            if step % 6 == 5:
                mgr.build_past_kv()
                mod.restore()
                assert mgr.get_stats() == mod.get_stats()
        assert evictions > 20
        got, want = tm_state(o, mgr), mod.tm.s.state()
        for key in ("sum", "ema", "hits", "last", "t_active", "hot", "c_active"):
            assert np.array_equal(got[key].view(np.uint8), want[key].view(np.uint8)), key
        mgr.build_past_kv()
        mod.restore()
        n = mod._total_tokens
        for li in range(LY):
            assert np.array_equal(mgr._key_bufs[li][0, :, :n].cpu().numpy(), mod.k[li][:, :n])
            assert np.array_equal(mgr._val_bufs[li][0, :, :n].cpu().numpy(), mod.v[li][:, :n])
    finally:
        mgr.destroy()


def test_fast_manager_qk_norm_proxy(cuda):
    from orchkv_b200.fast_manager import FastKVCacheManager
    from oracle.oracle import OracleSched
    torch = cuda
    rng = np.random.default_rng(4)
    mgr = FastKVCacheManager(LY, HKV, D, block_size=BS, dtype=torch.float32, max_seq_len=512)
    try:
        t0 = 300
        kv = tuple((torch.from_numpy(rng.standard_normal((1, HKV, t0, D)).astype(np.float32)).cuda(),
                    torch.from_numpy(rng.standard_normal((1, HKV, t0, D)).astype(np.float32)).cuda())
                   for _ in range(LY))
        mgr.ingest_step(kv)
        q = torch.from_numpy(rng.standard_normal((1, HQ, 1, D)).astype(np.float32)).cuda()
        mgr.report_qk_norm(2, q)
        # the reference's per-block loop (fast_kvcache_manager.py:255-270)
        gqa = HQ // HKV
        qk = torch.matmul(q[:, ::gqa], kv[2][0][:, :, :t0].transpose(-1, -2))
        qk_abs = qk.abs().squeeze(0).squeeze(1)
        nb = (t0 + BS - 1) // BS
        want = [float(qk_abs[:, b * BS:min((b + 1) * BS, t0)].sum()) for b in range(nb)]
        got = tm_state(__import__("orchkv_b200"), mgr)["sum"][:nb]
        assert np.allclose(got, np.float32(want), rtol=1e-5, atol=0)
    finally:
        mgr.destroy()
