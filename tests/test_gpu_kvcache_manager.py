"""orchkv_b200.kvcache_manager (the reference's block-level KVCacheManager on
the B200 path) against oracle/kvcache_manager_model.py (the reference
manager's decisions restated on the oracle tracker), over a decode loop that
evicts, spills to files and brings blocks back: every step the schedule
result, the statistics, each block's tier and access count are equal; every
rebuilt past_key_values and every spill file is bit-identical to the data
fed in; the tracker ends with the same hits and last-hit steps and sums and
EMA within 1e-5 relative (the per-block mass is summed in another order)."""
import ctypes as C
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL = 1e-5


def _tm_state(handle):
    import orchkv_b200 as o
    from orchkv_b200._lib import TieredManager
    L = o.lib()
    m = C.cast(C.c_void_p(handle), C.POINTER(TieredManager))
    n = L.tm_capacity(m)
    out = {"sum": np.zeros(n, np.float32), "ema": np.zeros(n, np.float32),
           "hits": np.zeros(n, np.uint32), "last": np.zeros(n, np.uint64)}
    assert L.tm_read_state(m, out["sum"].ctypes.data, out["ema"].ctypes.data,
                           out["hits"].ctypes.data, out["last"].ctypes.data,
                           None, None, None, None) == 0
    return out


def test_decode_loop_matches_reference_model(cuda, oracle_mod, tmp_path):
    torch = cuda
    from oracle.kvcache_manager_model import ModelKVManager
    from orchkv_b200.kvcache_manager import TIER_SSD, KVCacheManager
    Ly, H, Hq, d, bs, T0, steps = 4, 2, 4, 64, 16, 100, 30
    block_bytes = 2 * H * bs * d * 2
    budget = 30 * block_bytes          # 28 blocks after prefill: above 85%, evict to 70%
    ssd = str(tmp_path / "ssd")
    g = torch.Generator(device="cuda").manual_seed(11)
    K = [torch.randn(H, T0 + steps, d, generator=g, device="cuda").half() for _ in range(Ly)]
    V = [torch.randn(H, T0 + steps, d, generator=g, device="cuda").half() for _ in range(Ly)]
    Kh = [k.cpu().numpy() for k in K]
    Vh = [v.cpu().numpy() for v in V]

    mgr = KVCacheManager(Ly, H, d, block_size=bs, dtype=torch.float16, gpu_budget_bytes=budget,
                         ssd_dir=ssd, sink_tokens=4)
    try:
        model = ModelKVManager(Ly, H, d, bs, np.float16, budget, True, 4,
                               tracker_cap=mgr._cap)

        def pkv(n):
            return tuple((K[i][None, :, :n], V[i][None, :, :n]) for i in range(Ly))

        def kv_np(n):
            return [(Kh[i][:, :n], Vh[i][:, :n]) for i in range(Ly)]

        def same_blocks():
            for lb, mb in zip(mgr._blocks, model.blocks):
                assert [(b.block_id, b.token_start, b.token_count, b.tier, b.access_count,
                         b.is_sink) for b in lb] == \
                       [(b.block_id, b.token_start, b.token_count, b.tier, b.access_count,
                         b.is_sink) for b in mb]

        def same_stats():
            a, b = mgr.get_stats(), model.get_stats()
            a.pop("tm")
            assert a == b

        def check_build(n):
            out = mgr.build_past_kv()
            legacy = mgr._to_legacy(out)
            ref = model.build_past_kv()
            for i in range(Ly):
                k, v = legacy[i]
                assert k.shape == (1, H, n, d)
                assert np.array_equal(k[0].cpu().numpy(), ref[i][0])
                assert np.array_equal(v[0].cpu().numpy(), ref[i][1])
                assert np.array_equal(ref[i][0], Kh[i][:, :n])
                assert np.array_equal(ref[i][1], Vh[i][:, :n])

        # prefill through a DynamicCache, as an HF model returns it
        mgr.ingest_step(KVCacheManager._from_legacy(pkv(T0)))
        model.ingest_step(kv_np(T0))
        same_blocks()
        evicted_any = spilled_any = 0
        for s in range(steps):
            n = T0 + s + 1
            mgr.append_token(pkv(n))
            model.append_token(kv_np(n))
            for layer in range(Ly):
                logits = torch.randn(1, Hq, 1, n, generator=g, device="cuda") * 2.0
                attn = torch.softmax(logits, dim=-1)
                mgr.report_attention(layer, attn)
                model.report_attention(layer, attn.float().mean(dim=(0, 2)))
            mgr.step_done()
            model.step_done()
            got = mgr.schedule()
            got.pop("tm_stats")
            want = model.schedule()
            assert got == want, s
            evicted_any += got["evicted"]
            same_blocks()
            same_stats()
            spilled_any = max(spilled_any, model.get_stats()["blocks_ssd"])
            for b in model.all_blocks():
                if b.tier == TIER_SSD:
                    with open(os.path.join(ssd, f"blk_{b.block_id}.bin"), "rb") as fh:
                        assert fh.read() == b.file_bytes
            if s % 5 == 4:
                check_build(n)
                same_stats()
        assert evicted_any > 0 and spilled_any > 0
        assert model.get_stats()["migrations"]["ssd_to_dram"] > 0

        got, want = _tm_state(mgr._tm_handle), model.tm.s.state()
        for key in ("hits", "last"):
            assert np.array_equal(got[key], want[key]), key
        for key in ("sum", "ema"):
            a, b = got[key], want[key]
            assert np.all(np.abs(a - b) <= REL * np.maximum(np.abs(b), 1e-30)), key
        assert np.count_nonzero(want["hits"]) > 30
    finally:
        mgr.destroy()
