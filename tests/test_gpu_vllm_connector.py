"""orchkv_b200.vllm_connector against the behaviour of the reference's
python/orchkv/vllm_integration/connector.py: saved blocks come back
byte-identical after the GPU copy is overwritten, statistics count as the
reference counts (saves and loads per block and layer, one DRAM buffer per
saved (layer, block)), freed blocks are no longer loadable, and the
scheduler side produces the reference's metadata.  Cache tensors use the
[num_blocks, 2, block_size, kv_heads, head_dim] layout the reference indexes
with kv_layer[block_id]; one layer is a strided view to take the per-block
fallback."""
from types import SimpleNamespace

import pytest

pytestmark = pytest.mark.gpu


def _caches(torch, n_layers=3, nb=96):
    g = torch.Generator(device="cuda").manual_seed(5)
    kv = {}
    for i in range(n_layers):
        kv[f"layer_{i}"] = torch.randn(nb, 2, 16, 4, 64, generator=g, device="cuda",
                                       dtype=torch.float16)
    # a cache whose blocks are not contiguous chunks: [2, nb, ...] seen as [nb, 2, ...]
    base = torch.randn(2, nb, 16, 4, 64, generator=g, device="cuda", dtype=torch.float16)
    kv[f"layer_{n_layers}"] = base.transpose(0, 1)
    return kv


def test_worker_save_load_round_trip(cuda):
    torch = cuda
    from orchkv_b200.vllm_connector import OrchKvConnectorMetadata, OrchKvConnectorWorker
    w = OrchKvConnectorWorker({"dram_pool_bytes": 64 << 20, "d_head": 64})
    kv = _caches(torch)
    w.register_kv_caches(kv)
    try:
        orig = {k: v.clone() for k, v in kv.items()}
        blocks = [3, 7, 8, 20, 95]
        meta = OrchKvConnectorMetadata(blocks_to_save={k: list(blocks) for k in kv})
        for name, t in kv.items():
            w.save_kv_layer(name, t, meta)
        w.wait_for_save()
        for t in kv.values():
            t[blocks] = 0
        load = OrchKvConnectorMetadata(blocks_to_load={k: list(blocks) for k in kv})
        w.start_load_kv(load)
        for name in kv:
            w.wait_for_layer_load(name)
        for name in kv:
            assert torch.equal(kv[name], orig[name]), name
        n = len(kv) * len(blocks)
        assert w.get_stats() == {"save_count": n, "load_count": n, "dram_buffers": n}

        # more blocks than the first store held: the store grows, old slots kept
        more = list(range(30, 80))
        meta2 = OrchKvConnectorMetadata(blocks_to_save={k: more for k in kv})
        for name, t in kv.items():
            w.save_kv_layer(name, t, meta2)
        w.wait_for_save()
        for t in kv.values():
            t[blocks + more] = 0
        w.start_load_kv(OrchKvConnectorMetadata(
            blocks_to_load={k: blocks + more for k in kv}))
        for name in kv:
            w.wait_for_layer_load(name)
            assert torch.equal(kv[name], orig[name]), name
        assert w.get_stats()["dram_buffers"] == len(kv) * (len(blocks) + len(more))

        # freed blocks are gone: loading them leaves the GPU copy alone
        w.free_blocks("layer_0", [3, 7])
        assert w.get_stats()["dram_buffers"] == len(kv) * (len(blocks) + len(more)) - 2
        kv["layer_0"][[3, 7]] = 1
        w.start_load_kv(OrchKvConnectorMetadata(blocks_to_load={"layer_0": [3, 7, 8]}))
        w.wait_for_layer_load("layer_0")
        assert bool((kv["layer_0"][[3, 7]] == 1).all())
        assert torch.equal(kv["layer_0"][8], orig["layer_0"][8])
    finally:
        w.shutdown()


def test_connector_roles_and_scheduler_metadata(cuda):
    torch = cuda
    from orchkv_b200.vllm_connector import (KVConnectorRole, OrchKvConnectorMetadata,
                                            OrchKvOffloadingConnector)
    cfg = SimpleNamespace(
        kv_transfer_config=SimpleNamespace(kv_connector_extra_config={"dram_pool_gb": 1,
                                                                      "n_layers": 2}),
        model_config=SimpleNamespace(head_dim=64))
    sched = OrchKvOffloadingConnector(cfg, KVConnectorRole.SCHEDULER)
    req = SimpleNamespace(request_id="r1")
    assert sched.get_num_new_matched_tokens(req, 0) == (0, False)
    assert sched.request_finished(req, [4, 5, 6]) == (False, None)
    assert sched.get_num_new_matched_tokens(req, 1) == (2, True)
    sched.handle_preemptions({"r1"})
    meta = sched.build_connector_meta(None)
    assert {k: sorted(v) for k, v in meta.blocks_to_save.items()} == {
        "layer_0": [4, 5, 6], "layer_1": [4, 5, 6]}
    assert sched.build_connector_meta(None).blocks_to_save == {}

    wk = OrchKvOffloadingConnector(cfg, KVConnectorRole.WORKER)
    kv = _caches(torch, n_layers=2, nb=16)
    del kv["layer_2"]
    wk.register_kv_caches(kv)
    try:
        orig = {k: v.clone() for k, v in kv.items()}
        wk.bind_connector_metadata(meta)
        for name, t in kv.items():
            wk.save_kv_layer(name, t, None)
        wk.wait_for_save()
        for t in kv.values():
            t[[4, 5, 6]] = 0
        wk.bind_connector_metadata(OrchKvConnectorMetadata(
            blocks_to_load={k: [4, 5, 6] for k in kv}))
        wk.start_load_kv(None)
        for name in kv:
            wk.wait_for_layer_load(name)
            assert torch.equal(kv[name], orig[name])
        assert wk.prefer_cross_layer_blocks
    finally:
        wk.shutdown()


def test_worker_pinned_bytes_cap(cuda):
    """dram_pool_bytes caps the pinned bytes the worker's stores hold: a save
    that would grow a store past it raises and changes nothing; a freed slot
    is reused without growing."""
    torch = cuda
    from orchkv_b200.vllm_connector import OrchKvConnectorMetadata, OrchKvConnectorWorker
    kv = _caches(torch, n_layers=1, nb=64)
    del kv["layer_1"]                                   # keep the contiguous layer
    t = kv["layer_0"]
    slot = t[0].numel() * t.element_size()              # 16 KB per block
    w = OrchKvConnectorWorker({"dram_pool_bytes": 16 * slot})
    w.register_kv_caches(kv)
    try:
        orig = t.clone()
        w.save_kv_layer("layer_0", t, None, block_ids=list(range(16)))   # one 16-slot store
        w.wait_for_save()
        assert w.get_stats() == {"save_count": 16, "load_count": 0, "dram_buffers": 16}
        with pytest.raises(RuntimeError):
            w.save_kv_layer("layer_0", t, None, block_ids=[40])   # a 17th slot: 32 slots
        assert w.get_stats() == {"save_count": 16, "load_count": 0, "dram_buffers": 16}
        w.free_blocks("layer_0", [3])
        w.save_kv_layer("layer_0", t, None, block_ids=[40])       # takes the freed slot
        w.wait_for_save()
        t[[0, 40]] = 0
        w.start_load_kv(OrchKvConnectorMetadata(blocks_to_load={"layer_0": [0, 40]}))
        w.wait_for_layer_load("layer_0")
        assert torch.equal(t, orig)
        assert w.get_stats() == {"save_count": 17, "load_count": 2, "dram_buffers": 16}
    finally:
        w.shutdown()
