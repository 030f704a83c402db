"""orchkv_b200.attention_hook against the reference's
python/orchkv/vllm_integration/attention_hook.py: the collector's sampling
schedule and statistics, the block-mean scores (checked against torch's own
mean over the same padded view, the reduction the reference runs), and the
reports: after collecting several layers in each block-id mode (the default
layer/head/block ids, a block_id_fn, a block table whose ids every head
shares, and a mapping that puts two blocks on one tracker slot), the device
tracker equals the oracle tracker fed the reference's per-block
tm_report_attn sequence (oracle/hook_model.py, pinned to the reference
hook's own run) -- hits and last-hit steps exact, sums and EMA
within 1e-5 relative (the mean is summed in another order).  Also the hook
manager's wrapping of a model's self-attention modules."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL = 1e-5


@pytest.fixture
def hook_mod(cuda):
    from orchkv_b200 import attention_hook
    return attention_hook


@pytest.fixture
def tm(cuda):
    import orchkv_b200 as o
    core = o.core()
    h = core.tm_create(tracker_cap=1024, ema_lambda=0.9)
    yield h
    core.tm_destroy(h)


def torch_block_mean(torch, aw, n_blocks, block_size):
    """The reference's reduction (attention_hook.py:118-140), from the oracle's
    hook model (pinned to the reference hook's own run)."""
    from oracle.hook_model import block_means
    out = block_means(aw, block_size)
    assert out.shape[1] == n_blocks
    return out


def softmax_weights(torch, g, shape, dtype=None):
    w = torch.softmax(torch.randn(*shape, generator=g, device="cuda") * 2.0, dim=-1)
    return w if dtype is None else w.to(dtype)


# ---- sampling schedule and statistics -------------------------------------

def test_sampling_schedule(hook_mod, tm):
    c = hook_mod.AttentionScoreCollector(tm, block_size=16, sample_interval=5)
    assert (c.block_size, c.sample_interval, c._step) == (16, 5, 0)
    c.sample_interval = 3
    seen = []
    for _ in range(9):
        seen.append(c.should_sample())
        c.on_step_done()
    assert seen == [True, False, False] * 3
    c.set_enabled(False)
    assert not c.should_sample()
    c.set_enabled(True)
    c.sample_interval = 0
    assert c.sample_interval == 1


def test_stats_count_like_the_reference(hook_mod, tm, cuda):
    torch = cuda
    c = hook_mod.AttentionScoreCollector(tm, block_size=4, sample_interval=2)
    aw = torch.rand(1, 1, 1, 4, device="cuda")
    calls = []
    for _ in range(3):
        c.collect(0, aw, block_id_fn=lambda l, h, bi: calls.append(bi) or bi)
        c.on_step_done()
    st = c.get_stats()
    # steps 0 and 2 sampled; on_step_done counts the step it moves to
    assert len(calls) == 2 and st["blocks_reported"] == 2
    assert st["current_step"] == 3
    assert (st["samples_taken"], st["steps_skipped"]) == (1, 2)


# ---- the block-mean reduction ---------------------------------------------

def test_block_mean_known_values(hook_mod, tm, cuda):
    """The reference's reduction known answers (test/test_attention_hook.py:67-99)."""
    torch = cuda
    c = hook_mod.AttentionScoreCollector(tm, block_size=4, sample_interval=1)
    s = c._blockwise_reduce(torch.full((1, 2, 1, 8), 0.5, device="cuda"), 2)
    assert s.shape == (2, 2) and torch.allclose(s, torch.full_like(s, 0.5))
    s = c._blockwise_reduce(torch.ones(1, 1, 1, 6, device="cuda"), 2)      # padded tail
    assert s[0].tolist() == [1.0, 0.5]
    aw = torch.zeros(2, 4, 3, 12, device="cuda")
    for h in range(4):
        aw[:, h] = (h + 1) * 0.1
    s = c._blockwise_reduce(aw, 3)
    for h in range(4):
        assert torch.allclose(s[h], torch.full_like(s[h], (h + 1) * 0.1), atol=1e-6)


@pytest.mark.parametrize("shape,block_size", [((3, 8, 1, 1000), 16), ((2, 4, 5, 4096), 64),
                                              ((1, 2, 2, 77), 32), ((4, 3, 1, 300), 512)])
@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
def test_block_mean_matches_torch(hook_mod, tm, cuda, shape, block_size, dtype):
    torch = cuda
    dt = getattr(torch, dtype)
    g = torch.Generator(device="cuda").manual_seed(7)
    aw = softmax_weights(torch, g, shape, dt)
    c = hook_mod.AttentionScoreCollector(tm, block_size=block_size, sample_interval=1)
    nb = (shape[3] + block_size - 1) // block_size
    got = c._blockwise_reduce(aw, nb)
    want = torch_block_mean(torch, aw, nb, block_size)
    assert got.dtype == want.dtype and got.shape == want.shape
    a, b = got.float(), want.float()
    if dt == torch.float32:
        assert torch.all((a - b).abs() <= REL * b.abs().clamp_min(1e-30))
    else:
        # rounded to the weights' type: equal, or one unit in the last place
        # where the fp32 means straddle a rounding boundary
        ulp = 2.0 ** -7 if dt == torch.bfloat16 else 2.0 ** -10
        assert torch.all((a - b).abs() <= ulp * b.abs().clamp_min(1e-30))
        assert (a == b).float().mean().item() > 0.98


# ---- reports against the oracle tracker ------------------------------------

def _state(tm_handle):
    import orchkv_b200 as o
    from orchkv_b200._lib import TieredManager
    L = o.lib()
    m = C.cast(C.c_void_p(tm_handle), C.POINTER(TieredManager))
    n = L.tm_capacity(m)
    out = {"sum": np.zeros(n, np.float32), "ema": np.zeros(n, np.float32),
           "hits": np.zeros(n, np.uint32), "last": np.zeros(n, np.uint64)}
    assert L.tm_read_state(m, out["sum"].ctypes.data, out["ema"].ctypes.data,
                           out["hits"].ctypes.data, out["last"].ctypes.data,
                           None, None, None, None) == 0
    return out


def test_reports_match_reference_sequence(hook_mod, cuda, oracle_mod):
    torch = cuda
    import orchkv_b200 as o
    core = o.core()
    cap = 4096
    tm = core.tm_create(tracker_cap=cap, ema_lambda=0.9)
    try:
        orc = oracle_mod.OracleSched(cap, 0.9, 0.5, 0.3, 0.2, 50.0)
        H, bsz, kv, blk = 4, 2, 100, 16
        nb = (kv + blk - 1) // blk
        for bid in range(3000):
            assert core.tm_register_block_id(tm, bid, 0, 0) == 0
            orc.register(bid)
        c = hook_mod.AttentionScoreCollector(tm, block_size=blk, sample_interval=1)
        g = torch.Generator(device="cuda").manual_seed(3)
        table = torch.tensor([[2000 + 7 * i for i in range(nb - 2)]], device="cuda")
        from oracle.hook_model import hook_reports
        modes = [
            ("default", {}),
            ("fn", {"block_id_fn": lambda layer, h, bi: 1000 + 31 * h + bi}),
            ("table", {"block_table": table}),
            # blocks 0, 3 and 6 all report to id 2500: one tracker slot, three columns
            ("shared", {"block_id_fn": lambda layer, h, bi: 2500 + (bi % 3) + 4 * h}),
        ]
        for step in range(3):
            for layer, (name, kw) in enumerate(modes):
                aw = softmax_weights(torch, g, (bsz, H, 1, kv))
                c.collect(layer, aw, **kw)
                # the reference hook's report sequence (oracle/hook_model.py)
                for bid, score in hook_reports(layer, aw, blk, kw.get("block_table"),
                                               kw.get("block_id_fn")):
                    orc.update(bid, score)
            c.on_step_done()
            orc.step_done()
        core.tm_sync(tm)
        got, want = _state(tm), orc.state()
        for key in ("hits", "last"):
            assert np.array_equal(got[key], want[key]), key
        for key in ("sum", "ema"):
            a, b = got[key], want[key]
            assert np.all(np.abs(a - b) <= REL * np.maximum(np.abs(b), 1e-30)), key
        assert np.count_nonzero(want["hits"]) > 60          # every mode touched its slots
        assert c.get_stats()["blocks_reported"] == 3 * len(modes) * H * nb
    finally:
        core.tm_destroy(tm)


# ---- the hook manager -------------------------------------------------------

def _mock_model(torch, n_layers, heads, kv_len):
    class SelfAttn(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.calls = 0

        def forward(self, x, output_attentions=False, **kwargs):
            self.calls += 1
            out = torch.zeros(1, heads, 1, 8, device="cuda")
            if output_attentions:
                w = torch.rand(1, heads, 1, kv_len, device="cuda")
                return out, w / w.sum(-1, keepdim=True)
            return (out,)

    model = torch.nn.Module()
    model.layers = torch.nn.ModuleList()
    for _ in range(n_layers):
        layer = torch.nn.Module()
        layer.self_attn = SelfAttn()
        model.layers.append(layer)
    return model


def test_hook_manager_wraps_and_feeds(hook_mod, tm, cuda):
    torch = cuda
    c = hook_mod.AttentionScoreCollector(tm, block_size=4, sample_interval=5)
    mgr = hook_mod.AttentionHookManager(c)
    assert mgr.collector is c
    model = _mock_model(torch, 2, 2, 16)
    mgr.install(model)
    st = mgr.get_stats()
    assert st["installed"] and st["n_layers_hooked"] == 2
    x = torch.zeros(1, 1, 8, device="cuda")
    for step in range(20):
        for layer in model.layers:
            res = layer.self_attn(x)
            assert len(res) == (2 if step % 5 == 0 else 1)
        mgr.on_step_done()
    cs = c.get_stats()
    assert cs["current_step"] == 20 and cs["samples_taken"] == 4
    assert cs["blocks_reported"] == 4 * 2 * 2 * 4       # samples x layers x heads x blocks
    mgr.uninstall()
    assert not mgr.get_stats()["installed"]
    assert len(model.layers[0].self_attn(x, output_attentions=False)) == 1


def test_blockmean_rejects_bad_arguments(hook_mod, tm, cuda):
    """Invalid shapes, types, block sizes and null buffers return
    ORCHKV_ERR_INVALID (-2)."""
    torch = cuda
    import orchkv_b200 as o
    core = o.core()
    w = torch.rand(1, 2, 1, 64, device="cuda")
    s = torch.zeros(2, 4, device="cuda")
    ids = torch.zeros(2, 4, dtype=torch.int32, device="cuda")
    ok = (tm, w.data_ptr(), 2, 1, 2, 1, 64, 16, ids.data_ptr(), s.data_ptr())
    assert core.tm_report_attn_blockmean(*ok) == 0
    bad = [
        dict(i=2, v=3),            # dtype
        dict(i=3, v=0),            # batch
        dict(i=4, v=0),            # heads
        dict(i=5, v=0),            # q_len
        dict(i=6, v=0),            # kv_len
        dict(i=7, v=0),            # block_size
        dict(i=7, v=8192),         # block_size above 4096
        dict(i=1, v=0),            # weights
        dict(i=9, v=0),            # scores
    ]
    for b in bad:
        args = list(ok)
        args[b["i"]] = b["v"]
        assert core.tm_report_attn_blockmean(*args) == -2, b


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("shape,block_size", [((2, 8, 3, 4096), 16), ((1, 4, 1, 8192), 256),
                                              ((3, 2, 2, 1024), 4096), ((1, 1, 1, 64), 8),
                                              ((32, 28, 1, 8192), 16), ((5, 4, 3, 2048), 16)])
def test_block_mean_vector_path_is_bit_identical(hook_mod, tm, cuda, shape, block_size, dtype):
    """The 16-byte-load kernel (aligned weights, kv_len and block_size
    multiples of the vector width) against the one-element kernel (the same
    weights one element off a 16-byte boundary): scores equal bit for bit.
    The shapes cover one row group and several (the rows are split into up
    to 8 groups when heads x tokens alone would not fill the GPU), uneven
    groups and a group that starts mid-batch (15 rows of 3 query
    positions, groups of 8 and 7)."""
    torch = cuda
    import orchkv_b200 as o
    core = o.core()
    dt = getattr(torch, dtype)
    code = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}[dt]
    vw = 4 if dt == torch.float32 else 8
    if block_size % vw:
        pytest.skip("block size below the vector width")
    g = torch.Generator(device="cuda").manual_seed(5)
    aw = softmax_weights(torch, g, shape, dt).contiguous()
    n = aw.numel()
    flat = torch.empty(n + 1, dtype=dt, device="cuda")
    flat[1:].copy_(aw.reshape(-1))
    off = flat[1:]
    assert aw.data_ptr() % 16 == 0 and off.data_ptr() % 16 != 0
    B, H, Q, T = shape
    nb = (T + block_size - 1) // block_size
    ids = torch.zeros(H, nb, dtype=torch.int32, device="cuda")
    s_vec = torch.zeros(H, nb, device="cuda")
    s_one = torch.zeros(H, nb, device="cuda")
    assert core.tm_report_attn_blockmean(tm, aw.data_ptr(), code, B, H, Q, T, block_size,
                                         ids.data_ptr(), s_vec.data_ptr()) == 0
    assert core.tm_report_attn_blockmean(tm, off.data_ptr(), code, B, H, Q, T, block_size,
                                         ids.data_ptr(), s_one.data_ptr()) == 0
    core.tm_sync(tm)
    assert torch.equal(s_vec.view(torch.int32), s_one.view(torch.int32))
    want = torch_block_mean(torch, aw, nb, block_size).float()
    rel = REL if dt == torch.float32 else (2.0 ** -7 if dt == torch.bfloat16 else 2.0 ** -10)
    assert torch.all((s_vec - want).abs() <= rel * want.abs().clamp_min(1e-30))


@pytest.mark.parametrize("mode", ["default", "table", "fn"])
def test_reports_more_heads_than_a_warp(hook_mod, cuda, oracle_mod, mode):
    """72 heads: the tracker apply takes a column's heads 32 at a time, so a
    slot shared by every head of a column (block-table mode) is updated in
    three chunks that must follow one another in head order.  The tracker
    equals the oracle fed the reference hook's per-block report sequence."""
    torch = cuda
    import orchkv_b200 as o
    core = o.core()
    cap = 8192
    tm = core.tm_create(tracker_cap=cap, ema_lambda=0.9)
    try:
        orc = oracle_mod.OracleSched(cap, 0.9, 0.5, 0.3, 0.2, 50.0)
        H, bsz, kv, blk = 72, 2, 200, 16
        nb = (kv + blk - 1) // blk
        for bid in range(6000):
            assert core.tm_register_block_id(tm, bid, 0, 0) == 0
            orc.register(bid)
        c = hook_mod.AttentionScoreCollector(tm, block_size=blk, sample_interval=1)
        g = torch.Generator(device="cuda").manual_seed(9)
        kw = {"default": {},
              "table": {"block_table": torch.tensor([[5000 + 3 * i for i in range(nb)]],
                                                    device="cuda")},
              # heads 0-35 and 36-71 pairwise share an id: groups span chunks
              "fn": {"block_id_fn": lambda layer, h, bi: 4000 + 40 * bi + (h % 36)}}[mode]
        from oracle.hook_model import hook_reports
        for step in range(3):
            for layer in range(2):
                aw = softmax_weights(torch, g, (bsz, H, 1, kv))
                c.collect(layer, aw, **kw)
                for bid, score in hook_reports(layer, aw, blk, kw.get("block_table"),
                                               kw.get("block_id_fn")):
                    orc.update(bid, score)
            c.on_step_done()
            orc.step_done()
        core.tm_sync(tm)
        got, want = _state(tm), orc.state()
        for key in ("hits", "last"):
            assert np.array_equal(got[key], want[key]), key
        for key in ("sum", "ema"):
            a, b = got[key], want[key]
            assert np.all(np.abs(a - b) <= REL * np.maximum(np.abs(b), 1e-30)), key
        assert np.count_nonzero(want["hits"]) >= nb
    finally:
        core.tm_destroy(tm)


@pytest.mark.parametrize("shape,dtype", [((4, 8, 1, 8192), "float32"),
                                         ((4, 8, 1, 8192), "bfloat16"),
                                         ((32, 4, 1, 4096), "bfloat16")])
@pytest.mark.parametrize("mode", ["default", "column"])
def test_reports_over_many_tiles(cuda, oracle_mod, shape, dtype, mode):
    """Decode-length weights (several CTA tiles of blocks in the block-mean
    launch, the row-split instance for 32 rows): the oracle tracker is fed
    the launch's own scores in the reference hook's order (head by head,
    block by block), so with distinct ids per (head, block) and with every
    head of a column on one id the tracker must be bit-identical."""
    torch = cuda
    import orchkv_b200 as o
    core = o.core()
    bsz, H, q, kv = shape
    blk = 16
    nb = kv // blk
    code = {"float16": 0, "bfloat16": 1, "float32": 2}[dtype]
    cap = 1 << 15
    tm = core.tm_create(tracker_cap=cap, ema_lambda=0.9)
    try:
        orc = oracle_mod.OracleSched(cap, 0.9, 0.5, 0.3, 0.2, 50.0)
        h_idx = torch.arange(H, device="cuda")[:, None]
        b_idx = torch.arange(nb, device="cuda")[None, :]
        if mode == "default":
            tables = [(layer * H * nb + h_idx * nb + b_idx).int() for layer in range(2)]
        else:
            tables = [(20000 + 600 * layer + b_idx).expand(H, nb).int().contiguous()
                      for layer in range(2)]
        for bid in sorted({int(x) for t in tables for x in t.flatten().tolist()}):
            assert core.tm_register_block_id(tm, bid, 0, 0) == 0
            orc.register(bid)
        scores = torch.empty(H, nb, dtype=torch.float32, device="cuda")
        g = torch.Generator(device="cuda").manual_seed(21)
        for step in range(3):
            for layer in range(2):
                aw = softmax_weights(torch, g, shape, getattr(torch, dtype)).contiguous()
                assert core.tm_report_attn_blockmean(tm, aw.data_ptr(), code, bsz, H, q, kv, blk,
                                                     tables[layer].data_ptr(),
                                                     scores.data_ptr()) == 0
                core.tm_sync(tm)
                ids_h, sc_h = tables[layer].cpu().numpy(), scores.cpu().numpy()
                for h in range(H):
                    for bi in range(nb):
                        orc.update(int(ids_h[h, bi]), float(sc_h[h, bi]))
            core.tm_step_done(tm)
            orc.step_done()
        core.tm_sync(tm)
        got, want = _state(tm), orc.state()
        for key in ("hits", "last", "sum", "ema"):
            assert np.array_equal(got[key], want[key]), key
        assert np.count_nonzero(want["hits"]) >= 2 * nb
    finally:
        core.tm_destroy(tm)
