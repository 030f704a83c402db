"""The oracle's restatements of the reference's two Python managers pinned
to the reference itself.  Replayed on the seeded inputs of a fixture recorded
from the reference's own module, each model makes every tracker call the
reference made, in the same order with the same arguments (scores and usage
ratios bit for bit), and reaches the same results after every step:

* oracle/kvcache_manager_model.py vs python/orchkv/kvcache_manager.py
  (tests/golden/kvcache_manager_decode.json, gen_kvcache_manager.py):
  schedule results, statistics, block tiers and access counts, also after
  every rebuild;
* oracle/fast_manager_model.py vs python/orchkv/fast_kvcache_manager.py
  (tests/golden/fast_manager_decode.json, gen_fast_manager.py, the reference
  run against the reference scheduler compiled from its sources): schedule
  results, statistics and evicted blocks, also after every restore."""
import json
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


class RecordingTM:
    """The oracle tracker behind a log in the fixture's call format."""

    def __init__(self, tm, f32bits):
        self.tm, self.f32bits, self.calls = tm, f32bits, []

    def register(self, bid, tier=0, flags=0):
        self.calls.append(["reg", int(bid), int(tier), int(flags)])
        return self.tm.register(bid, tier, flags)

    def report(self, bid, w):
        self.calls.append(["rep", int(bid), self.f32bits(w)])
        self.tm.report(bid, w)

    def step_done(self):
        self.calls.append(["step"])
        self.tm.step_done()

    def set_usage(self, g, d):
        self.calls.append(["usage", self.f32bits(g), self.f32bits(d)])
        self.tm.set_usage(g, d)

    def schedule_once(self):
        self.calls.append(["sched"])
        self.tm.schedule_once()

    def set_block_tier(self, bid, tier):
        self.calls.append(["tier", int(bid), int(tier)])
        self.tm.set_block_tier(bid, tier)

    def __getattr__(self, name):               # reads (score, heat, stats, s) pass through
        return getattr(self.tm, name)


def test_model_matches_reference_manager_run(oracle_mod):
    from oracle.kvcache_manager_model import ModelKVManager
    from tests.golden.gen_kvcache_manager import f32bits, inputs
    with open(os.path.join(HERE, "golden", "kvcache_manager_decode.json")) as fh:
        fx = json.load(fh)
    c = fx["case"]
    k, v, attn = inputs(c)
    block_bytes = 2 * c["n_kv_heads"] * c["block_size"] * c["head_dim"] * 2
    model = ModelKVManager(c["n_layers"], c["n_kv_heads"], c["head_dim"], c["block_size"],
                           np.float16, c["budget_blocks"] * block_bytes, True, c["sink_tokens"],
                           tracker_cap=4096)
    model.tm = RecordingTM(model.tm, f32bits)

    def kv(n):
        return [(k[i][:, :n], v[i][:, :n]) for i in range(c["n_layers"])]

    def blocks():
        return [[b.block_id, b.token_start, b.token_count, b.tier, b.access_count,
                 int(b.is_sink)] for b in model.all_blocks()]

    model.ingest_step(kv(c["prefill"]))
    for s, want in enumerate(fx["steps"]):
        n = c["prefill"] + s + 1
        model.append_token(kv(n))
        for layer in range(c["n_layers"]):
            model.report_attention(layer, torch.from_numpy(attn[s][layer]).float()
                                   .mean(dim=(0, 2)))
        model.step_done()
        assert model.schedule() == want["schedule"], s
        assert model.get_stats() == want["stats"], s
        assert blocks() == want["blocks"], s
        if "after_build" in want:
            model.build_past_kv()
            assert model.get_stats() == want["after_build"]["stats"], s
            assert blocks() == want["after_build"]["blocks"], s
    assert model.tm.calls == fx["calls"]
    assert want["stats"]["migrations"]["ssd_to_dram"] > 0


def test_fast_model_matches_reference_manager_run(oracle_mod):
    from oracle.fast_manager_model import FastManagerModel
    from tests.golden.gen_fast_manager import inputs
    from tests.golden.gen_kvcache_manager import f32bits
    with open(os.path.join(HERE, "golden", "fast_manager_decode.json")) as fh:
        fx = json.load(fh)
    c = fx["case"]
    k0, v0, kt, vt, attn = inputs(c)
    L, H, d, bs = c["n_layers"], c["n_kv_heads"], c["head_dim"], c["block_size"]
    model = FastManagerModel(L, H, d, block_size=bs, dtype=np.float16,
                             gpu_budget_bytes=c["budget_blocks_per_layer"] * L * 2 * H * bs * d * 2,
                             max_seq_len=c["max_seq_len"], sink_tokens=c["sink_tokens"])
    model.tm = RecordingTM(model.tm, f32bits)
    model.ingest([k0[i] for i in range(L)], [v0[i] for i in range(L)])
    for s, want in enumerate(fx["steps"]):
        model.append([kt[s, i] for i in range(L)], [vt[s, i] for i in range(L)])
        for layer in range(L):
            model.report_attention(attn[s][layer][0, :, 0, :])
        model.step_done()
        assert model.schedule() == want["schedule"], s
        assert model.get_stats() == want["stats"], s
        assert model.evicted_blocks() == want["evicted"], s
        if "after_restore" in want:
            model.restore()
            assert model.get_stats() == want["after_restore"]["stats"], s
    assert model.tm.calls == fx["calls"]
    assert sum(st["stats"]["migrations"]["evictions_this_step"] for st in fx["steps"]) > 20


def test_hook_model_matches_reference_hook_run():
    """oracle/hook_model.py (the report sequence the GPU hook tests compare
    with) against the reference's own AttentionScoreCollector
    (tests/golden/attention_hook_reports.json, gen_attention_hook.py): the
    same tm_report_attn calls, scores bit for bit, in every block-id mode,
    on the sampled steps only."""
    from oracle.hook_model import hook_reports
    from tests.golden.gen_attention_hook import MODES, id_fn, weights
    from tests.golden.gen_kvcache_manager import f32bits
    with open(os.path.join(HERE, "golden", "attention_hook_reports.json")) as fh:
        fx = json.load(fh)
    c = fx["case"]
    ws = weights(c)
    table = torch.tensor([c["table"]], dtype=torch.int64)
    calls = []
    for s in range(c["steps"]):
        if s % c["sample_interval"] == 0:
            for layer, mode in enumerate(MODES):
                for bid, score in hook_reports(layer, torch.from_numpy(ws[s][layer]),
                                               c["block_size"],
                                               table if mode == "table" else None,
                                               id_fn(mode)):
                    calls.append(["rep", bid, f32bits(score)])
        calls.append(["step"])
    assert calls == fx["calls"]
    assert fx["stats"]["blocks_reported"] == sum(1 for x in calls if x[0] == "rep")
