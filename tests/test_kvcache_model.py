"""The oracle's restatement of the reference KVCacheManager
(oracle/kvcache_manager_model.py) pinned to the reference itself: replayed on
the seeded inputs of tests/golden/kvcache_manager_decode.json (recorded from
the reference's python/orchkv/kvcache_manager.py by
tests/golden/gen_kvcache_manager.py), it makes every tracker call the
reference made, in the same order with the same arguments (scores and usage
ratios bit for bit), and reaches the same schedule results, statistics, block
tiers and access counts after every step and every rebuild."""
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
