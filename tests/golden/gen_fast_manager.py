"""Generate tests/golden/fast_manager_decode.json by running the reference's
own python/orchkv/fast_kvcache_manager.py (FastKVCacheManager) over a seeded
decode loop on the CPU, with an orchkv_core stand-in backed by the
reference's scheduler compiled from its sources (oracle/_ref), so the
manager's score-ordered evictions see the reference's own scores.  Every
mutating call the manager makes (register, report, step, usage, schedule) is
recorded, with every tm_get_block_score the manager asks for (its position in
the call stream, the block and the reference's answer), and after each step
its schedule result, statistics and the set of evicted blocks.

Only needed to regenerate; the fixture is committed.  Needs the reference
source tree and `make -C oracle`.

    python tests/golden/gen_fast_manager.py
"""
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from tests.golden.refpath import reference_file  # noqa: E402

from oracle import oracle as O  # noqa: E402
from tests.golden.gen_kvcache_manager import f32bits, load_reference  # noqa: E402

REFERENCE = "python/orchkv/fast_kvcache_manager.py"      # inside the reference tree (tests/golden/refpath.py)
CASE = dict(n_layers=4, n_kv_heads=2, q_heads=4, head_dim=64, block_size=16, max_seq_len=1024,
            prefill=700, steps=40, budget_blocks_per_layer=40, sink_tokens=4, restore_every=6,
            seed=3)


def inputs(case):
    """Seeded prefill K/V [layer][head][token][d], one new token per step and
    layer, and attention weights per (step, layer) in multiples of 1/4096
    (every per-block sum is exact in fp32, whatever the summation order)."""
    rng = np.random.default_rng(case["seed"])
    L, H, d = case["n_layers"], case["n_kv_heads"], case["head_dim"]
    k0 = rng.standard_normal((L, H, case["prefill"], d)).astype(np.float16)
    v0 = rng.standard_normal((L, H, case["prefill"], d)).astype(np.float16)
    kt = rng.standard_normal((case["steps"], L, H, d)).astype(np.float16)
    vt = rng.standard_normal((case["steps"], L, H, d)).astype(np.float16)
    attn = []
    for s in range(case["steps"]):
        t = case["prefill"] + s + 1
        attn.append([(rng.integers(0, 16, (1, case["q_heads"], 1, t)) / 4096.0)
                     .astype(np.float32) for _ in range(L)])
    return k0, v0, kt, vt, attn


class RefCore(types.ModuleType):
    """orchkv_core stand-in over the compiled reference scheduler."""
    GPU_HBM, HOST_DRAM, SSD = 0, 1, 3

    def __init__(self):
        super().__init__("orchkv_core")
        self.calls = []
        self.scores = []
        self.tm = None

    def tm_create(self, *a, **k):
        self.tm = O.RefTM(cooldown_sec=0.0)     # the binding's defaults, no wall-clock gate
        return 1

    def tm_destroy(self, h):
        self.tm.close()

    def tm_register_block_id(self, h, bid, a=0, b=0):
        self.calls.append(["reg", int(bid), int(a), int(b)])
        return self.tm.register(int(bid), int(a), int(b))

    def tm_report_attn(self, h, bid, score):
        self.calls.append(["rep", int(bid), f32bits(score)])
        self.tm.report(int(bid), float(score))

    def tm_step_done(self, h):
        self.calls.append(["step"])
        self.tm.step_done()

    def tm_set_usage(self, h, g, d):
        self.calls.append(["usage", f32bits(g), f32bits(d)])
        self.tm.set_usage(g, d)

    def tm_schedule_once(self, h):
        self.calls.append(["sched"])
        self.tm.schedule_once()

    def tm_get_block_score(self, h, bid):
        sc = self.tm.score(int(bid))
        # where in the call stream the manager asked, and what it was told
        self.scores.append([len(self.calls), int(bid), f32bits(sc)])
        return sc

    def tm_get_stats(self, h):
        return {}


def main():
    if not O.ref_available():
        raise SystemExit("build the reference first: make -C oracle")
    c = CASE
    core = RefCore()
    mod = load_reference(core, reference_file(REFERENCE), "ref_fast_kvcache_manager")
    k0, v0, kt, vt, attn = inputs(c)
    L, H, d, bs = c["n_layers"], c["n_kv_heads"], c["head_dim"], c["block_size"]
    block_bytes = 2 * H * bs * d * 2
    mgr = mod.FastKVCacheManager(L, H, d, block_size=bs, dtype=torch.float16,
                                 gpu_budget_bytes=c["budget_blocks_per_layer"] * L * block_bytes,
                                 max_seq_len=c["max_seq_len"], sink_tokens=c["sink_tokens"])
    mgr.ingest_step(tuple((torch.from_numpy(k0[i])[None], torch.from_numpy(v0[i])[None])
                          for i in range(L)))
    steps = []
    for s in range(c["steps"]):
        mgr.append_token(tuple((torch.from_numpy(kt[s, i])[None, :, None],
                                torch.from_numpy(vt[s, i])[None, :, None]) for i in range(L)))
        for layer in range(L):
            mgr.report_attention(layer, torch.from_numpy(attn[s][layer]))
        mgr.step_done()
        rec = {"schedule": mgr.schedule(), "stats": mgr.get_stats(),
               "evicted": sorted({st // bs for st, _ in mgr._evicted_ranges[0]})}
        if s % c["restore_every"] == c["restore_every"] - 1:
            mgr.build_past_kv()
            rec["after_restore"] = {"stats": mgr.get_stats()}
        steps.append(rec)
    mgr.destroy()
    fx = {"case": c, "steps": steps, "calls": core.calls, "score_queries": core.scores,
          "source": "the reference's python/orchkv/fast_kvcache_manager.py run unmodified on "
                    "the CPU (CUDA placements mapped to the CPU) with orchkv_core backed by "
                    "the reference scheduler compiled from src/scheduler (oracle/_ref); "
                    "scores and usage ratios as float32 bit patterns"}
    with open(os.path.join(HERE, "fast_manager_decode.json"), "w") as fh:
        json.dump(fx, fh, separators=(",", ":"))
    print("wrote fast_manager_decode.json:", len(steps), "steps,", len(core.calls), "calls")


if __name__ == "__main__":
    main()
