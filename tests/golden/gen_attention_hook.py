"""Generate tests/golden/attention_hook_reports.json by running the
reference's own python/orchkv/vllm_integration/attention_hook.py
(AttentionScoreCollector) on the CPU with a recording orchkv_core: seeded
fp32 attention weights for several layers and steps, in each block-id mode
(default ids, a block_id_fn, a block table narrower than the blocks, a
mapping that repeats ids), and a sampling interval that skips steps.  Records
every tm_report_attn / tm_step_done call and the collector's statistics.

Only needed to regenerate; the fixture is committed.  Needs the reference
source tree.  The module is loaded unmodified; its side stream and pinned
buffers become plain CPU ones for this run.

    python tests/golden/gen_attention_hook.py
"""
import contextlib
import importlib.util
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

from tests.golden.gen_kvcache_manager import f32bits  # noqa: E402

REFERENCE = "python/orchkv/vllm_integration/attention_hook.py"      # inside the reference tree (tests/golden/refpath.py)
CASE = dict(seed=9, steps=5, sample_interval=2, block_size=16, batch=2, heads=4, q_len=1,
            kv_len=100, table=[500, 507, 514, 521, 528])
MODES = ["default", "fn", "table", "repeat"]


def weights(case):
    """Per (step, mode/layer): softmax of N(0, 2) logits, fp32 [b, h, q, kv]."""
    rng = np.random.default_rng(case["seed"])
    out = []
    for _ in range(case["steps"]):
        per = []
        for _ in MODES:
            x = rng.normal(0, 2, (case["batch"], case["heads"], case["q_len"],
                                  case["kv_len"])).astype(np.float32)
            x = np.exp(x - x.max(-1, keepdims=True))
            per.append((x / x.sum(-1, keepdims=True)).astype(np.float32))
        out.append(per)
    return out


def id_fn(mode):
    if mode == "fn":
        return lambda layer, h, bi: 1000 + 31 * h + bi
    if mode == "repeat":
        return lambda layer, h, bi: None if bi == 2 else 2500 + (bi % 3) + 4 * h
    return None


class Recorder(types.ModuleType):
    def __init__(self):
        super().__init__("orchkv_core")
        self.calls = []

    def tm_report_attn(self, tm, bid, score):
        self.calls.append(["rep", int(bid), f32bits(score)])

    def tm_step_done(self, tm):
        self.calls.append(["step"])


def load_reference(rec):
    sys.modules["orchkv_core"] = rec
    spec = importlib.util.spec_from_file_location("ref_attention_hook", reference_file(REFERENCE))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)

    class Stream:
        def synchronize(self):
            pass

    class CpuTorch:
        def __getattr__(self, name):
            return getattr(torch, name)

        @staticmethod
        def empty(*a, device=None, pin_memory=False, **k):
            return torch.empty(*a, **k)

        cuda = types.SimpleNamespace(Stream=Stream,
                                     stream=lambda s: contextlib.nullcontext())

    mod.torch = CpuTorch()
    return mod


def main():
    c = CASE
    rec = Recorder()
    mod = load_reference(rec)
    col = mod.AttentionScoreCollector(1, block_size=c["block_size"],
                                      sample_interval=c["sample_interval"])
    ws = weights(c)
    table = torch.tensor([c["table"]], dtype=torch.int64)
    for s in range(c["steps"]):
        for layer, mode in enumerate(MODES):
            col.collect(layer, torch.from_numpy(ws[s][layer]),
                        block_table=table if mode == "table" else None,
                        block_id_fn=id_fn(mode))
        col.on_step_done()
    fx = {"case": c, "modes": MODES, "calls": rec.calls, "stats": col.get_stats(),
          "source": "the reference's python/orchkv/vllm_integration/attention_hook.py run "
                    "unmodified on the CPU with a recording orchkv_core; scores as float32 "
                    "bit patterns"}
    with open(os.path.join(HERE, "attention_hook_reports.json"), "w") as fh:
        json.dump(fx, fh, separators=(",", ":"))
    print("wrote attention_hook_reports.json:", len(rec.calls), "calls", col.get_stats())


if __name__ == "__main__":
    main()
