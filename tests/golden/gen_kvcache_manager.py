"""Generate tests/golden/kvcache_manager_decode.json by running the
reference's own python/orchkv/kvcache_manager.py (KVCacheManager) over a
seeded decode loop, on the CPU, with a stand-in orchkv_core that records
every call the manager makes (register, report, step, usage, schedule, tier)
and the manager's own results (schedule dicts, statistics, every block's
tier and access count) after each step.

Only needed to regenerate; the fixture is committed.  Needs the reference
source tree.  The manager module is loaded unmodified; its CUDA placements
are mapped to the CPU for this run (tensor `.to("cuda")`, `device="cuda"`,
`pin_memory`), which changes where bytes live, not any decision.

    python tests/golden/gen_kvcache_manager.py
"""
import importlib.util
import json
import os
import sys
import tempfile
import types

import numpy as np
import torch

try:
    from tests.golden.refpath import reference_file
except ImportError:          # run as a script from tests/golden
    from refpath import reference_file

HERE = os.path.dirname(os.path.abspath(__file__))
REFERENCE = "python/orchkv/kvcache_manager.py"      # inside the reference tree (tests/golden/refpath.py)

CASE = dict(n_layers=4, n_kv_heads=2, q_heads=4, head_dim=64, block_size=16, prefill=100,
            steps=30, budget_blocks=30, sink_tokens=4, build_every=5, seed=5)


def f32bits(x):
    return int(np.array([x], np.float32).view(np.uint32)[0])


def inputs(case):
    """Seeded K/V [layer][head][token][d] (fp16) and attention weights per
    (step, layer): softmax of N(0, 2) logits over the step's positions."""
    rng = np.random.default_rng(case["seed"])
    n = case["prefill"] + case["steps"]
    shape = (case["n_layers"], case["n_kv_heads"], n, case["head_dim"])
    k = rng.standard_normal(shape).astype(np.float16)
    v = rng.standard_normal(shape).astype(np.float16)
    attn = []
    for s in range(case["steps"]):
        t = case["prefill"] + s + 1
        per_layer = []
        for _ in range(case["n_layers"]):
            x = rng.normal(0, 2, (1, case["q_heads"], 1, t)).astype(np.float32)
            x = np.exp(x - x.max(-1, keepdims=True))
            per_layer.append((x / x.sum(-1, keepdims=True)).astype(np.float32))
        attn.append(per_layer)
    return k, v, attn


class Recorder(types.ModuleType):
    """orchkv_core stand-in: records the calls, answers like the binding."""
    GPU_HBM, HOST_DRAM, SSD = 0, 1, 3

    def __init__(self):
        super().__init__("orchkv_core")
        self.calls = []

    def tm_create(self, *a, **k):
        return 1

    def tm_destroy(self, tm):
        pass

    def tm_register_block_id(self, tm, bid, a=0, b=0):
        self.calls.append(["reg", int(bid), int(a), int(b)])
        return 0

    def tm_report_attn(self, tm, bid, score):
        self.calls.append(["rep", int(bid), f32bits(score)])

    def tm_step_done(self, tm):
        self.calls.append(["step"])

    def tm_set_usage(self, tm, g, d):
        self.calls.append(["usage", f32bits(g), f32bits(d)])

    def tm_schedule_once(self, tm):
        self.calls.append(["sched"])

    def tm_get_stats(self, tm):
        return {}

    def tm_set_block_tier(self, tm, bid, tier):
        self.calls.append(["tier", int(bid), int(tier)])


def load_reference(rec, path=None, name="ref_kvcache_manager"):
    """Load a reference manager module with `rec` as its orchkv_core and its
    CUDA placements mapped to the CPU."""
    sys.modules["orchkv_core"] = rec
    path = path or reference_file(REFERENCE)
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod              # its dataclasses look their module up
    spec.loader.exec_module(mod)
    mod.HAS_DYNAMIC_CACHE = False             # legacy tuples in and out

    class CpuTorch:                           # the module's `torch`, placements on the CPU
        def __getattr__(self, name):
            return getattr(torch, name)

        @staticmethod
        def zeros(*a, device=None, pin_memory=False, **k):
            return torch.zeros(*a, **k)

        @staticmethod
        def empty(*a, device=None, pin_memory=False, **k):
            return torch.empty(*a, **k)

        @staticmethod
        def empty_like(t, device=None, pin_memory=False, **k):
            return torch.empty_like(t, **k)

    mod.torch = CpuTorch()
    orig_to = torch.Tensor.to

    def to(self, *a, **k):
        a = tuple("cpu" if x == "cuda" else x for x in a)
        if k.get("device") == "cuda":
            k["device"] = "cpu"
        return orig_to(self, *a, **k)

    torch.Tensor.to = to
    torch.Tensor.pin_memory = lambda self, *a, **k: self
    return mod


def blocks_of(mgr):
    return [[b.block_id, b.token_start, b.token_count, b.tier, b.access_count, int(b.is_sink)]
            for lb in mgr._blocks for b in lb]


def main():
    c = CASE
    rec = Recorder()
    mod = load_reference(rec)
    k, v, attn = inputs(c)
    block_bytes = 2 * c["n_kv_heads"] * c["block_size"] * c["head_dim"] * 2
    with tempfile.TemporaryDirectory() as ssd:
        mgr = mod.KVCacheManager(c["n_layers"], c["n_kv_heads"], c["head_dim"],
                                 block_size=c["block_size"], dtype=torch.float16,
                                 gpu_budget_bytes=c["budget_blocks"] * block_bytes,
                                 ssd_dir=ssd, sink_tokens=c["sink_tokens"])

        def pkv(n):
            return tuple((torch.from_numpy(k[i][None, :, :n].copy()),
                          torch.from_numpy(v[i][None, :, :n].copy()))
                         for i in range(c["n_layers"]))

        mgr.ingest_step(pkv(c["prefill"]))
        steps = []
        for s in range(c["steps"]):
            n = c["prefill"] + s + 1
            mgr.append_token(pkv(n))
            for layer in range(c["n_layers"]):
                mgr.report_attention(layer, torch.from_numpy(attn[s][layer]))
            mgr.step_done()
            res = mgr.schedule()
            res.pop("tm_stats")
            st = mgr.get_stats()
            st.pop("tm")
            rec_step = {"schedule": res, "stats": st, "blocks": blocks_of(mgr)}
            if s % c["build_every"] == c["build_every"] - 1:
                mgr.build_past_kv()
                rec_step["after_build"] = {"stats": {kk: vv for kk, vv in mgr.get_stats().items()
                                                     if kk != "tm"},
                                           "blocks": blocks_of(mgr)}
            steps.append(rec_step)
        mgr.destroy()
    fx = {"case": c, "steps": steps, "calls": rec.calls,
          "source": "the reference's python/orchkv/kvcache_manager.py run unmodified on the "
                    "CPU (CUDA placements mapped to the CPU) with a recording orchkv_core; "
                    "scores and usage ratios as float32 bit patterns"}
    with open(os.path.join(HERE, "kvcache_manager_decode.json"), "w") as fh:
        json.dump(fx, fh, separators=(",", ":"))
    print("wrote kvcache_manager_decode.json:", len(steps), "steps,", len(rec.calls), "calls")


if __name__ == "__main__":
    main()
