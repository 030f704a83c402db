"""orchkv_core as a drop-in under the reference's own Python managers.

The reference's FastKVCacheManager and KVCacheManager
(python/orchkv/fast_kvcache_manager.py:106-341,
python/orchkv/kvcache_manager.py:117-427) reach the scheduler only through
orchkv_core: tm_create, tm_register_block_id, tm_report_attn, tm_step_done,
tm_set_usage, tm_schedule_once, tm_set_block_tier, tm_get_stats and, for
the fast manager's eviction order, tm_get_block_score.  Given the same
inputs, a manager's calls and decisions are a function of what those calls
return.  So if this module returns what the reference returned at every
point of the call stream the unmodified manager produced against the
reference, the unmodified manager makes the same calls and decisions on this
module, step by step.

* Stream form (always): the committed fixtures hold the call streams that
  the reference managers made, unmodified, against the reference scheduler
  compiled from its sources (tests/golden/gen_fast_manager.py,
  gen_kvcache_manager.py), and every tm_get_block_score answer the fast
  manager got.  They are replayed through this module, created with the
  binding's defaults exactly as the managers create it: every answer the
  manager asked for is bit-identical, and after the KVCacheManager's stream
  every block's score equals the compiled reference scheduler's on the same
  stream (oracle/_ref).
* Literal form (where the reference tree is at hand): with
  ORCHKV_REFERENCE_PY naming the reference's `python` directory, its two
  manager modules are loaded unmodified with this module as orchkv_core and
  run on the GPU on the fixtures' seeded decode loops; their call streams,
  score answers, schedule results, statistics, evictions and block tiers
  must equal the fixtures.  The module's own HAS_DYNAMIC_CACHE switch is set
  to False, its legacy-tuple branch, as in the fixture runs (the installed
  transformers' DynamicCache lacks the constructor the module's other branch
  calls); no code of the module changes.  Skipped where the variable is
  unset: the reference tree is not shipped to machines that only run tests.
"""
import importlib.util
import json
import os
import sys
import tempfile
import types

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")


def f32bits(x):
    return int(np.array([x], np.float32).view(np.uint32)[0])


def _fixture(name):
    with open(os.path.join(GOLDEN, name)) as fh:
        return json.load(fh)


@pytest.fixture(scope="module")
def core(cuda):
    import orchkv_b200
    return orchkv_b200.core()


def _replay(core, tm, op):
    k = op[0]
    if k == "reg":
        core.tm_register_block_id(tm, op[1], op[2], op[3])
    elif k == "rep":
        core.tm_report_attn(tm, op[1], np.array([op[2]], np.uint32).view(np.float32)[0].item())
    elif k == "step":
        core.tm_step_done(tm)
    elif k == "usage":
        g = np.array([op[1]], np.uint32).view(np.float32)[0].item()
        d = np.array([op[2]], np.uint32).view(np.float32)[0].item()
        core.tm_set_usage(tm, g, d)
    elif k == "sched":
        core.tm_schedule_once(tm)
    elif k == "tier":
        core.tm_set_block_tier(tm, op[1], op[2])
    else:
        raise AssertionError(f"unknown op {op}")


def test_fast_manager_stream_answers(core):
    """Every tm_get_block_score the unmodified FastKVCacheManager asked the
    reference scheduler, at its place in the manager's call stream, gets the
    same float bits from this module."""
    fx = _fixture("fast_manager_decode.json")
    queries = fx["score_queries"]
    assert len(queries) > 0
    tm = core.tm_create()                       # as the manager creates it
    try:
        qi = 0
        for pos, op in enumerate(fx["calls"] + [None]):
            while qi < len(queries) and queries[qi][0] == pos:
                _, bid, bits = queries[qi]
                assert f32bits(core.tm_get_block_score(tm, bid)) == bits, (pos, bid)
                qi += 1
            if op is not None:
                _replay(core, tm, op)
        assert qi == len(queries)
    finally:
        core.tm_destroy(tm)


def test_kvcache_manager_stream_state(core, oracle_mod):
    """The unmodified KVCacheManager's call stream leaves every block's score
    bit-identical to the compiled reference scheduler's on the same stream,
    checked after every step."""
    O = oracle_mod
    if not O.ref_available():
        pytest.skip("oracle/_ref (the reference compiled from its sources) is not built")
    fx = _fixture("kvcache_manager_decode.json")
    tm = core.tm_create()
    ref = O.RefTM()                             # the binding's defaults
    ids = set()
    try:
        checks = 0
        for op in fx["calls"]:
            _replay(core, tm, op)
            k = op[0]
            if k == "reg":
                ids.add(op[1])
                ref.register(op[1], op[2], op[3])
            elif k == "rep":
                ref.report(op[1], np.array([op[2]], np.uint32).view(np.float32)[0].item())
            elif k == "step":
                ref.step_done()
            elif k == "usage":
                ref.set_usage(*(np.array([op[1], op[2]], np.uint32).view(np.float32).tolist()))
            elif k == "sched":
                ref.schedule_once()
            elif k == "tier":
                ref.set_block_tier(op[1], op[2])
            if k == "step":
                for b in sorted(ids):
                    assert f32bits(core.tm_get_block_score(tm, b)) == f32bits(ref.score(b)), b
                checks += 1
        assert checks == fx["case"]["steps"]
        assert core.tm_get_stats(tm)["schedule_cycles"] == ref.stats()["schedule_cycles"]
    finally:
        core.tm_destroy(tm)
        ref.close()


# ---------------------------------------------------------------------------
# literal form: the reference's manager modules, unmodified, on this module
# ---------------------------------------------------------------------------

def _reference_py():
    d = os.environ.get("ORCHKV_REFERENCE_PY")
    if not d or not os.path.isfile(os.path.join(d, "orchkv", "fast_kvcache_manager.py")):
        pytest.skip("set ORCHKV_REFERENCE_PY to the reference's python directory")
    return d


class RecordingCore(types.ModuleType):
    """orchkv_core for the managers: this repository's module, with the
    manager's calls and score answers recorded as the fixtures hold them."""

    def __init__(self, real):
        super().__init__("orchkv_core")
        self._real = real
        self.calls, self.scores = [], []

    def __getattr__(self, name):
        return getattr(self._real, name)

    def tm_register_block_id(self, h, bid, a=0, b=0):
        self.calls.append(["reg", int(bid), int(a), int(b)])
        return self._real.tm_register_block_id(h, bid, a, b)

    def tm_report_attn(self, h, bid, score):
        self.calls.append(["rep", int(bid), f32bits(score)])
        return self._real.tm_report_attn(h, bid, score)

    def tm_step_done(self, h):
        self.calls.append(["step"])
        return self._real.tm_step_done(h)

    def tm_set_usage(self, h, g, d):
        self.calls.append(["usage", f32bits(g), f32bits(d)])
        return self._real.tm_set_usage(h, g, d)

    def tm_schedule_once(self, h):
        self.calls.append(["sched"])
        return self._real.tm_schedule_once(h)

    def tm_set_block_tier(self, h, bid, tier):
        self.calls.append(["tier", int(bid), int(tier)])
        return self._real.tm_set_block_tier(h, bid, tier)

    def tm_get_block_score(self, h, bid):
        s = self._real.tm_get_block_score(h, bid)
        self.scores.append([len(self.calls), int(bid), f32bits(s)])
        return s


def _load_manager(rec, path, name):
    sys.modules["orchkv_core"] = rec
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    try:
        spec.loader.exec_module(mod)
    finally:
        del sys.modules["orchkv_core"]
    mod.HAS_DYNAMIC_CACHE = False
    return mod


def test_reference_fast_manager_on_this_module(core, cuda):
    import torch

    from tests.golden.gen_fast_manager import inputs
    d = _reference_py()
    fx = _fixture("fast_manager_decode.json")
    c = fx["case"]
    rec = RecordingCore(core)
    mod = _load_manager(rec, os.path.join(d, "orchkv", "fast_kvcache_manager.py"),
                        "ref_fast_kvcache_manager_on_b200")
    k0, v0, kt, vt, attn = inputs(c)
    L, H, dh, bs = c["n_layers"], c["n_kv_heads"], c["head_dim"], c["block_size"]
    block_bytes = 2 * H * bs * dh * 2
    mgr = mod.FastKVCacheManager(L, H, dh, block_size=bs, dtype=torch.float16,
                                 gpu_budget_bytes=c["budget_blocks_per_layer"] * L * block_bytes,
                                 max_seq_len=c["max_seq_len"], sink_tokens=c["sink_tokens"])
    try:
        mgr.ingest_step(tuple((torch.from_numpy(k0[i])[None].cuda(),
                               torch.from_numpy(v0[i])[None].cuda()) for i in range(L)))
        for s in range(c["steps"]):
            mgr.append_token(tuple((torch.from_numpy(kt[s, i])[None, :, None].cuda(),
                                    torch.from_numpy(vt[s, i])[None, :, None].cuda())
                                   for i in range(L)))
            for layer in range(L):
                mgr.report_attention(layer, torch.from_numpy(attn[s][layer]).cuda())
            mgr.step_done()
            want = fx["steps"][s]
            assert mgr.schedule() == want["schedule"], s
            assert mgr.get_stats() == want["stats"], s
            assert sorted({st // bs for st, _ in mgr._evicted_ranges[0]}) == want["evicted"], s
            if "after_restore" in want:
                mgr.build_past_kv()
                assert mgr.get_stats() == want["after_restore"]["stats"], s
    finally:
        mgr.destroy()
    assert rec.calls == fx["calls"]
    assert rec.scores == fx["score_queries"]


def test_reference_kvcache_manager_on_this_module(core, cuda):
    import torch

    from tests.golden.gen_kvcache_manager import blocks_of, inputs
    d = _reference_py()
    fx = _fixture("kvcache_manager_decode.json")
    c = fx["case"]
    rec = RecordingCore(core)
    mod = _load_manager(rec, os.path.join(d, "orchkv", "kvcache_manager.py"),
                        "ref_kvcache_manager_on_b200")
    k, v, attn = inputs(c)
    block_bytes = 2 * c["n_kv_heads"] * c["block_size"] * c["head_dim"] * 2
    with tempfile.TemporaryDirectory() as ssd:
        mgr = mod.KVCacheManager(c["n_layers"], c["n_kv_heads"], c["head_dim"],
                                 block_size=c["block_size"], dtype=torch.float16,
                                 gpu_budget_bytes=c["budget_blocks"] * block_bytes,
                                 ssd_dir=ssd, sink_tokens=c["sink_tokens"])

        def pkv(n):
            return tuple((torch.from_numpy(k[i][None, :, :n].copy()).cuda(),
                          torch.from_numpy(v[i][None, :, :n].copy()).cuda())
                         for i in range(c["n_layers"]))
        try:
            mgr.ingest_step(pkv(c["prefill"]))
            for s in range(c["steps"]):
                mgr.append_token(pkv(c["prefill"] + s + 1))
                for layer in range(c["n_layers"]):
                    mgr.report_attention(layer, torch.from_numpy(attn[s][layer]).cuda())
                mgr.step_done()
                want = fx["steps"][s]
                res = mgr.schedule()
                res.pop("tm_stats")
                st = mgr.get_stats()
                st.pop("tm")
                assert res == want["schedule"], s
                assert st == want["stats"], s
                assert blocks_of(mgr) == want["blocks"], s
                if "after_build" in want:
                    mgr.build_past_kv()
                    assert blocks_of(mgr) == want["after_build"]["blocks"], s
        finally:
            mgr.destroy()
    assert rec.calls == fx["calls"]
