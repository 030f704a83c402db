"""Generate tests/golden/vllm_connector_scheduler.json by driving the
reference's own python/orchkv/vllm_integration/connector.py
(OrchKvOffloadingConnector in the scheduler role, connector.py:227-289,
390-421) through a seeded sequence of scheduler calls: prefix-match queries,
finished requests (with repeated block ids), preemptions of known and unknown
requests, allocation notices and metadata builds.  Records every return
value, and each metadata object's blocks to save and load in their order.
Two configurations: layers from the connector's extra config, and from the
model config (which takes precedence).  Preempted request ids are passed in
sorted order, so the pending lists' order does not depend on the process's
string-hash salt.

Only needed to regenerate; the fixture is committed.  Needs the reference
source tree; the scheduler role touches no GPU and no orchkv_core.

    python tests/golden/gen_vllm_connector.py
"""
import importlib.util
import json
import os
import random
import sys
from types import SimpleNamespace

try:
    from tests.golden.refpath import reference_file
except ImportError:          # run as a script from tests/golden
    from refpath import reference_file

HERE = os.path.dirname(os.path.abspath(__file__))
REFERENCE = "python/orchkv/vllm_integration/connector.py"      # inside the reference tree (tests/golden/refpath.py)
CONFIGS = [
    {"extra": {"dram_pool_gb": 1, "n_layers": 3}, "model": {"head_dim": 64}},
    {"extra": {"dram_pool_gb": 1, "n_layers": 5}, "model": {"head_dim": 128, "num_layers": 2}},
]


def vllm_config(case):
    return SimpleNamespace(
        kv_transfer_config=SimpleNamespace(kv_connector_extra_config=dict(case["extra"])),
        model_config=SimpleNamespace(**case["model"]))


def script(seed=21, n_ops=120, n_req=8):
    """The call sequence: [op, request id, argument]."""
    rng = random.Random(seed)
    ops = []
    for _ in range(n_ops):
        op = rng.choice(["match", "match", "finish", "preempt", "alloc", "meta"])
        req = f"r{rng.randrange(n_req)}"
        if op == "match":
            ops.append([op, req, rng.randrange(0, 12)])
        elif op == "finish":
            ops.append([op, req, [rng.randrange(0, 40) for _ in range(rng.randrange(0, 10))]])
        elif op == "preempt":
            ops.append([op, None, sorted({f"r{rng.randrange(n_req + 2)}"
                                          for _ in range(rng.randrange(1, 4))})])
        elif op == "alloc":
            ops.append([op, req, rng.randrange(0, 5)])
        else:
            ops.append([op, None, None])
    return ops


def run(connector_cls, role, case, ops):
    """Replay ops on a scheduler-role connector; returns the results."""
    c = connector_cls(vllm_config(case), role)
    out = []
    for op, req, arg in ops:
        r = SimpleNamespace(request_id=req)
        if op == "match":
            a, b = c.get_num_new_matched_tokens(r, arg)
            out.append([a, b])
        elif op == "finish":
            a, b = c.request_finished(r, list(arg))
            out.append([a, b])
        elif op == "preempt":
            # in sorted order: a set of strings iterates in an order that
            # changes from process to process (string hashing is salted),
            # and both connectors extend the pending lists in iteration order
            out.append(c.handle_preemptions(list(arg)))
        elif op == "alloc":
            out.append(c.update_state_after_alloc(r, None, arg))
        else:
            m = c.build_connector_meta(None)
            out.append({"save": {k: list(v) for k, v in m.blocks_to_save.items()},
                        "load": {k: list(v) for k, v in m.blocks_to_load.items()}})
    return out


def main():
    spec = importlib.util.spec_from_file_location("ref_orchkv_connector", reference_file(REFERENCE))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    ops = script()
    cases = [{"config": case, "results": run(mod.OrchKvOffloadingConnector,
                                             mod.KVConnectorRole.SCHEDULER, case, ops)}
             for case in CONFIGS]
    with open(os.path.join(HERE, "vllm_connector_scheduler.json"), "w") as fh:
        json.dump({"ops": ops, "cases": cases}, fh)


if __name__ == "__main__":
    main()
