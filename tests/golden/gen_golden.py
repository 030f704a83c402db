"""Generate tests/golden/*.json from the reference compiled from its own
sources (oracle/_ref/liborchkv_ref.so, built by `make -C oracle`).

Each fixture is a seeded op sequence driven through the reference's tiered
manager exactly as its Python binding does (tm_create defaults, binding-owned
blocks registered by id), plus the observables recorded afterwards.  The
reference source tree is only needed to regenerate; the fixtures themselves
are committed.

    python tests/golden/gen_golden.py
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from tests.golden.replay import observe  # noqa: E402


def ref_stats(r):
    s = r.stats()
    return s


def make_ops(rng, n_ids, id_space, steps, reports, tiers=(0,), flags=(0,), usage=None,
             sched_every=1, dup_frac=0.0, tier_changes=0, policy_at=None):
    ids = [int(x) for x in rng.choice(id_space, n_ids, replace=False)]
    ops = []
    for i in ids:
        ops.append(["reg", i, int(rng.choice(tiers)), int(rng.choice(flags))])
    for i in ids[: int(dup_frac * n_ids)]:
        ops.append(["reg", i, 1, 0])             # re-registration: reset + duplicate entry
    for s in range(steps):
        for r in rng.choice(ids, reports):
            ops.append(["rep", int(r), float(np.float32(rng.random()))])
        ops.append(["step"])
        if usage is None:
            g, d = float(np.float32(rng.random())), float(np.float32(rng.random()))
        else:
            g, d = usage
        ops.append(["usage", g, d])
        if s % sched_every == 0:
            ops.append(["sched"])
        for _ in range(tier_changes):
            ops.append(["tier", int(rng.choice(ids)), int(rng.choice([0, 1, 2]))])
        if policy_at is not None and s == policy_at:
            ops.append(["policy", 0.6, 0.25, 0.15])
    return ids, ops


def run_ref(cfg, ops):
    r = O.RefTM(cooldown_sec=0.0, **cfg)
    for op in ops:
        k = op[0]
        if k == "reg":
            r.register(op[1], op[2], op[3])
        elif k == "rep":
            r.report(op[1], op[2])
        elif k == "step":
            r.step_done()
        elif k == "usage":
            r.set_usage(op[1], op[2])
        elif k == "sched":
            r.schedule_once()
        elif k == "tier":
            r.set_block_tier(op[1], op[2])
        elif k == "policy":
            r.set_policy(op[1], op[2], op[3])
    return r


CASES = {
    "sched_default": dict(
        seed=1, cfg=dict(tracker_cap=256, max_blocks=8192),
        ops=dict(n_ids=150, id_space=256, steps=30, reports=40)),
    "sched_custom_weights": dict(
        seed=2, cfg=dict(tracker_cap=512, max_blocks=8192, ema_lambda=0.8, alpha=0.6,
                         beta=0.25, gamma=0.15, recency_tau=7.0),
        ops=dict(n_ids=200, id_space=512, steps=40, reports=60, flags=(0, 0, 8, 1),
                 policy_at=20)),
    "sched_prefetch_counters": dict(
        seed=3, cfg=dict(tracker_cap=256, max_blocks=300, threshold_to_gpu=0.3,
                         threshold_to_dram=0.1, prefetch_budget=5),
        ops=dict(n_ids=180, id_space=256, steps=25, reports=70, tiers=(0, 0, 1, 2, 4),
                 flags=(0, 8), dup_frac=0.3, tier_changes=3)),
    "sched_fast_manager_pattern": dict(
        # FastKVCacheManager: ids = block index, sinks registered with tier 1
        # (positional quirk, python/orchkv/fast_kvcache_manager.py:155), every
        # layer reports into the same id (:227-235)
        seed=4, cfg=dict(),
        ops=None),
}


def fast_manager_ops(rng):
    n_blocks, layers = 40, 6
    ops = [["reg", b, 1 if b == 0 else 0, 0] for b in range(n_blocks)]
    for s in range(20):
        for layer in range(layers):
            for b in range(n_blocks):
                ops.append(["rep", b, float(np.float32(rng.random() * 0.05))])
        ops.append(["step"])
        ops.append(["usage", float(np.float32(1.0 - 0.01 * s)), 0.0])
        ops.append(["sched"])
    return list(range(n_blocks)), ops


def main():
    if not O.ref_available():
        raise SystemExit("build the reference first: make -C oracle")
    for name, case in CASES.items():
        rng = np.random.default_rng(case["seed"])
        if case["ops"] is None:
            ids, ops = fast_manager_ops(rng)
        else:
            ids, ops = make_ops(rng, **case["ops"])
        r = run_ref(case["cfg"], ops)
        exp = observe(r.state(), ref_stats(r), ids, r.cap)
        exp.pop("stat_demote_checks", None)
        fx = {"name": name, "config": case["cfg"], "ids": ids, "ops": ops, "expect": exp,
              "source": "reference src/scheduler/*.c compiled by oracle/Makefile, driven "
                        "like bindings/orchkv_pybind.cpp"}
        with open(os.path.join(HERE, name + ".json"), "w") as fh:
            json.dump(fx, fh, separators=(",", ":"))
        r.close()
        print("wrote", name, len(ops), "ops")


if __name__ == "__main__":
    main()
