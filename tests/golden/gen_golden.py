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
    "sched_slot_collisions": dict(
        # ids far beyond the tracker capacity: several ids share a slot
        # (slot = id & (capacity - 1), src/scheduler/attention_tracker.c:27-33)
        seed=5, cfg=dict(tracker_cap=64, max_blocks=8192),
        ops=dict(n_ids=200, id_space=2000, steps=20, reports=80, flags=(0, 0, 8),
                 dup_frac=0.1)),
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


def c4_case(seed=11, n=240, steps=16):
    """Demotion through the callback path: tm_schedule_once with a memcpy
    transfer callback, calloc/free allocators and 64-byte payloads (the
    set-up of test/test_tiered_manager.c), memory pressure varying per step."""
    rng = np.random.default_rng(seed)
    ids = [int(x) for x in rng.choice(4096, n, replace=False)]
    tiers = [int(t) for t in rng.choice([0, 0, 0, 1, 1, 2], n)]
    flags = [int(f) for f in rng.choice([0, 0, 0, 0, 1, 8], n)]
    touch = [int(t) for t in rng.integers(0, n, 3 * n)]
    rep_ids, rep_w, rep_off = [], [], [0]
    for _ in range(steps):
        for i in rng.choice(n, 60):
            rep_ids.append(ids[int(i)])
            rep_w.append(float(np.float32(rng.random())))
        rep_off.append(len(rep_ids))
    gpu = [float(np.float32(x)) for x in rng.uniform(0.6, 1.0, steps)]
    dram = [float(np.float32(x)) for x in rng.uniform(0.6, 1.0, steps)]
    return dict(ids=ids, tiers=tiers, flags=flags, touch=touch, steps=steps, rep_ids=rep_ids,
                rep_w=rep_w, rep_off=rep_off, gpu_ratio=gpu, dram_ratio=dram,
                demote_batch=8, alpha=0.5, beta=0.3, gamma=0.2)


def run_ref_c4(c):
    n = len(c["ids"])
    out_tier = np.zeros(n, np.int32)
    out_state = np.zeros(n, np.int32)
    out_byte = np.zeros(n, np.int32)
    o = np.zeros(16, np.float64)
    rc = O.ref().ref_c4_scenario(
        n, np.asarray(c["ids"], np.uint64), np.asarray(c["tiers"], np.int32),
        np.asarray(c["flags"], np.uint8), np.asarray(c["touch"], np.uint32), len(c["touch"]),
        c["steps"], np.asarray(c["rep_ids"], np.uint64), np.asarray(c["rep_w"], np.float32),
        np.asarray(c["rep_off"], np.uint32), np.asarray(c["gpu_ratio"], np.float32),
        np.asarray(c["dram_ratio"], np.float32), c["demote_batch"], c["alpha"], c["beta"],
        c["gamma"], out_tier, out_state, out_byte, o, c.get("fail_every", 0))
    assert rc == 0
    return dict(tier=out_tier.tolist(), state=out_state.tolist(), byte=out_byte.tolist(),
                stats=[int(x) for x in o])


def main():
    if not O.ref_available():
        raise SystemExit("build the reference first: make -C oracle")
    for name, c in (("c4_demote_callbacks", c4_case()),
                    ("c4_demote_callbacks_failing", dict(c4_case(seed=12), fail_every=3))):
        fx = {"name": name, "case": c, "expect": run_ref_c4(c),
              "stats_order": "gpu_demotes dram_demotes blocks_migrated op_errors op_count[6] "
                             "op_bytes[6]/64",
              "source": "reference src/scheduler/*.c compiled by oracle/Makefile, driven like "
                        "test/test_tiered_manager.c (transfer/alloc/free callbacks; with "
                        "fail_every, every n-th transfer fails with ORCHKV_ERR_IO as "
                        "test/test_migration_engine.c's failing mock)"}
        with open(os.path.join(HERE, name + ".json"), "w") as fh:
            json.dump(fx, fh, separators=(",", ":"))
        print("wrote", name, fx["expect"]["stats"])
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
