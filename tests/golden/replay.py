"""Replay a recorded scheduler op sequence (tests/golden/*.json) through the
oracle restatement or through the GPU library's tm_* C ABI, and return the
same observables the fixture recorded from the reference.

Op encoding (one list per op):
    ["reg", id, tier, flags]      tm_register_block_id
    ["rep", id, weight]           tm_report_attn
    ["step"]                      tm_step_done
    ["usage", gpu, dram]          tm_set_usage
    ["sched"]                     tm_schedule_once
    ["tier", id, tier]            tm_set_block_tier
    ["policy", a, b, g]           tm_set_policy
Floats in "expect" are stored as uint32 bit patterns so comparisons are exact.
"""
import numpy as np

STATS = ["schedule_cycles", "prefetches_dispatched", "n_hot", "n_warm", "n_cold",
         "threshold_adj_up", "threshold_adj_down", "total_scanned", "total_enqueued",
         "total_dispatched", "prefetch_wasted", "demote_checks"]
STATS_F32 = ["threshold_hot", "threshold_warm"]


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32).astype(np.int64).tolist()


def observe(state, stats, ids, cap):
    slots = [int(i) % cap for i in ids]
    out = {
        "ema": bits(state["ema"][slots]),
        "hot": bits(state["hot"][slots]),
        "hits": state["hits"][slots].astype(np.int64).tolist(),
        "last": [int(x) for x in state["last"][slots]],
        "heat": state["heat"][slots].astype(np.int64).tolist(),
    }
    for k in STATS:
        if k in stats:
            out["stat_" + k] = int(stats[k])
    for k in STATS_F32:
        if k in stats:
            out["stat_" + k] = bits([stats[k]])[0]
    return out


def _run(tm, ops):
    for op in ops:
        kind = op[0]
        if kind == "reg":
            tm.register(op[1], op[2], op[3]) if hasattr(tm, "register") else tm.register_id(op[1], op[2], op[3])
        elif kind == "rep":
            tm.report(op[1], op[2])
        elif kind == "step":
            tm.step_done()
        elif kind == "usage":
            tm.set_usage(op[1], op[2])
        elif kind == "sched":
            tm.schedule_once()
        elif kind == "tier":
            tm.set_block_tier(op[1], op[2])
        elif kind == "policy":
            (tm.set_policy if hasattr(tm, "set_policy") else tm.s.set_weights)(op[1], op[2], op[3])
        else:
            raise ValueError(kind)


def replay_oracle(O, fx):
    cfg = dict(fx["config"])
    cfg.pop("cooldown_sec", None)
    tm = O.OracleTM(**cfg)
    _run(tm, fx["ops"])
    return observe(tm.s.state(), tm.stats(), fx["ids"], tm.s.cap)


def replay_gpu(orchkv_b200, fx):
    cfg = dict(fx["config"])
    m = orchkv_b200.Manager(cooldown_sec=0.0, **{k: v for k, v in cfg.items()
                                                 if k != "cooldown_sec"})
    try:
        class _Adapter:
            register = staticmethod(m.register_id)
            report = staticmethod(m.report)
            step_done = staticmethod(m.step_done)
            set_usage = staticmethod(m.set_usage)
            schedule_once = staticmethod(m.schedule_once)
            set_block_tier = staticmethod(m.set_block_tier)

            @staticmethod
            def set_policy(a, b, g):
                orchkv_b200.lib().tm_set_policy(m.ref, a, b, g)
        _run(_Adapter, fx["ops"])
        st = m.stats()
        st["demote_checks"] = None
        st = {k: v for k, v in st.items() if v is not None}
        return observe(m.state(), st, fx["ids"], m.cap)
    finally:
        m.close()
