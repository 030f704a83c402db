"""ctypes front end of the test oracle.

TEST INFRASTRUCTURE ONLY.  ``OracleSched`` drives the CPU restatement in
``liborchkv_oracle.so`` (built from orchkv_oracle.c); ``RefTM`` and
``RefDramPool`` drive the reference's own C code compiled from its sources
into ``_ref/liborchkv_ref.so`` (present only where the reference tree was
available at build time).  Only tests/, ``__graft_entry__.smoke`` and the CPU
legs of bench.py import this module; the product never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liborchkv_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "liborchkv_ref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")

STEP_NEVER = np.uint64(0xFFFFFFFFFFFFFFFF)


def build(reference: str | None = None) -> None:
    """Compile the oracle (and the reference, if its tree is present)."""
    env = dict(os.environ)
    args = ["make", "-s", "-C", HERE, "-j8"]
    if reference:
        args.append(f"REF={reference}")
    subprocess.run(args, check=True, env=env)


def _load(path):
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is missing; run `make -C oracle`")
    return C.CDLL(path)


class _SchedStruct(C.Structure):
    _fields_ = [
        ("cap", C.c_uint32), ("mask", C.c_uint32), ("step", C.c_uint64),
        ("lam", C.c_float),
        ("sum", C.POINTER(C.c_float)), ("max", C.POINTER(C.c_float)),
        ("ema", C.POINTER(C.c_float)), ("hits", C.POINTER(C.c_uint32)),
        ("last", C.POINTER(C.c_uint64)), ("t_active", C.POINTER(C.c_uint8)),
        ("hot", C.POINTER(C.c_float)), ("heat", C.POINTER(C.c_uint8)),
        ("c_flags", C.POINTER(C.c_uint8)), ("c_active", C.POINTER(C.c_uint8)),
        ("alpha", C.c_float), ("beta", C.c_float), ("gamma", C.c_float),
        ("tau", C.c_float), ("th_hot", C.c_float), ("th_warm", C.c_float),
        ("table", C.c_float * 512),
    ]


class _Athresh(C.Structure):
    _fields_ = [(n, C.c_float) for n in (
        "th_hot", "th_warm", "min_hot", "max_hot", "min_warm", "max_warm",
        "gpu_hwm", "gpu_lwm", "dram_hwm", "dram_lwm", "step")] + [
        ("up", C.c_uint64), ("down", C.c_uint64), ("checks", C.c_uint64)]


_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        L = _load(ORACLE_SO)
        S = C.POINTER(_SchedStruct)
        L.oc_sched_init.argtypes = [S, C.c_uint32, C.c_float, C.c_float, C.c_float,
                                    C.c_float, C.c_float, C.c_float, C.c_float]
        L.oc_sched_free.argtypes = [S]
        L.oc_register.argtypes = [S, C.c_uint64, C.c_uint8]
        L.oc_unregister.argtypes = [S, C.c_uint64]
        L.oc_update.argtypes = [S, C.c_uint64, C.c_float]
        L.oc_update_batch.argtypes = [S, _u64p, _f32p, C.c_uint32]
        L.oc_step_done.argtypes = [S]
        L.oc_update_all.argtypes = [S]
        L.oc_set_thresholds.argtypes = [S, C.c_float, C.c_float]
        L.oc_set_weights.argtypes = [S, C.c_float, C.c_float, C.c_float]
        L.oc_build_decay_table.argtypes = [_f32p, C.c_float]
        L.oc_athresh_update.argtypes = [C.POINTER(_Athresh), C.c_float, C.c_float]
        L.oc_athresh_update.restype = C.c_int
        L.oc_orderable.argtypes = [C.c_float]
        L.oc_orderable.restype = C.c_uint32
        L.oc_select_coldest.argtypes = [_f32p, _u8p, C.c_uint32, C.c_uint32, _u32p]
        L.oc_select_coldest.restype = C.c_uint32
        L.oc_select_prefetch.argtypes = [_f32p, _u8p, _u8p, C.c_uint32, C.c_float,
                                         C.c_float, C.c_uint32, _u32p]
        L.oc_select_prefetch.restype = C.c_uint32
        L.oc_score_blocks.argtypes = [_f32p, C.c_uint32, C.c_uint32, C.c_uint32,
                                      C.c_uint32, C.c_uint32, C.c_void_p, _f32p]
        _LIB = L
    return _LIB


class OracleSched:
    """Tracker + classifier restatement, slot arrays exposed as numpy views."""

    def __init__(self, capacity=4096, ema_lambda=0.9, alpha=0.5, beta=0.3,
                 gamma=0.2, recency_tau=50.0, th_hot=0.5, th_warm=0.2):
        self._s = _SchedStruct()
        rc = lib().oc_sched_init(C.byref(self._s), capacity, ema_lambda, alpha,
                                 beta, gamma, recency_tau, th_hot, th_warm)
        if rc != 0:
            raise RuntimeError(f"oc_sched_init failed: {rc}")
        self.cap = self._s.cap

    def __del__(self):
        if getattr(self, "_s", None) is not None and _LIB is not None:
            _LIB.oc_sched_free(C.byref(self._s))
            self._s = None

    def _arr(self, name, dtype):
        ptr = getattr(self._s, name)
        return np.ctypeslib.as_array(ptr, shape=(self.cap,)).view(dtype)

    @property
    def step(self):
        return self._s.step

    def register(self, bid, flags=0):
        lib().oc_register(C.byref(self._s), bid, flags)

    def unregister(self, bid):
        lib().oc_unregister(C.byref(self._s), bid)

    def update(self, bid, w):
        lib().oc_update(C.byref(self._s), bid, w)

    def update_batch(self, ids, w):
        ids = np.ascontiguousarray(ids, np.uint64)
        w = np.ascontiguousarray(w, np.float32)
        lib().oc_update_batch(C.byref(self._s), ids, w, len(ids))

    def step_done(self):
        lib().oc_step_done(C.byref(self._s))

    def update_all(self):
        lib().oc_update_all(C.byref(self._s))

    def set_thresholds(self, h, w):
        lib().oc_set_thresholds(C.byref(self._s), h, w)

    def set_weights(self, a, b, g):
        lib().oc_set_weights(C.byref(self._s), a, b, g)

    def state(self):
        """Copies of every per-slot array."""
        return {
            "sum": self._arr("sum", np.float32).copy(),
            "max": self._arr("max", np.float32).copy(),
            "ema": self._arr("ema", np.float32).copy(),
            "hits": self._arr("hits", np.uint32).copy(),
            "last": self._arr("last", np.uint64).copy(),
            "t_active": self._arr("t_active", np.uint8).copy(),
            "hot": self._arr("hot", np.float32).copy(),
            "heat": self._arr("heat", np.uint8).copy(),
            "c_active": self._arr("c_active", np.uint8).copy(),
            "c_flags": self._arr("c_flags", np.uint8).copy(),
        }

    def table(self):
        return np.array(self._s.table[:], dtype=np.float32)


def decay_table(tau):
    t = np.zeros(512, np.float32)
    lib().oc_build_decay_table(t, tau)
    return t


def orderable(x: np.ndarray) -> np.ndarray:
    """Vectorised oc_orderable (same mapping as the C function)."""
    x = np.asarray(x, np.float32).copy()
    x[x == 0.0] = 0.0
    u = x.view(np.uint32)
    out = np.where(u & 0x80000000, ~u, u | 0x80000000).astype(np.uint32)
    out[np.isnan(x)] = 0xFFFFFFFE
    return out


def select_coldest(hot, eligible, k):
    hot = np.ascontiguousarray(hot, np.float32)
    el = np.ascontiguousarray(eligible, np.uint8)
    out = np.zeros(max(len(hot), 1), np.uint32)
    c = lib().oc_select_coldest(hot, el, len(hot), k, out)
    return out[:c].copy()


def select_prefetch(ema, active, tier, th_gpu, th_dram, k):
    ema = np.ascontiguousarray(ema, np.float32)
    out = np.zeros(max(len(ema), 1), np.uint32)
    c = lib().oc_select_prefetch(ema, np.ascontiguousarray(active, np.uint8),
                                 np.ascontiguousarray(tier, np.uint8), len(ema),
                                 th_gpu, th_dram, k, out)
    return out[:c].copy()


def score_blocks(probs, Hq, Hkv, tpb, lens=None):
    """probs: float32 [R, Hq, T] -> block mass [R, Hkv, nb]."""
    probs = np.ascontiguousarray(probs, np.float32)
    R, hq, T = probs.shape
    assert hq == Hq
    nb = (T + tpb - 1) // tpb
    out = np.zeros((R, Hkv, nb), np.float32)
    lens_arr = None if lens is None else np.ascontiguousarray(lens, np.uint32)
    lib().oc_score_blocks(probs.reshape(-1), R, Hq, Hkv, T, tpb,
                          None if lens_arr is None else lens_arr.ctypes.data,
                          out.reshape(-1))
    return out


class Athresh:
    """Adaptive threshold restatement (cooldown handled by the caller)."""

    def __init__(self, th_hot=0.5, th_warm=0.2, min_hot=0.2, max_hot=0.9,
                 min_warm=0.05, max_warm=0.5, gpu_hwm=0.9, gpu_lwm=0.7,
                 dram_hwm=0.9, dram_lwm=0.7, step=0.02):
        self._a = _Athresh(th_hot, th_warm, min_hot, max_hot, min_warm, max_warm,
                           gpu_hwm, gpu_lwm, dram_hwm, dram_lwm, step, 0, 0, 0)

    def update(self, gpu, dram):
        return bool(lib().oc_athresh_update(C.byref(self._a), gpu, dram))

    def __getattr__(self, name):
        return getattr(self.__dict__["_a"], name)


class OracleTM:
    """tiered_manager restatement over OracleSched + Athresh.

    Follows src/scheduler/tiered_manager.c: register (:147-167) appends to the
    registry (duplicates included, ERR_TIER_FULL past max_blocks); step_done
    (:205-213) = tracker step + prefetch step reset; schedule_once (:314-336) =
    classify, threshold update, GPU/DRAM demote checks (no transfer callback,
    as from the binding, so nothing moves), prefetch scan + dispatch counts
    (src/scheduler/prefetch_scheduler.c:131-228, heap capacity 1024, tracking
    capacity 512).  The threshold cooldown is taken as 0 (always elapsed).
    """

    HEAP_CAP = 1024
    TRACK_CAP = 512

    def __init__(self, tracker_cap=4096, ema_lambda=0.9, alpha=0.5, beta=0.3, gamma=0.2,
                 prefetch_budget=16, gpu_hwm=0.9, gpu_lwm=0.7, dram_hwm=0.9,
                 dram_lwm=0.7, max_blocks=8192, threshold_to_gpu=0.5,
                 threshold_to_dram=0.2, recency_tau=50.0, adjust_step=0.02,
                 demote_batch=8, prefetch_batch=8):
        self.s = OracleSched(tracker_cap, ema_lambda, alpha, beta, gamma, recency_tau)
        self.a = Athresh(gpu_hwm=gpu_hwm, gpu_lwm=gpu_lwm, dram_hwm=dram_hwm,
                         dram_lwm=dram_lwm, step=adjust_step if adjust_step > 0 else 0.02)
        self.s.set_thresholds(self.a.th_hot, self.a.th_warm)
        self.max_blocks = max_blocks if max_blocks > 0 else 4096
        self.registry = []            # [id, tier, flags]
        self.budget = prefetch_budget if prefetch_budget > 0 else 16
        self.th_gpu, self.th_dram = threshold_to_gpu, threshold_to_dram
        self.prefetch_batch = prefetch_batch
        self.heap_size = 0
        self.tracked = 0
        self.cnt = dict(schedule_cycles=0, prefetches_dispatched=0, total_scanned=0,
                        total_enqueued=0, total_dispatched=0, prefetch_wasted=0,
                        demote_checks=0)
        self.gpu_ratio = 0.0
        self.dram_ratio = 0.0

    def register(self, bid, tier=0, flags=0):
        if len(self.registry) >= self.max_blocks:
            return -4
        self.registry.append([bid, tier, flags])
        self.s.register(bid, flags)
        return 0

    def set_block_tier(self, bid, tier):
        for e in self.registry:
            if e[0] == bid:
                e[1] = tier
                return

    def report(self, bid, w):
        self.s.update(bid, np.float32(w))

    def step_done(self):
        self.s.step_done()
        self.cnt["prefetch_wasted"] += self.tracked
        self.tracked = 0
        self.heap_size = 0

    def set_usage(self, g, d):
        self.gpu_ratio, self.dram_ratio = np.float32(g), np.float32(d)

    def schedule_once(self):
        self.s.update_all()
        if self.a.update(self.gpu_ratio, self.dram_ratio):
            self.s.set_thresholds(self.a.th_hot, self.a.th_warm)
        self.cnt["demote_checks"] += 2
        st = self.s.state()
        mask = self.s.cap - 1
        for bid, tier, _ in self.registry:
            if tier in (0, 4):
                continue
            self.cnt["total_scanned"] += 1
            slot = bid & mask
            if not st["t_active"][slot]:
                continue
            e = st["ema"][slot]
            if e >= np.float32(self.th_gpu) or (e >= np.float32(self.th_dram) and tier != 1):
                if self.heap_size < self.HEAP_CAP:
                    self.heap_size += 1
                    self.cnt["total_enqueued"] += 1
        lim = min(self.prefetch_batch, self.budget)
        d = min(lim, self.heap_size)
        self.heap_size -= d
        self.tracked = min(self.tracked + d, self.TRACK_CAP)
        self.cnt["total_dispatched"] += d
        self.cnt["prefetches_dispatched"] += d
        self.cnt["schedule_cycles"] += 1

    def score(self, bid):
        st = self.s.state()
        slot = bid & (self.s.cap - 1)
        return st["hot"][slot] if st["c_active"][slot] else np.float32(0.0)

    def heat(self, bid):
        st = self.s.state()
        slot = bid & (self.s.cap - 1)
        return int(st["heat"][slot]) if st["c_active"][slot] else 2

    def stats(self):
        st = self.s.state()
        act = st["c_active"].astype(bool)
        heat = st["heat"][act]
        out = dict(self.cnt)
        out.update(n_hot=int((heat == 0).sum()), n_warm=int((heat == 1).sum()),
                   n_cold=int((heat == 2).sum()),
                   threshold_adj_up=int(self.a.up), threshold_adj_down=int(self.a.down),
                   threshold_hot=float(np.float32(self.a.th_hot)),
                   threshold_warm=float(np.float32(self.a.th_warm)),
                   gpu_used_ratio=float(self.gpu_ratio), dram_used_ratio=float(self.dram_ratio),
                   n_attn_sink=int((st["c_flags"][act] & 0x08 != 0).sum()))
        return out


# ---------------------------------------------------------------------------
# Data-plane restatement (byte/integer work): numpy + small Python loops
# ---------------------------------------------------------------------------

def loc(tier, slab):
    return (int(tier) << 29) | int(slab)


def loc_tier(w):
    return int(w) >> 29


def loc_slab(w):
    return int(w) & 0x1FFFFFFF


class Pool:
    """LIFO slab pool (src/tiered_store/gpu_tier.cu:36-93, dram_tier.cu)."""

    def __init__(self, total):
        self.stack = list(range(total - 1, -1, -1))
        self.total = total

    @property
    def top(self):
        return len(self.stack)

    def pop(self):
        return self.stack.pop() if self.stack else None

    def push(self, idx):
        self.stack.append(idx)


def evict_batch(gpu, dram, locs, state, flags, handles, gpu_bytes, dram_bytes, slab):
    """Reference per-block evict (src/api/orchkv_api.cu:353-389) in list order.
    gpu_bytes/dram_bytes are uint8 arrays of pool_slabs*slab bytes."""
    done = skipped = 0
    for h in handles:
        w = locs[h]
        if loc_tier(w) != 0 or (flags is not None and flags[h] & 0x01):
            skipped += 1
            continue
        d = dram.pop()
        if d is None:
            skipped += 1
            continue
        g = loc_slab(w)
        dram_bytes[d * slab:(d + 1) * slab] = gpu_bytes[g * slab:(g + 1) * slab]
        locs[h] = loc(1, d)
        state[h] = 3
        gpu.push(g)
        done += 1
    return done, skipped


def promote_batch(gpu, dram, locs, state, handles, gpu_bytes, dram_bytes, slab):
    """Reference per-block promote (src/api/orchkv_api.cu:393-428) in list order."""
    done = skipped = 0
    for h in handles:
        w = locs[h]
        if loc_tier(w) != 1:
            skipped += 1
            continue
        g = gpu.pop()
        if g is None:
            skipped += 1
            continue
        d = loc_slab(w)
        gpu_bytes[g * slab:(g + 1) * slab] = dram_bytes[d * slab:(d + 1) * slab]
        locs[h] = loc(0, g)
        state[h] = 2
        dram.push(d)
        done += 1
    return done, skipped


# ---------------------------------------------------------------------------
# The reference itself, compiled from its sources (oracle/_ref)
# ---------------------------------------------------------------------------

_REF = None


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref():
    global _REF
    if _REF is None:
        L = _load(REF_SO)
        vp = C.c_void_p
        L.ref_tm_create.argtypes = [C.c_uint32, C.c_float, C.c_float, C.c_float, C.c_float,
                                    C.c_uint32, C.c_float, C.c_float, C.c_float, C.c_float,
                                    C.c_uint32, C.c_float, C.c_float, C.c_float, C.c_double,
                                    C.c_float, C.c_uint32, C.c_uint32]
        L.ref_tm_create.restype = vp
        L.ref_tm_destroy.argtypes = [vp]
        L.ref_tm_register_id.argtypes = [vp, C.c_uint64, C.c_int, C.c_uint8]
        L.ref_tm_register_id.restype = C.c_int
        L.ref_tm_set_block_tier.argtypes = [vp, C.c_uint64, C.c_int]
        L.ref_tm_register_range.argtypes = [vp, C.c_uint32]
        L.ref_tm_register_range.restype = C.c_int
        L.ref_tm_set_tiers.argtypes = [vp, _u64p, C.c_uint32, C.c_int]
        L.ref_tm_notify_access.argtypes = [vp, C.c_uint64]
        L.ref_tm_report.argtypes = [vp, C.c_uint64, C.c_float]
        L.ref_tm_report_batch.argtypes = [vp, _u64p, _f32p, C.c_uint32]
        L.ref_tm_step_done.argtypes = [vp]
        L.ref_tm_set_usage.argtypes = [vp, C.c_float, C.c_float]
        L.ref_tm_schedule_once.argtypes = [vp]
        L.ref_tm_update_all.argtypes = [vp]
        L.ref_tm_set_policy.argtypes = [vp, C.c_float, C.c_float, C.c_float]
        L.ref_tm_score.argtypes = [vp, C.c_uint64]
        L.ref_tm_score.restype = C.c_float
        L.ref_tm_heat.argtypes = [vp, C.c_uint64]
        L.ref_tm_heat.restype = C.c_int
        L.ref_tm_capacity.argtypes = [vp]
        L.ref_tm_capacity.restype = C.c_uint32
        L.ref_tm_step.argtypes = [vp]
        L.ref_tm_step.restype = C.c_uint64
        L.ref_tm_stats.argtypes = [vp, _f64p]
        L.ref_tm_dump.argtypes = [vp, _f32p, _f32p, _u32p, _u64p, _u8p, _f32p, _u8p, _u8p]
        L.ref_tm_select_gpu_victims.argtypes = [vp, C.c_uint32, _u64p, _f32p]
        L.ref_tm_select_gpu_victims.restype = C.c_uint32
        L.ref_tm_decay_table.argtypes = [vp, _f32p]
        L.ref_dram_pool_create.argtypes = [C.c_uint32, C.c_uint32]
        L.ref_dram_pool_create.restype = vp
        L.ref_dram_pool_alloc.argtypes = [vp]
        L.ref_dram_pool_alloc.restype = C.c_longlong
        L.ref_dram_pool_free.argtypes = [vp, C.c_uint32]
        L.ref_dram_pool_free.restype = C.c_int
        L.ref_dram_pool_destroy.argtypes = [vp]
        L.ref_arm_sched_step.argtypes = [vp, _u64p, _f32p, C.c_uint32, C.c_float,
                                         C.c_uint32, _u64p, _f64p]
        L.ref_arm_sched_step.restype = C.c_uint32
        L.ref_api_init.argtypes = [C.c_int, C.c_size_t, C.c_size_t, C.c_uint32, C.c_uint32,
                                   C.c_int, C.c_int, C.c_uint32, C.c_char_p]
        L.ref_api_init.restype = C.c_int
        L.ref_api_shutdown.restype = C.c_int
        L.ref_api_request_create.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32]
        L.ref_api_request_create.restype = vp
        L.ref_api_request_destroy.argtypes = [vp]
        L.ref_api_request_destroy.restype = C.c_int
        L.ref_api_prefill.argtypes = [vp, C.c_uint32, vp, vp, C.c_uint32]
        L.ref_api_prefill.restype = C.c_int
        L.ref_api_append.argtypes = [vp, C.c_uint32, vp, vp]
        L.ref_api_append.restype = C.c_int
        for n in ("ref_api_evict", "ref_api_promote", "ref_api_evict_cold",
                  "ref_api_promote_storage"):
            getattr(L, n).argtypes = [vp, C.c_uint32, C.c_uint32, C.c_uint32]
            getattr(L, n).restype = C.c_int
        L.ref_api_get.argtypes = [vp, C.c_uint32, C.c_uint32, C.c_uint32,
                                  C.POINTER(vp), C.POINTER(vp)]
        L.ref_api_get.restype = C.c_int
        L.ref_api_dram_base.restype = vp
        L.ref_api_gpu_base.restype = vp
        L.ref_api_block.argtypes = [vp, C.c_uint32, C.c_uint32, C.c_uint32,
                                    C.POINTER(C.c_int), C.POINTER(vp)]
        L.ref_api_block.restype = C.c_int
        L.ref_api_migrate_list.argtypes = [vp, _u32p, C.c_uint32, C.c_uint32, _f64p]
        L.ref_api_migrate_list.restype = C.c_int
        L.ref_storage_read.argtypes = [C.c_char_p, C.c_uint64, C.c_uint32, C.c_uint32,
                                       C.c_uint32, C.c_size_t, C.c_uint32, C.c_uint32,
                                       C.c_uint32, vp]
        L.ref_storage_read.restype = C.c_int
        _i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
        L.ref_c4_scenario.argtypes = [C.c_uint32, _u64p, _i32p, _u8p, _u32p, C.c_uint32,
                                      C.c_uint32, _u64p, _f32p, _u32p, _f32p, _f32p,
                                      C.c_uint32, C.c_float, C.c_float, C.c_float, _i32p,
                                      _i32p, _i32p, _f64p, C.c_uint32]
        L.ref_c4_scenario.restype = C.c_int
        _REF = L
    return _REF


STAT_KEYS = ["schedule_cycles", "gpu_demotes", "dram_demotes", "prefetches_dispatched",
             "gpu_used_ratio", "dram_used_ratio", "blocks_migrated", "migration_errors",
             "prefetch_hits", "prefetch_wasted", "prefetch_hit_rate", "n_hot", "n_warm",
             "n_cold", "threshold_adj_up", "threshold_adj_down", "threshold_hot",
             "threshold_warm", "total_scanned", "total_enqueued", "total_dispatched",
             "n_attn_sink", "avg_hotness", "max_hotness", "min_hotness", "demote_checks"]


class RefTM:
    """The reference tiered manager, configured like the reference binding's
    tm_create (bindings/orchkv_pybind.cpp:215-271, same defaults)."""

    def __init__(self, tracker_cap=4096, ema_lambda=0.9, alpha=0.5, beta=0.3, gamma=0.2,
                 prefetch_budget=16, gpu_hwm=0.9, gpu_lwm=0.7, dram_hwm=0.9,
                 dram_lwm=0.7, max_blocks=8192, threshold_to_gpu=0.5,
                 threshold_to_dram=0.2, recency_tau=50.0, cooldown_sec=0.5,
                 adjust_step=0.02, demote_batch=0, prefetch_batch=0):
        self.h = ref().ref_tm_create(tracker_cap, ema_lambda, alpha, beta, gamma,
                                     prefetch_budget, gpu_hwm, gpu_lwm, dram_hwm, dram_lwm,
                                     max_blocks, threshold_to_gpu, threshold_to_dram,
                                     recency_tau, cooldown_sec, adjust_step,
                                     demote_batch, prefetch_batch)
        if not self.h:
            raise RuntimeError("ref_tm_create failed")
        self.cap = ref().ref_tm_capacity(self.h)

    def close(self):
        if self.h:
            ref().ref_tm_destroy(self.h)
            self.h = None

    __del__ = close

    def register(self, bid, tier=0, flags=0):
        return ref().ref_tm_register_id(self.h, bid, tier, flags)

    def set_block_tier(self, bid, tier):
        ref().ref_tm_set_block_tier(self.h, bid, tier)

    def register_range(self, n):
        """Register ids 0..n-1 (tier GPU, no flags) in order."""
        rc = ref().ref_tm_register_range(self.h, n)
        if rc != 0:
            raise RuntimeError(f"ref_tm_register_range: {rc}")

    def set_tiers(self, ids, tier):
        ids = np.ascontiguousarray(ids, np.uint64)
        ref().ref_tm_set_tiers(self.h, ids, len(ids), tier)

    def notify_access(self, bid):
        ref().ref_tm_notify_access(self.h, bid)

    def report(self, bid, w):
        ref().ref_tm_report(self.h, bid, w)

    def report_batch(self, ids, w):
        ids = np.ascontiguousarray(ids, np.uint64)
        ref().ref_tm_report_batch(self.h, ids, np.ascontiguousarray(w, np.float32), len(ids))

    def step_done(self):
        ref().ref_tm_step_done(self.h)

    def set_usage(self, g, d):
        ref().ref_tm_set_usage(self.h, g, d)

    def schedule_once(self):
        ref().ref_tm_schedule_once(self.h)

    def update_all(self):
        ref().ref_tm_update_all(self.h)

    def set_policy(self, a, b, g):
        ref().ref_tm_set_policy(self.h, a, b, g)

    def score(self, bid):
        return ref().ref_tm_score(self.h, bid)

    def heat(self, bid):
        return ref().ref_tm_heat(self.h, bid)

    @property
    def step(self):
        return ref().ref_tm_step(self.h)

    def stats(self):
        o = np.zeros(len(STAT_KEYS), np.float64)
        ref().ref_tm_stats(self.h, o)
        return dict(zip(STAT_KEYS, o.tolist()))

    def state(self):
        n = self.cap
        out = {"sum": np.zeros(n, np.float32), "ema": np.zeros(n, np.float32),
               "hits": np.zeros(n, np.uint32), "last": np.zeros(n, np.uint64),
               "t_active": np.zeros(n, np.uint8), "hot": np.zeros(n, np.float32),
               "heat": np.zeros(n, np.uint8), "c_active": np.zeros(n, np.uint8)}
        ref().ref_tm_dump(self.h, out["sum"], out["ema"], out["hits"], out["last"],
                          out["t_active"], out["hot"], out["heat"], out["c_active"])
        return out

    def select_gpu_victims(self, n):
        ids = np.zeros(max(n, 1), np.uint64)
        sc = np.zeros(max(n, 1), np.float32)
        f = ref().ref_tm_select_gpu_victims(self.h, n, ids, sc)
        return ids[:f].copy(), sc[:f].copy()

    def decay_table(self):
        t = np.zeros(512, np.float32)
        ref().ref_tm_decay_table(self.h, t)
        return t


class RefDramPool:
    def __init__(self, slabs, slab_size=64):
        self.h = ref().ref_dram_pool_create(slabs, slab_size)

    def alloc(self):
        r = ref().ref_dram_pool_alloc(self.h)
        return None if r < 0 else int(r)

    def free(self, idx):
        return ref().ref_dram_pool_free(self.h, idx)

    def close(self):
        if self.h:
            ref().ref_dram_pool_destroy(self.h)
            self.h = None

    __del__ = close
