"""orchkv_b200 — B200-native (sm_100a) implementation of OrchKvCache's
per-decode-step KV-cache scheduling and migration path.

Two doors into the same native library (liborchkv_b200.so):

* the C ABI (include/orchkv/*.h), bound here with ctypes (``lib()``), and
* the ``orchkv_core`` pybind11 module with the reference binding's names;
  ``core()`` loads it and registers it as the top-level module
  ``orchkv_core`` so unmodified callers doing ``import orchkv_core`` get it.

Callers of the reference's Python layer have B200 counterparts with the
same interfaces: ``fast_manager.FastKVCacheManager``,
``kvcache_manager.KVCacheManager``, ``vllm_connector.OrchKvOffloadingConnector``
and ``attention_hook.AttentionScoreCollector`` / ``AttentionHookManager``.

There is no CPU fallback: if the library has not been built, the first call
into it (``lib()`` or ``core()``) raises.
"""
from __future__ import annotations

import ctypes as C
import importlib.machinery
import importlib.util
import os
import sys

from . import _lib
from ._lib import (KvBlock, OrchkvConfig, OrchkvConfigExt, OrchkvStats, TieredManager,
                   TmConfig, TmStats)

__all__ = ["lib", "core", "Manager", "make_config", "KvBlock", "OrchkvConfig",
           "OrchkvConfigExt", "OrchkvStats", "TieredManager", "TmConfig", "TmStats",
           "ERR"]

ERR = dict(OK=0, OOM=-1, INVALID=-2, NOT_FOUND=-3, TIER_FULL=-4, CUDA=-5, IO=-6,
           LOCKED=-7, STATE=-8, INIT=-9, ALREADY=-10)


def lib() -> C.CDLL:
    return _lib.load()


_CORE = None


def core():
    """Load the orchkv_core extension and register it as ``orchkv_core``."""
    global _CORE
    if _CORE is None:
        from .build import core_module_path
        path = core_module_path(_lib.LIB_DIR)
        if not os.path.exists(path):
            raise ImportError(f"{path} not built: run `python -m orchkv_b200.build`")
        loader = importlib.machinery.ExtensionFileLoader("orchkv_core", path)
        spec = importlib.util.spec_from_file_location("orchkv_core", path, loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        sys.modules["orchkv_core"] = mod
        _CORE = mod
    return _CORE


def make_config(gpu_pool_bytes, dram_pool_bytes, tokens_per_block=64, d_head=128, dtype=0,
                device=0, max_blocks_per_head=256):
    cfg = OrchkvConfig()
    cfg.gpu_device_id = device
    cfg.gpu_pool_bytes = gpu_pool_bytes
    cfg.dram_pool_bytes = dram_pool_bytes
    cfg.dram_use_pinned = True
    cfg.num_cuda_streams = 4
    cfg.tokens_per_block = tokens_per_block
    cfg.d_head = d_head
    cfg.dtype = dtype
    cfg.gpu_hwm, cfg.gpu_lwm, cfg.dram_hwm, cfg.dram_lwm = 0.9, 0.7, 0.9, 0.7
    cfg.orchfs_base_dir = b"/dev/shm/orchkv"
    cfg.nvm_io_threads, cfg.ssd_io_threads, cfg.orchfs_io_workers = 4, 16, 4
    cfg.max_blocks_per_head = max_blocks_per_head
    return cfg


class Manager:
    """Thin owner of one tiered_manager_t through the C ABI."""

    def __init__(self, tracker_cap=4096, ema_lambda=0.9, alpha=0.5, beta=0.3, gamma=0.2,
                 recency_tau=50.0, prefetch_budget=16, max_blocks=8192, gpu_hwm=0.9,
                 gpu_lwm=0.7, dram_hwm=0.9, dram_lwm=0.7, threshold_to_gpu=0.5,
                 threshold_to_dram=0.2, cooldown_sec=0.5, adjust_step=0.02,
                 demote_batch_size=8, prefetch_batch_size=8):
        L = lib()
        cfg = TmConfig()
        L.tm_config_default(C.byref(cfg))
        cfg.tracker_capacity = tracker_cap
        cfg.ema_lambda = ema_lambda
        cfg.hcc_params.alpha, cfg.hcc_params.beta, cfg.hcc_params.gamma = alpha, beta, gamma
        cfg.hcc_params.recency_tau = recency_tau
        cfg.prefetch_budget = prefetch_budget
        cfg.max_blocks = max_blocks
        ap = cfg.athresh_params
        ap.gpu_hwm, ap.gpu_lwm, ap.dram_hwm, ap.dram_lwm = gpu_hwm, gpu_lwm, dram_hwm, dram_lwm
        ap.cooldown_sec = cooldown_sec
        ap.adjust_step = adjust_step
        cfg.threshold_to_gpu = threshold_to_gpu
        cfg.threshold_to_dram = threshold_to_dram
        cfg.demote_batch_size = demote_batch_size
        cfg.prefetch_batch_size = prefetch_batch_size
        self.cfg = cfg
        self.tm = TieredManager()
        rc = L.tm_init(C.byref(self.tm), C.byref(cfg))
        if rc != 0:
            raise RuntimeError(f"tm_init failed: {rc}")
        self.cap = L.tm_capacity(C.byref(self.tm))
        self._blocks = []

    @property
    def ref(self):
        return C.byref(self.tm)

    def close(self):
        if self.tm.impl:
            lib().tm_destroy(C.byref(self.tm))

    def register_id(self, block_id, tier=0, flags=0):
        b = KvBlock()
        b.block_id = block_id
        b.tier = tier
        b.flags = flags
        rc = lib().tm_register_block(self.ref, C.byref(b))
        if rc == 0:
            self._blocks.append(b)
        return rc

    def set_block_tier(self, block_id, tier):
        return lib().tm_set_block_tier_id(self.ref, block_id, tier)

    def report(self, block_id, w):
        lib().tm_notify_attn(self.ref, block_id, w)

    def step_done(self):
        lib().tm_step_done(self.ref)

    def set_usage(self, g, d):
        lib().tm_set_usage(self.ref, g, d)

    def schedule_once(self):
        lib().tm_schedule_once(self.ref)

    def score(self, block_id):
        return lib().tm_get_block_score(self.ref, block_id)

    def heat(self, block_id):
        return lib().tm_get_block_heat(self.ref, block_id)

    def stats(self):
        s = TmStats()
        lib().tm_get_stats(self.ref, C.byref(s))
        hot, warm = C.c_float(), C.c_float()
        up, down = C.c_uint64(), C.c_uint64()
        lib().tm_get_threshold_state(self.ref, C.byref(hot), C.byref(warm), C.byref(up),
                                     C.byref(down))
        return dict(
            schedule_cycles=s.schedule_cycles, gpu_demotes=s.gpu_demotes,
            dram_demotes=s.dram_demotes, prefetches_dispatched=s.prefetches_dispatched,
            gpu_used_ratio=s.gpu_used_ratio, dram_used_ratio=s.dram_used_ratio,
            blocks_migrated=s.migration_stats.blocks_migrated,
            migration_errors=s.migration_stats.op_errors,
            prefetch_hits=s.prefetch_stats.prefetch_hits,
            prefetch_wasted=s.prefetch_stats.prefetch_wasted,
            prefetch_hit_rate=s.prefetch_stats.hit_rate,
            n_hot=s.hcc_stats.n_hot, n_warm=s.hcc_stats.n_warm, n_cold=s.hcc_stats.n_cold,
            threshold_adj_up=up.value, threshold_adj_down=down.value,
            threshold_hot=hot.value, threshold_warm=warm.value,
            total_scanned=s.prefetch_stats.total_scanned,
            total_enqueued=s.prefetch_stats.total_enqueued,
            total_dispatched=s.prefetch_stats.total_dispatched,
            n_attn_sink=s.hcc_stats.n_attn_sink, avg_hotness=s.hcc_stats.avg_hotness,
            max_hotness=s.hcc_stats.max_hotness, min_hotness=s.hcc_stats.min_hotness)

    def state(self):
        import numpy as np
        n = self.cap
        out = {"sum": np.zeros(n, np.float32), "ema": np.zeros(n, np.float32),
               "hits": np.zeros(n, np.uint32), "last": np.zeros(n, np.uint64),
               "t_active": np.zeros(n, np.uint8), "hot": np.zeros(n, np.float32),
               "heat": np.zeros(n, np.uint8), "c_active": np.zeros(n, np.uint8)}
        rc = lib().tm_read_state(self.ref, *(out[k].ctypes.data for k in (
            "sum", "ema", "hits", "last", "t_active", "hot", "heat", "c_active")))
        if rc != 0:
            raise RuntimeError(f"tm_read_state failed: {rc}")
        return out
