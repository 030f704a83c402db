"""ctypes binding of liborchkv_b200.so (the C ABI in include/orchkv/*.h).

The library is required: importing this module without a built library
raises, so no caller can silently run without the CUDA implementation.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
# ORCHKV_CHECKED=1 selects the checked build (bounds-checked data-plane kernels)
LIB_DIR = os.path.join(PKG, "_checked") if os.environ.get("ORCHKV_CHECKED") == "1" else PKG
LIB_PATH = os.path.join(LIB_DIR, "liborchkv_b200.so")

vp = C.c_void_p
u8, u32, u64, i32, f32, f64 = C.c_uint8, C.c_uint32, C.c_uint64, C.c_int, C.c_float, C.c_double
P = C.POINTER


class OrchkvConfig(C.Structure):
    """orchkv_config_t (include/orchkv/kv_types.h)."""
    _fields_ = [
        ("gpu_device_id", i32), ("gpu_pool_bytes", C.c_size_t), ("dram_pool_bytes", C.c_size_t),
        ("dram_use_pinned", C.c_bool), ("num_cuda_streams", i32), ("tokens_per_block", u32),
        ("d_head", u32), ("dtype", i32), ("gpu_hwm", f32), ("gpu_lwm", f32), ("dram_hwm", f32),
        ("dram_lwm", f32), ("orchfs_base_dir", C.c_char_p), ("orchfs_nvm_path", C.c_char_p),
        ("orchfs_ssd_path", C.c_char_p), ("nvm_io_threads", i32), ("ssd_io_threads", i32),
        ("orchfs_io_workers", i32), ("max_blocks_per_head", u32),
    ]


class OrchkvConfigExt(C.Structure):
    _fields_ = [("max_blocks", u32), ("max_requests", u32), ("table_entries", u64),
                ("staging_mb", u32), ("reserved", u32 * 11)]


class OrchkvStats(C.Structure):
    _fields_ = [
        ("gpu_pool_total", C.c_size_t), ("gpu_pool_used", C.c_size_t),
        ("gpu_slabs_total", u32), ("gpu_slabs_used", u32),
        ("dram_pool_total", C.c_size_t), ("dram_pool_used", C.c_size_t),
        ("dram_slabs_total", u32), ("dram_slabs_used", u32),
        ("total_blocks", u64), ("blocks_on_gpu", u64), ("blocks_on_dram", u64),
        ("blocks_on_nvm", u64), ("blocks_on_ssd", u64), ("transfers_d2h", u64),
        ("transfers_h2d", u64), ("bytes_d2h", u64), ("bytes_h2d", u64),
        ("active_requests", u32),
    ]


class HccParams(C.Structure):
    _fields_ = [(n, f32) for n in ("alpha", "beta", "gamma", "recency_tau", "threshold_hot",
                                   "threshold_warm")]


class AthreshParams(C.Structure):
    _fields_ = [(n, f32) for n in ("threshold_hot", "threshold_warm", "min_hot", "max_hot",
                                   "min_warm", "max_warm", "gpu_hwm", "gpu_lwm", "dram_hwm",
                                   "dram_lwm", "adjust_step")] + [("cooldown_sec", f64)]


class TmConfig(C.Structure):
    """tm_config_t (include/orchkv/tiered_manager.h)."""
    _fields_ = [
        ("tracker_capacity", u32), ("ema_lambda", f32), ("hcc_params", HccParams),
        ("athresh_params", AthreshParams), ("w_heat", f32), ("w_lru", f32),
        ("tokens_per_block", u32), ("prefetch_budget", u32), ("threshold_to_gpu", f32),
        ("threshold_to_dram", f32), ("transfer_fn", vp), ("transfer_ctx", vp),
        ("alloc_fn", vp), ("free_fn", vp), ("alloc_ctx", vp), ("block_data_size", C.c_size_t),
        ("schedule_interval_us", u32), ("demote_batch_size", u32), ("prefetch_batch_size", u32),
        ("max_blocks", u32), ("auto_schedule", C.c_bool),
    ]


class HccStats(C.Structure):
    _fields_ = [("n_hot", u32), ("n_warm", u32), ("n_cold", u32), ("n_attn_sink", u32),
                ("avg_hotness", f32), ("max_hotness", f32), ("min_hotness", f32)]


class PrefetchStats(C.Structure):
    _fields_ = [("total_scanned", u64), ("total_enqueued", u64), ("total_dispatched", u64),
                ("prefetch_hits", u64), ("prefetch_wasted", u64), ("hit_rate", f32)]


class MigStats(C.Structure):
    _fields_ = [("op_count", u64 * 6), ("op_bytes", u64 * 6), ("op_errors", u64),
                ("blocks_migrated", u64)]


class TmStats(C.Structure):
    _fields_ = [("schedule_cycles", u64), ("gpu_demotes", u64), ("dram_demotes", u64),
                ("prefetches_dispatched", u64), ("gpu_used_ratio", f32),
                ("dram_used_ratio", f32), ("hcc_stats", HccStats),
                ("prefetch_stats", PrefetchStats), ("migration_stats", MigStats)]


class TieredManager(C.Structure):
    _fields_ = [("impl", vp), ("reserved", u64 * 7)]


class KvBlock(C.Structure):
    """kv_block_t (layout of the reference's src/core/kv_block.h:22-52)."""
    _fields_ = [
        ("block_id", u64), ("request_id", u64), ("layer_id", C.c_uint16), ("head_id", C.c_uint16),
        ("token_start", u32), ("token_count", C.c_uint16), ("_pad0", C.c_uint16), ("tier", i32),
        ("data_ptr", vp), ("persistent_offset", u64), ("hotness", f32),
        ("last_access_step", u64), ("access_count", u32), ("state", i32), ("flags", u8),
        ("lock", C.c_byte * 56), ("prev", vp), ("next", vp),
    ]


_SIGS = {
    # data plane
    "orchkv_init": (i32, [P(OrchkvConfig)]),
    "orchkv_init_ext": (i32, [P(OrchkvConfig), P(OrchkvConfigExt)]),
    "orchkv_shutdown": (i32, []),
    "orchkv_is_initialized": (C.c_bool, []),
    "orchkv_request_create": (vp, [u64, u32, u32]),
    "orchkv_request_destroy": (i32, [vp]),
    "orchkv_prefill": (i32, [vp, u32, vp, vp, u32]),
    "orchkv_append_token": (i32, [vp, u32, vp, vp]),
    "orchkv_get_kv_block": (i32, [vp, u32, u32, u32, P(vp), P(vp)]),
    "orchkv_evict_to_dram": (i32, [vp, u32, u32, u32]),
    "orchkv_promote_to_gpu": (i32, [vp, u32, u32, u32]),
    "orchkv_evict_to_storage": (i32, [vp, u32, u32, u32]),
    "orchkv_promote_from_storage": (i32, [vp, u32, u32, u32]),
    "orchkv_evict_cold": (i32, [vp, u32, u32, u32]),
    "orchkv_storage_flush": (None, []),
    "orchkv_get_stats": (i32, [P(OrchkvStats)]),
    "orchkv_gpu_tier": (vp, []),
    "orchkv_dram_tier": (vp, []),
    "orchkv_orchfs_tier": (vp, []),
    "orchkv_set_stream": (i32, [vp]),
    "orchkv_sync": (i32, []),
    "orchkv_attach_scheduler": (i32, [P(TieredManager)]),
    "orchkv_append_token_batch": (i32, [P(vp), u32, vp, vp]),
    "orchkv_evict_batch_to_dram": (i32, [vp, vp, u32, vp]),
    "orchkv_promote_batch_to_gpu": (i32, [vp, vp, u32, vp]),
    "orchkv_block_id_table": (i32, [P(vp), u32, u32, vp]),
    "orchkv_block_info": (i32, [vp, u32, u32, u32, P(u64), P(i32), P(u32), P(i32), P(u32)]),
    "orchkv_set_block_flags": (i32, [vp, u32, u32, u32, u8]),
    "orchkv_read_pool": (i32, [i32, vp, P(u32)]),
    "orchkv_read_block_locs": (i32, [vp, vp]),
    "orchkv_max_blocks": (u32, []),
    "orchkv_kernel_launches": (C.c_ulonglong, []),
    "orchkv_last_migration_profile": (i32, [P(f32), P(C.c_ulonglong), P(u32), P(f32)]),
    "orchkv_last_evict_layout": (i32, [P(u32), P(u32), P(u32)]),
    "orchkv_last_pack_chunks": (i32, [P(f32), u32, P(u32)]),
    "orchkv_last_unpack_chunks": (i32, [P(f32), P(C.c_ulonglong), u32, P(u32)]),
    "orchkv_evict_batch_to_storage": (i32, [vp, vp, u32, vp]),
    "orchkv_promote_batch_from_storage": (i32, [vp, vp, u32, vp]),
    "orchkv_evict_cold_batch": (i32, [vp, vp, u32, vp]),
    "orchkv_last_promote_layout": (i32, [P(u32), P(u32), P(u32), P(i32)]),
    "orchkv_swap_batch": (i32, [vp, vp, u32, vp, vp, u32, vp]),
    "orchkv_block_checksums": (i32, [vp, u32, vp, vp]),
    "orchkv_checked_build": (i32, []),
    "orchkv_check_status": (i32, [vp, i32]),
    "orchkv_check_inject": (i32, [u32]),
    "orchkv_gpu_pool_base": (vp, []),
    "orchkv_dram_pool_base": (vp, []),
    # scheduler
    "tm_config_default": (None, [P(TmConfig)]),
    "tm_init": (i32, [P(TieredManager), P(TmConfig)]),
    "tm_destroy": (None, [P(TieredManager)]),
    "tm_register_block": (i32, [P(TieredManager), P(KvBlock)]),
    "tm_unregister_block": (None, [P(TieredManager), P(KvBlock)]),
    "tm_notify_attn": (None, [P(TieredManager), u64, f32]),
    "tm_notify_access": (None, [P(TieredManager), P(KvBlock)]),
    "tm_step_done": (None, [P(TieredManager)]),
    "tm_schedule_once": (None, [P(TieredManager)]),
    "tm_start": (i32, [P(TieredManager)]),
    "tm_stop": (None, [P(TieredManager)]),
    "tm_set_usage": (None, [P(TieredManager), f32, f32]),
    "tm_set_policy": (None, [P(TieredManager), f32, f32, f32]),
    "tm_get_block_score": (f32, [P(TieredManager), u64]),
    "tm_get_block_heat": (i32, [P(TieredManager), u64]),
    "tm_get_stats": (None, [P(TieredManager), P(TmStats)]),
    "tm_set_stream": (i32, [P(TieredManager), vp]),
    "tm_sync": (i32, [P(TieredManager)]),
    "tm_capacity": (u32, [P(TieredManager)]),
    "tm_current_step": (u64, [P(TieredManager)]),
    "tm_set_block_tier_id": (i32, [P(TieredManager), u64, i32]),
    "tm_read_state": (i32, [P(TieredManager), vp, vp, vp, vp, vp, vp, vp, vp]),
    "tm_report_attn_probs": (i32, [P(TieredManager), vp, u32, u32, u32, u32, u32, vp, vp]),
    "tm_report_attn_batch_dev": (i32, [P(TieredManager), vp, vp, u32]),
    "tm_stage_input_async": (i32, [P(TieredManager), vp, C.c_size_t]),
    "tm_profile_reports": (i32, [P(TieredManager), i32]),
    "tm_last_report_times": (i32, [P(TieredManager), P(f32), P(f32), P(f32)]),
    "tm_report_attn_ranges": (i32, [P(TieredManager), vp, u32, u32, vp, vp, vp, u32]),
    "tm_report_attn_blockmean": (i32, [P(TieredManager), vp, i32, u32, u32, u32, u32, u32, vp,
                                       vp]),
    "tm_step_and_classify": (i32, [P(TieredManager)]),
    "tm_select_victims": (i32, [P(TieredManager), u32, vp, vp]),
    "tm_select_victims_frac": (i32, [P(TieredManager), f32, vp, vp, u32]),
    "tm_select_victims_masked": (i32, [P(TieredManager), u32, vp, vp, vp]),
    "orchkv_copy_token_blocks": (i32, [vp, u32, u32, u64, u32, u32, u32, vp, u32, vp, vp, i32, vp]),
    "tm_select_prefetch": (i32, [P(TieredManager), u32, f32, f32, vp, vp]),
    "tm_get_threshold_state": (i32, [P(TieredManager), P(f32), P(f32), P(u64), P(u64)]),
    "orchkv_select_coldest_noalloc": (i32, [vp, vp, u32, u32, vp, vp, vp]),
    # multi-GPU
    "orchkv_comm_unique_id": (i32, [vp]),
    "orchkv_comm_create": (vp, [i32, i32, vp, f64]),
    "orchkv_comm_destroy": (i32, [vp]),
    "orchkv_comm_allreduce_u32": (i32, [vp, vp, vp, u32, vp]),
    "orchkv_comm_exchange_time": (i32, [vp, P(f32), P(u32)]),
    "tm_set_comm": (i32, [P(TieredManager), vp]),
}

_lib = None


def load() -> C.CDLL:
    """Load liborchkv_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} not built: run `python -m orchkv_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def exported_names():
    return list(_SIGS)
