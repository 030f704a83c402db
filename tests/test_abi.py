"""C-ABI boundary checks that need no GPU: the library loads, exports every
function declared in include/orchkv/*.h, the struct layouts the reference
callers compile against are unchanged, and orchkv_core exposes the reference
binding's names (bindings/orchkv_pybind.cpp:26-416)."""
import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(ROOT, "include", "orchkv")


def declared_functions():
    names = set()
    for f in os.listdir(INC):
        if not f.endswith(".h"):
            continue
        src = open(os.path.join(INC, f)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"static inline[^{]*\{.*?\n\}", "", src, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w \*]*?\b(\w+)\s*\([^;{]*\)\s*;", src, flags=re.M):
            name = m.group(1)
            if name.startswith(("orchkv_", "tm_")):
                names.add(name)
    return sorted(names)


def test_library_loads_and_exports_every_declared_function():
    import orchkv_b200
    L = orchkv_b200.lib()
    names = declared_functions()
    assert len(names) >= 60
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    # every declared function is also bound by the ctypes layer
    from orchkv_b200 import _lib
    assert set(names) <= set(_lib.exported_names())


def test_accessors_before_init_return_null():
    """The subsystem accessors answer NULL while the data plane is not
    initialised (no CUDA call is made)."""
    from orchkv_b200 import _lib
    L = _lib.load()
    assert not L.orchkv_is_initialized()
    assert L.orchkv_gpu_tier() is None
    assert L.orchkv_dram_tier() is None
    assert L.orchkv_orchfs_tier() is None


def test_no_gpu_code_path_without_library():
    # the package refuses to run without the native library (no CPU fallback)
    import orchkv_b200._lib as lb
    assert os.path.exists(lb.LIB_PATH)


def test_struct_layouts_match_reference_abi():
    from orchkv_b200 import _lib
    # sizes of the reference structs on x86-64 (computed from the reference
    # headers: src/core/kv_types.h, src/core/kv_block.h, src/scheduler/*.h)
    assert C.sizeof(_lib.OrchkvConfig) == 104
    assert C.sizeof(_lib.OrchkvStats) == 128
    assert C.sizeof(_lib.KvBlock) == 152
    assert C.sizeof(_lib.TmConfig) == 184
    assert C.sizeof(_lib.TmStats) == 232


def test_orchfs_tier_snapshot_layout():
    """orchfs_tier_t as the reference lays it out on x86-64 (computed from
    src/tiered_store/orchfs_tier.h:40-51): 344 bytes, total_writes at 272,
    total_reads at 280, the mutex at 304, so the reference's inline
    orchfs_tier_writes / orchfs_tier_reads read the counters."""
    src = r"""
#include <stdio.h>
#include <stddef.h>
#include "orchkv/orchkv_api.h"
int main(void) {
  printf("%zu %zu %zu %zu\n", sizeof(orchfs_tier_t), offsetof(orchfs_tier_t, total_writes),
         offsetof(orchfs_tier_t, total_reads), offsetof(orchfs_tier_t, lock));
  return 0;
}
"""
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        open(c, "w").write(src)
        exe = os.path.join(d, "t")
        subprocess.run(["gcc", "-std=gnu11", "-I" + os.path.join(ROOT, "include"), c, "-o", exe],
                       check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()
    assert [int(x) for x in out] == [344, 272, 280, 304]


def test_enum_names_as_the_reference_prints_them():
    """dtype_name, tier_name and block_state_name return the reference's
    strings (src/core/kv_types.h:142-178), "unknown"/"UNKNOWN" out of range."""
    src = r"""
#include <stdio.h>
#include "orchkv/kv_types.h"
int main(void) {
  for (int i = 0; i <= 5; i++) printf("%s ", dtype_name((DataType)i));
  for (int i = 0; i <= 5; i++) printf("%s ", tier_name((StorageTier)i));
  for (int i = 0; i <= 7; i++) printf("%s ", block_state_name((KVBlockState)i));
  printf("%s\n", tier_name((StorageTier)-1));
  return 0;
}
"""
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        open(c, "w").write(src)
        exe = os.path.join(d, "t")
        subprocess.run(["gcc", "-std=gnu11", "-I" + os.path.join(ROOT, "include"), c, "-o", exe],
                       check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()
    assert out == ["fp16", "bf16", "fp32", "int8", "int4", "unknown",
                   "GPU_HBM", "HOST_DRAM", "NVM", "SSD", "NONE", "UNKNOWN",
                   "FREE", "ALLOCATED", "HOT", "WARM", "COLD", "MIGRATING", "EVICTED", "UNKNOWN",
                   "UNKNOWN"]


def test_struct_layouts_against_headers():
    """Compile the public headers and compare sizeof() with the ctypes mirror."""
    src = r"""
#include <stdio.h>
#include "orchkv/orchkv_api.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu %zu\n", sizeof(orchkv_config_t), sizeof(orchkv_stats_t),
         sizeof(kv_block_t), sizeof(tm_config_t), sizeof(tm_stats_t), sizeof(tiered_manager_t));
  return 0;
}
"""
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        open(c, "w").write(src)
        exe = os.path.join(d, "t")
        subprocess.run(["gcc", "-std=gnu11", "-I" + os.path.join(ROOT, "include"), c, "-o", exe],
                       check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()
    from orchkv_b200 import _lib
    assert [int(x) for x in out] == [C.sizeof(_lib.OrchkvConfig), C.sizeof(_lib.OrchkvStats),
                                     C.sizeof(_lib.KvBlock), C.sizeof(_lib.TmConfig),
                                     C.sizeof(_lib.TmStats), C.sizeof(_lib.TieredManager)]


REFERENCE_BINDING_NAMES = [
    "StorageTier", "DataType", "OK", "ERR_OOM", "ERR_INVALID", "ERR_NOT_FOUND",
    "ERR_TIER_FULL", "ERR_CUDA", "ERR_IO", "Config", "init", "shutdown", "is_initialized",
    "request_create", "request_destroy", "prefill", "get_kv_block", "evict_to_dram",
    "promote_to_gpu", "evict_to_storage", "promote_from_storage", "evict_cold",
    "storage_flush", "get_stats", "tm_create", "tm_destroy", "tm_register_block_id",
    "tm_set_block_tier", "tm_report_attn", "tm_step_done", "tm_set_usage",
    "tm_schedule_once", "tm_get_block_score", "tm_get_block_heat", "tm_start", "tm_stop",
    "tm_set_policy", "tm_get_stats", "GPU_HBM", "HOST_DRAM", "NVM", "SSD", "NONE", "FP16",
    "BF16", "FP32", "INT8", "INT4",
]


def test_orchkv_core_names_and_defaults():
    import orchkv_b200
    m = orchkv_b200.core()
    import orchkv_core
    assert orchkv_core is m
    for n in REFERENCE_BINDING_NAMES:
        assert hasattr(m, n), n
    c = m.Config()
    assert repr(c) == "<orchkv.Config gpu_pool=40960MB dram_pool=65536MB d_head=128>"
    assert c.tokens_per_block == 64 and c.max_blocks_per_head == 256
    assert int(m.GPU_HBM) == 0 and int(m.NONE) == 4 and m.ERR_TIER_FULL == -4
    doc = m.tm_create.__doc__
    for kw, val in [("tracker_cap", "4096"), ("max_blocks", "8192"), ("cooldown_sec", "0.5"),
                    ("recency_tau", "50.0"), ("prefetch_budget", "16"),
                    ("schedule_interval_us", "1000")]:
        assert re.search(kw + r":[^=,]*= " + re.escape(val) + r"\b", doc), kw
    assert re.search(r"tier:[^=,]*= 0\b", m.tm_register_block_id.__doc__)
    assert re.search(r"flags:[^=,]*= 0\b", m.tm_register_block_id.__doc__)


def test_orchkv_core_tensor_level_extensions():
    """The module's additions for device-resident inputs (no counterpart in
    the reference binding): every batched data-plane and report call of the
    C ABI is reachable from Python without ctypes."""
    import orchkv_b200
    m = orchkv_b200.core()
    for n in ["append_token", "append_token_batch", "block_id_table", "block_checksums",
              "evict_batch_to_dram", "promote_batch_to_gpu", "swap_batch", "evict_cold_batch",
              "copy_token_blocks", "attach_scheduler", "set_stream", "sync", "tm_sync",
              "tm_report_attn_probs", "tm_report_attn_ranges", "tm_report_attn_batch_dev",
              "tm_report_attn_blockmean", "tm_stage_input_async", "tm_step_and_classify",
              "tm_select_victims", "tm_select_victims_masked", "tm_select_prefetch"]:
        assert hasattr(m, n), n
    assert re.search(r"tiers_ptr:[^=,]*= 0\b", m.block_checksums.__doc__)
