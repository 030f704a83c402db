"""The bounds-checked build: every slab, free-stack and block index a
data-plane kernel reads from memory is compared with its bound, an index out
of range is recorded and its access skipped (nothing traps), and
orchkv_sync / tm_sync report it.

The data-plane GPU suites run once more in a child process on that build
(ORCHKV_CHECKED=1 selects orchkv_b200/_checked/): the small shapes, and the
bench's own step at full size (1,835,008 slabs, 14-chunk evicts through the
whole-evict staging and through the wrapping three-slot rings); the session
ends by reading the check words and fails if any index was out of range.  The check words'
plumbing is tested by a recorded violation that touches no other memory
(orchkv_check_inject): orchkv_sync and tm_sync then return ORCHKV_ERR_CUDA
until the tally is reset."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CHECKED_LIB = os.path.join(ROOT, "orchkv_b200", "_checked", "liborchkv_b200.so")
CHECKED_SUITES = ["tests/test_gpu_pool.py", "tests/test_gpu_staged_evict.py",
               "tests/test_gpu_staged_promote_swap.py", "tests/test_gpu_storage.py",
               "tests/test_gpu_sched.py", "tests/test_gpu_c4_callbacks.py",
               "tests/test_gpu_cpu_step_e2e.py", "tests/test_gpu_workloads.py",
               "tests/test_gpu_core_module.py", "tests/test_gpu_fast_manager.py",
               "tests/test_gpu_kvcache_manager.py", "tests/test_gpu_report_aliasing.py",
               "tests/test_gpu_staged_input.py", "tests/test_gpu_fullsize.py"]

PLUMBING = r'''
import ctypes as C
import orchkv_b200 as okv
L = okv.lib()
assert L.orchkv_checked_build() == 1
slab = 16 * 128 * 2 * 2
cfg = okv.make_config(gpu_pool_bytes=64 * slab, dram_pool_bytes=64 * slab, tokens_per_block=16,
                      d_head=128, dtype=1, max_blocks_per_head=16)
ext = okv.OrchkvConfigExt()
ext.max_blocks = 256
assert L.orchkv_init_ext(C.byref(cfg), C.byref(ext)) == 0
m = okv.Manager(tracker_cap=256)
assert L.orchkv_attach_scheduler(m.ref) == 0
w = (C.c_uint32 * 4)()
assert L.orchkv_check_status(w, 0) == 0 and list(w) == [0, 0, 0, 0]
assert L.orchkv_sync() == 0 and L.tm_sync(m.ref) == 0
assert L.orchkv_check_inject(4321) == 0
assert L.orchkv_sync() == -5 and L.tm_sync(m.ref) == -5        # ORCHKV_ERR_CUDA
assert L.orchkv_check_status(w, 1) == 0 and list(w) == [1, 4321, 1, 0]
assert L.orchkv_sync() == 0 and L.tm_sync(m.ref) == 0
m.close()
assert L.orchkv_shutdown() == 0
print("plumbing ok")
'''


def _child(args, timeout):
    env = dict(os.environ, ORCHKV_CHECKED="1")
    return subprocess.run([sys.executable] + args, cwd=ROOT, env=env, capture_output=True,
                          text=True, timeout=timeout)


def test_check_words_plumbing(cuda):
    if not os.path.exists(CHECKED_LIB):
        pytest.fail("the checked build is missing: python -m orchkv_b200.build --checked")
    r = _child(["-c", PLUMBING], 300)
    assert r.returncode == 0 and "plumbing ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


def test_data_plane_suites_on_checked_build(cuda):
    if not os.path.exists(CHECKED_LIB):
        pytest.fail("the checked build is missing: python -m orchkv_b200.build --checked")
    r = _child(["-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider"] + CHECKED_SUITES,
               1500)
    tail = r.stdout[-3000:] + r.stderr[-2000:]
    assert r.returncode == 0, tail
    assert "checked build: 0 indices out of range" in r.stdout, tail
