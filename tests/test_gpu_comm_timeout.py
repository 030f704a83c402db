"""Failure detection for the multi-GPU selection, made on the host: a rank
that never joins.  Rank 0 of a two-rank communicator is created alone; the
non-blocking NCCL init must give up at its deadline (the communicator is
aborted, orchkv_comm_create returns NULL) instead of waiting for ever.  No
kernel is launched and no GPU waits on anything.  Runs in a child process
with NVLS off, so NCCL state cannot leak into other tests."""
import os
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = textwrap.dedent("""
    import ctypes as C, sys, time
    sys.path.insert(0, %r)
    import torch
    torch.cuda.set_device(0)
    import orchkv_b200 as o
    L = o.lib()
    uid = (C.c_ubyte * 128)()
    assert L.orchkv_comm_unique_id(uid) == 0
    t0 = time.monotonic()
    h = L.orchkv_comm_create(0, 2, uid, 3.0)        # rank 1 never comes
    dt = time.monotonic() - t0
    print("handle", h, "seconds", round(dt, 2))
    sys.exit(0 if (not h and 2.5 <= dt <= 30.0) else 1)
""") % ROOT


def test_comm_create_gives_up_when_a_rank_never_joins(cuda):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-c", CHILD], env=env, capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "aborting communicator" in r.stderr
