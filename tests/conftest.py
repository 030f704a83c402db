import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "ref: needs the reference compiled into oracle/_ref")


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle as O
    if not os.path.exists(O.ORACLE_SO):
        O.build()
    return O


@pytest.fixture(scope="session")
def cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.init()
    return torch


def pytest_sessionfinish(session, exitstatus):
    """Under the checked build (ORCHKV_CHECKED=1) the session fails if any
    data-plane kernel met an index out of range; the tally is printed."""
    if os.environ.get("ORCHKV_CHECKED") != "1" or "orchkv_b200" not in sys.modules:
        return
    import ctypes as C
    import orchkv_b200
    words = (C.c_uint32 * 4)()
    if orchkv_b200.lib().orchkv_check_status(words, 0) != 0:
        return
    msg = (f"checked build: {words[0]} indices out of range"
           + (f" (first at pool_kernels.cu:{words[1]}, index {words[2]}, bound {words[3]})"
              if words[0] else ""))
    tr = session.config.pluginmanager.get_plugin("terminalreporter")
    if tr is not None:
        tr.write_line(msg)
    else:
        print(msg)
    if words[0]:
        session.exitstatus = 1
