"""tm_stage_input_async: a report's host input uploaded ahead of the call.

A caller whose attention probabilities arrive in host memory can start their
upload while the GPU does other work (the bench starts the next step's
upload while the current step's swap runs); the report given the same host
range then reads the uploaded copy.  Checked: the staged report equals a
report from device memory bit for bit; it reads the copy taken at staging
time (the host buffer is overwritten afterwards on purpose to tell the two
apart); two staged uploads are consumed oldest first; a third while two wait
is refused, and NULL drops them."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _state_sum(m):
    return m.state()["sum"].copy()


def test_staged_probabilities(cuda):
    import orchkv_b200 as okv
    torch = cuda
    L = okv.lib()
    R, Hq, Hkv, T, tpb = 4, 8, 2, 1024, 16
    nb = T // tpb
    g = torch.Generator(device="cuda").manual_seed(9)
    dev = [torch.softmax(torch.randn(R, Hq, T, generator=g, device="cuda") * 2, -1)
           for _ in range(3)]
    host = [d.cpu().pin_memory() for d in dev]
    ids = torch.arange(R * Hkv * nb, dtype=torch.int32, device="cuda")
    nbytes = R * Hq * T * 4

    def manager():
        m = okv.Manager(tracker_cap=R * Hkv * nb, max_blocks=1 << 16)
        for i in range(R * Hkv * nb):
            m.register_id(i)
        return m

    def report(m, probs_ptr):
        assert L.tm_report_attn_probs(m.ref, C.c_void_p(probs_ptr), R, Hq, Hkv, T, tpb, None,
                                      C.c_void_p(ids.data_ptr())) == 0

    want = []
    for d in dev:
        m = manager()
        report(m, d.data_ptr())
        want.append(_state_sum(m))
        m.close()

    m = manager()
    try:
        # staged, then reported from the same host range: equals the device report
        assert L.tm_stage_input_async(m.ref, C.c_void_p(host[0].data_ptr()), nbytes) == 0
        report(m, host[0].data_ptr())
        got = _state_sum(m)
        assert np.array_equal(got.view(np.uint32), want[0].view(np.uint32))
        m.step_done()

        # two uploads of one buffer wait at once; the first report takes the
        # older one -- whose bytes predate the overwrite below
        assert L.tm_stage_input_async(m.ref, C.c_void_p(host[1].data_ptr()), nbytes) == 0
        assert L.tm_sync(m.ref) == 0
        torch.cuda.synchronize()
        host[1].copy_(host[2])                           # the host bytes change after upload 1
        assert L.tm_stage_input_async(m.ref, C.c_void_p(host[1].data_ptr()), nbytes) == 0
        assert L.tm_stage_input_async(m.ref, C.c_void_p(host[0].data_ptr()), nbytes) == -8          # ORCHKV_ERR_STATE
        report(m, host[1].data_ptr())                    # reads upload 1 (dev[1]'s values)
        assert np.array_equal(_state_sum(m).view(np.uint32), want[1].view(np.uint32))
        m.step_done()
        report(m, host[1].data_ptr())                    # reads upload 2 (dev[2]'s values)
        assert np.array_equal(_state_sum(m).view(np.uint32), want[2].view(np.uint32))
        m.step_done()

        # nothing waits now: a plain host report copies on the spot
        host[1].copy_(dev[0].cpu())
        report(m, host[1].data_ptr())
        assert np.array_equal(_state_sum(m).view(np.uint32), want[0].view(np.uint32))
        m.step_done()

        # NULL drops a waiting upload; the next report copies on the spot
        assert L.tm_stage_input_async(m.ref, C.c_void_p(host[2].data_ptr()), nbytes) == 0
        assert L.tm_stage_input_async(m.ref, None, 0) == 0
        torch.cuda.synchronize()
        host[2].copy_(dev[0].cpu())
        report(m, host[2].data_ptr())
        assert np.array_equal(_state_sum(m).view(np.uint32), want[0].view(np.uint32))
        # device memory is refused (it is read in place anyway)
        assert L.tm_stage_input_async(m.ref, C.c_void_p(dev[0].data_ptr()), nbytes) == -2
    finally:
        m.close()
