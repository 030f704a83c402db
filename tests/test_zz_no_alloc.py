"""The allocation-free selection entry point (orchkv_select_coldest_noalloc)
against the regular one (tm_select_victims).

Callers that cannot call cudaMalloc while running — engines that hand all
device memory to their own allocator at start-up, or paths that must not
take the CUDA allocator's locks — use the variant whose scratch is a static
device array.  Called through the C ABI twice in a row, it must return the
same block ids as tm_select_victims on the same scores (exact: integer ids,
no tolerance), and it must refuse inputs larger than its static capacity.
This file is collected last so a stop-at-first-failure run has already run
every other test.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_N = 1 << 20


def test_noalloc_selection_matches_regular_entry_point(cuda):
    import orchkv_b200 as okv
    torch = cuda
    L = okv.lib()
    rng = np.random.default_rng(12)
    n = 60000
    m = okv.Manager(tracker_cap=n, max_blocks=1 << 20)
    try:
        for i in range(n):
            assert m.register_id(i, 0, 0) == 0
        ids = rng.choice(n, n // 2, replace=False).astype(np.uint32)
        w = (rng.integers(0, 9, len(ids)) / 8).astype(np.float32)   # many exact ties
        d_ids = torch.from_numpy(ids.view(np.int32)).cuda()
        d_w = torch.from_numpy(w).cuda()
        assert L.tm_report_attn_batch_dev(m.ref, d_ids.data_ptr(), d_w.data_ptr(), len(ids)) == 0
        assert L.tm_step_and_classify(m.ref) == 0
        st = m.state()
        cap = m.cap
        # every registered block is on the GPU with no flags: eligible = active
        eligible = (st["c_active"] & st["t_active"]).astype(np.uint8)
        d_hot = torch.from_numpy(st["hot"]).cuda()
        d_el = torch.from_numpy(eligible).cuda()
        torch.cuda.synchronize()
        for k in (15001, 4321):                      # two calls in a row
            ref_out = torch.zeros(k, dtype=torch.int32, device="cuda")
            ref_cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
            assert L.tm_select_victims(m.ref, k, ref_out.data_ptr(), ref_cnt.data_ptr()) == 0
            assert L.tm_sync(m.ref) == 0
            out = torch.full((k,), -1, dtype=torch.int32, device="cuda")
            cnt = torch.full((1,), -1, dtype=torch.int32, device="cuda")
            rc = L.orchkv_select_coldest_noalloc(d_hot.data_ptr(), d_el.data_ptr(), cap, k,
                                                 out.data_ptr(), cnt.data_ptr(), None)
            assert rc == 0
            torch.cuda.synchronize()
            c = int(cnt.item())
            assert c == int(ref_cnt.item()) == k
            assert torch.equal(out[:c], ref_out[:c])
    finally:
        m.close()


def test_noalloc_selection_rejects_oversize(cuda):
    import orchkv_b200 as okv
    L = okv.lib()
    x = cuda.zeros(8, dtype=cuda.float32, device="cuda")
    rc = L.orchkv_select_coldest_noalloc(x.data_ptr(), x.data_ptr(), MAX_N + 1, 4,
                                         x.data_ptr(), x.data_ptr(), None)
    assert rc == -2                                   # ORCHKV_ERR_INVALID


@pytest.mark.parametrize("n", [4097, 70001, MAX_N])
def test_noalloc_selection_sizes(cuda, oracle_mod, n):
    """A partial last 4,096-key tile (4,097 and 70,001 values) and the
    documented maximum (1,048,576, every tile of the static scratch in use):
    the picks equal the oracle's coldest-k over the same values -- ties
    (values on a 1/8 grid) in ascending index order -- on calls in a row
    with different k, the last taking every eligible value."""
    import orchkv_b200 as okv
    torch = cuda
    L = okv.lib()
    rng = np.random.default_rng(n)
    vals = (rng.integers(0, 64, n) / 8).astype(np.float32)
    elig = (rng.random(n) < 0.9).astype(np.uint8)
    d_v = torch.from_numpy(vals).cuda()
    d_e = torch.from_numpy(elig).cuda()
    out = torch.full((n,), -1, dtype=torch.int32, device="cuda")
    cnt = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    for k in (1, n // 3, n):
        rc = L.orchkv_select_coldest_noalloc(d_v.data_ptr(), d_e.data_ptr(), n, k,
                                             out.data_ptr(), cnt.data_ptr(), None)
        assert rc == 0
        torch.cuda.synchronize()
        want = oracle_mod.select_coldest(vals, elig, k)
        c = int(cnt.item())
        assert c == len(want) == min(k, int(elig.sum()))
        assert np.array_equal(out[:c].cpu().numpy().view(np.uint32), want)
