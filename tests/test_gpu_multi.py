"""Multi-GPU selection through NCCL (needs >= 2 GPUs; skipped otherwise).

Each rank owns one shard of blocks (KV-head sharding) with its own manager;
with a communicator set, tm_select_victims(k) selects the global coldest k:
the union of the ranks' picks must equal the single-rank oracle over all
ranks' hotness, ties in (rank, block id) order.  NVLS is disabled for the test
processes.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N_PER_RANK = 20000


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, k, q):
    import ctypes as C

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    import orchkv_b200 as okv
    L = okv.lib()
    try:
        uid = (C.c_ubyte * 128)()
        if rank == 0:
            assert L.orchkv_comm_unique_id(uid) == 0
        obj = [bytes(uid)]
        dist.broadcast_object_list(obj, 0)
        uid = (C.c_ubyte * 128)(*obj[0])
        comm = L.orchkv_comm_create(rank, world, uid, 60.0)
        assert comm
        m = okv.Manager(tracker_cap=N_PER_RANK, max_blocks=1 << 20)
        for i in range(N_PER_RANK):
            m.register_id(i, 0, 0)
        rng = np.random.default_rng(100 + rank)
        ids = rng.choice(N_PER_RANK, N_PER_RANK // 2, replace=False).astype(np.uint32)
        w = (rng.integers(0, 6, len(ids)) / 8).astype(np.float32)     # many ties
        di = torch.from_numpy(ids.view(np.int32)).cuda()
        dw = torch.from_numpy(w).cuda()
        assert L.tm_report_attn_batch_dev(m.ref, di.data_ptr(), dw.data_ptr(), len(ids)) == 0
        assert L.tm_step_and_classify(m.ref) == 0
        assert L.tm_set_comm(m.ref, comm) == 0
        out = torch.zeros(N_PER_RANK, dtype=torch.int32, device="cuda")
        cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
        assert L.tm_select_victims(m.ref, k, out.data_ptr(), cnt.data_ptr()) == 0
        assert L.tm_sync(m.ref) == 0
        c = int(cnt.item())
        picks = out[:c].cpu().numpy().tolist()
        st = m.state()
        q.put((rank, picks, st["hot"][:N_PER_RANK].tolist()))
        L.tm_set_comm(m.ref, None)
        m.close()
        L.orchkv_comm_destroy(comm)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("k", [7000, 1, 19999])
def test_global_coldest_k_two_gpus(cuda, oracle_mod, k):
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, k, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, picks, hot = q.get(timeout=300)
        res[r] = (picks, hot)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    hot = np.concatenate([np.array(res[r][1], np.float32) for r in range(world)])
    want = oracle_mod.select_coldest(hot, np.ones(len(hot), np.uint8), k)
    got = np.sort(np.concatenate([np.array(res[r][0], np.int64) + r * N_PER_RANK
                                  for r in range(world)]))
    assert np.array_equal(got, want.astype(np.int64))
