"""Multi-GPU selection through NCCL (two-rank cases need >= 2 GPUs and are
skipped otherwise; the one-rank case runs on any GPU box).

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
        ms, calls = C.c_float(), C.c_uint32()
        assert L.orchkv_comm_exchange_time(comm, C.byref(ms), C.byref(calls)) == 0
        q.put((rank, picks, st["hot"][:N_PER_RANK].tolist(), calls.value))
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
        r, picks, hot, _ = q.get(timeout=300)
        res[r] = (picks, hot)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    hot = np.concatenate([np.array(res[r][1], np.float32) for r in range(world)])
    want = oracle_mod.select_coldest(hot, np.ones(len(hot), np.uint8), k)
    got = np.sort(np.concatenate([np.array(res[r][0], np.int64) + r * N_PER_RANK
                                  for r in range(world)]))
    assert np.array_equal(got, want.astype(np.int64))


@pytest.mark.parametrize("k", [7000, 1])
def test_global_coldest_k_one_rank_communicator(cuda, oracle_mod, k):
    """The same selection through a one-rank NCCL communicator, on any box
    with a GPU: the histogram all-reduces and the tie all-gather of comm.cu
    run, and the picks equal the oracle's coldest k of the rank's scores."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_worker, args=(0, 1, _free_port(), k, q))
    p.start()
    r, picks, hot, exchanges = q.get(timeout=300)
    p.join(timeout=120)
    assert p.exitcode == 0 and r == 0
    assert exchanges >= 4              # three histogram all-reduces and the tie all-gather
    hot = np.array(hot, np.float32)
    want = oracle_mod.select_coldest(hot, np.ones(len(hot), np.uint8), k)
    assert np.array_equal(np.sort(np.array(picks, np.int64)), want.astype(np.int64))


def _sharded_worker(rank, world, port, q):
    """One rank of bench.py's KV-head-sharded pool, cut to one request (the
    Llama-3-8B shape: 32 layers, 8/world KV heads here, 32,768 tokens, fp16,
    64-token blocks): one checked step, the victims' bytes before and after."""
    import ctypes as C

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    import bench
    import orchkv_b200 as okv
    from tests.test_gpu_fullsize import _dram_total, dev_checksums, host_checksums
    L = okv.lib()
    try:
        uid = (C.c_ubyte * 128)()
        if rank == 0:
            assert L.orchkv_comm_unique_id(uid) == 0
        obj = [bytes(uid)]
        dist.broadcast_object_list(obj, 0)
        comm = L.orchkv_comm_create(rank, world, (C.c_ubyte * 128)(*obj[0]), 60.0)
        assert comm
        stream = torch.cuda.Stream()
        torch.cuda.set_stream(stream)
        sw = bench.ShardedWorkload(torch, okv, rank, world, comm, requests=1)
        seen = {}

        def check():
            seen["view"] = sw.selection_view()
            picks = torch.as_tensor(seen["view"][2].astype(np.int32), device="cuda")
            seen["ids"] = picks
            seen["before"], _ = dev_checksums(torch, L, picks)

        sw.step(check=check)
        torch.cuda.synchronize()
        n_ev = sw.h_counts.tolist()[2]                 # the evict's result, words 2-3
        loc = np.zeros(sw.cap, np.uint32)
        assert L.orchkv_read_block_locs(loc.ctypes.data, None) == 0
        picks = seen["view"][2]
        on_dram = bool(((loc[picks] >> 29) == 1).all())
        dram = host_checksums(L.orchkv_dram_pool_base(), sw.slab, _dram_total(L),
                              loc[picks].astype(np.int64) & 0x1FFFFFFF)
        sw.restore()
        back, _ = dev_checksums(torch, L, seen["ids"])
        ok = (on_dram and n_ev == len(picks) and np.array_equal(dram, seen["before"])
              and np.array_equal(back, seen["before"]))
        hot, elig, _ = seen["view"]
        q.put((rank, hot, elig, picks, ok, sw.k_global, sw.cap))
        sw.close()
        L.orchkv_comm_destroy(comm)
    finally:
        dist.destroy_process_group()


def test_sharded_pool_step_two_gpus(cuda, oracle_mod):
    """bench.py's sharded step on two GPUs: each rank holds 4 of the 8 KV
    heads; the ranks' picks together are the oracle's global coldest 60% of
    both ranks' blocks (ties in (rank, slot) order), and every picked block's
    bytes reach the rank's DRAM tier and come back unchanged."""
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, hot, elig, picks, ok, k, cap = q.get(timeout=600)
        res[r] = (hot, elig, picks, ok, k, cap)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(res[r][3] for r in range(world)), "victim bytes differ after the round trip"
    k, cap = res[0][4], res[0][5]
    hot = np.concatenate([res[r][0] for r in range(world)])
    elig = np.concatenate([res[r][1] for r in range(world)]).astype(np.uint8)
    want = oracle_mod.select_coldest(hot, elig, k).astype(np.int64)
    got = np.sort(np.concatenate([res[r][2] + r * cap for r in range(world)]))
    assert len(got) == k
    assert np.array_equal(got, want)
