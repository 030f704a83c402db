"""Multi-rank selection algorithm on CPU ranks (torch.distributed gloo,
world size 2 and 3): the union of every rank's picks equals the single-rank
coldest-k over the concatenated keys, ties broken in (rank, index) order —
the guarantee the NCCL path of the GPU selector gives."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, seed, k, out_q):
    import torch
    import torch.distributed as dist

    from oracle.dist_select import select_local
    from oracle.oracle import orderable
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(seed)
        n = 3000
        all_vals = (rng.integers(0, 40, (world, n)) / 16).astype(np.float32)   # many ties
        all_elig = rng.random((world, n)) < 0.8
        keys = orderable(all_vals[rank])
        keys[~all_elig[rank]] = 0xFFFFFFFF

        def allreduce(a):
            t = torch.tensor(a, dtype=torch.int64)
            dist.all_reduce(t)
            return t.numpy()

        def allgather(x):
            out = [None] * world
            dist.all_gather_object(out, x)
            return out

        picked = select_local(keys, k, allreduce, allgather, rank)
        out_q.put((rank, picked.tolist()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,k,seed", [(2, 1700, 1), (2, 0, 2), (3, 4000, 3), (2, 10 ** 6, 4)])
def test_distributed_select_matches_single_rank(world, k, seed, oracle_mod):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, seed, k, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rng = np.random.default_rng(seed)
    n = 3000
    all_vals = (rng.integers(0, 40, (world, n)) / 16).astype(np.float32)
    all_elig = rng.random((world, n)) < 0.8
    want = oracle_mod.select_coldest(all_vals.reshape(-1), all_elig.reshape(-1).astype(np.uint8), k)
    got = np.sort(np.concatenate([np.array(res[r], np.int64) + r * n for r in range(world)]))
    assert np.array_equal(got, want.astype(np.int64))
