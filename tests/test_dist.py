"""CPU: data-parallel prompt sharding (LPT bin-packing, micro-batching) and the gather of results across
ranks, with two gloo ranks as separate processes."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sa3_b200 import dist as sdist


def test_band_pairs_matches_bruteforce():
    for n in (1, 17, 300, 513, 600, 2000, 5000):
        i = np.arange(n)[:, None]
        j = np.arange(n)[None, :]
        brute = int(((j - i >= -256) & (j - i <= 256)).sum())
        assert sdist.band_pairs(n) == brute, n


def test_lpt_shard_covers_all_and_balances():
    rng = np.random.default_rng(0)
    lengths = rng.integers(108, 8184, size=256)
    costs = [sdist.prompt_cost(int(n)) for n in lengths]
    for world in (1, 2, 4, 8):
        bins = sdist.lpt_shard(costs, world)
        flat = sorted(i for b in bins for i in b)
        assert flat == list(range(256))
        loads = [sum(costs[i] for i in b) for b in bins]
        # LPT guarantee: max load <= 4/3 OPT; with many small items it is within a few percent of the mean
        assert max(loads) <= 1.05 * (sum(loads) / world) + max(costs)
    assert sdist.lpt_shard(costs, 4) == sdist.lpt_shard(costs, 4)  # deterministic


def test_micro_batches_respect_token_budget():
    lengths = [1000, 5000, 200, 8000, 300, 50]
    mbs = sdist.micro_batches(range(6), lengths, max_tokens=20000)
    assert [i for mb in mbs for i in mb] == list(range(6))
    for mb in mbs:
        rows = sum(2 * (lengths[i] + 64) for i in mb)
        assert rows <= 20000 or len(mb) == 1


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, lengths, outq):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # a stand-in step: each prompt's "result" encodes its index and length
        def step(mb):
            return [torch.full((2,), float(i)) + lengths[i] * 1000 for i in mb]

        shard, res = sdist.run_data_parallel(step, lengths, world, rank, max_tokens=30000)
        allres = sdist.gather_results(shard, res, len(lengths))
        outq.put((rank, shard, [r.tolist() for r in allres]))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_gather():
    rng = np.random.default_rng(1)
    lengths = [int(x) for x in rng.integers(108, 8184, size=23)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, lengths, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    shards = {r: s for r, s, _ in got}
    assert sorted(shards[0] + shards[1]) == list(range(23)) and not set(shards[0]) & set(shards[1])
    for _, _, allres in got:
        for i, r in enumerate(allres):
            assert r == [float(i) + lengths[i] * 1000] * 2
