"""Multi-rank host logic on CPU: 2 gloo ranks reduce timings; LPT sharding properties."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vf_b200.dist import attention_cost, lpt_shard, reduce_timing


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        ms, fl, tok = reduce_timing(10.0 + rank, 100.0 * (rank + 1), 7.0)
        q.put((rank, ms, fl, tok))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_reduce_timing_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, ms, fl, tok in out:
        assert ms == 11.0 and fl == 300.0 and tok == 14.0


def test_reduce_timing_single_process_is_identity():
    assert reduce_timing(3.0, 5.0, 7.0) == (3.0, 5.0, 7.0)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_lpt_shard_covers_every_sequence_once_and_balances(world):
    g = torch.Generator().manual_seed(world)
    lengths = torch.randint(128, 769, (256,), generator=g).tolist()
    costs = [attention_cost(L) for L in lengths]
    shards = lpt_shard(costs, world)
    flat = sorted(i for s in shards for i in s)
    assert flat == list(range(len(lengths)))
    loads = [sum(costs[i] for i in s) for s in shards]
    # LPT is within 4/3 of optimal; against the average load it is far tighter here
    assert max(loads) <= sum(loads) / world + max(costs)


def test_lpt_shard_rejects_bad_world():
    with pytest.raises(ValueError):
        lpt_shard([1.0], 0)
