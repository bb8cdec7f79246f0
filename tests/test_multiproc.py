"""Host-side logic of the multi-GPU path, without a GPU: the benchmark's max-over-ranks
timing reduction on a 2-rank gloo process group, and the sharding of a batch across replicas
(order, shard sizes, error propagation) with fake per-GPU networks."""

import os
import socket
import threading
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

from marina_b200.network import Evaluation, Network, NetworkError, ShardedNetwork


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import bench

    out[rank] = bench.reduce_max(float(10 * rank + 3), world, torch.device("cpu"))
    dist.barrier()
    dist.destroy_process_group()


def test_reduce_max_over_two_gloo_ranks():
    port = _free_port()
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    out = manager.dict()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out)) for r in range(2)]
    [p.start() for p in procs]
    [p.join(120) for p in procs]
    assert all(p.exitcode == 0 for p in procs)
    assert dict(out) == {0: 13.0, 1: 13.0}


class FakeNet(Network):
    """Deterministic priors from the action indices; records which thread evaluated it."""

    def __init__(self, tag, fail=False, delay=0.0):
        self.tag, self.fail, self.delay, self.seen = tag, fail, delay, []

    def evaluate(self, batch):
        self.seen.append((threading.get_ident(), len(batch)))
        time.sleep(self.delay)
        if self.fail:
            raise NetworkError(f"replica {self.tag} lost its device", 6)
        return [Evaluation(np.asarray(acts, np.float32) / max(1, sum(acts)), (float(board[0]), 0.0, 0.0))
                for board, acts in batch]

    def describe(self):
        return f"fake {self.tag}"


def _leaves(n):
    return [(np.array([i] + [0] * 65, np.uint8), [i + 1, i + 2]) for i in range(n)]


def test_shards_are_contiguous_and_balanced():
    assert ShardedNetwork.shards(10, 4) == [(0, 3), (3, 6), (6, 8), (8, 10)]
    assert ShardedNetwork.shards(2, 4) == [(0, 1), (1, 2), (2, 2), (2, 2)]
    assert ShardedNetwork.shards(0, 3) == [(0, 0), (0, 0), (0, 0)]


def test_sharded_network_keeps_order_and_runs_replicas_concurrently():
    reps = [FakeNet(i, delay=0.2) for i in range(4)]
    net = ShardedNetwork(reps)
    t0 = time.perf_counter()
    out = net.evaluate(_leaves(10))
    assert time.perf_counter() - t0 < 0.6  # four 0.2 s shards overlap
    assert [e.wdl[0] for e in out] == list(range(10))
    assert [n for r in reps for _, n in r.seen] == [3, 3, 2, 2]
    assert len({tid for r in reps for tid, _ in r.seen}) == 4
    assert "fake 0" in net.describe()


def test_a_failing_replica_fails_the_batch():
    net = ShardedNetwork([FakeNet(0), FakeNet(1, fail=True)])
    with pytest.raises(NetworkError, match="replica 1"):
        net.evaluate(_leaves(5))
    # the healthy configuration still works afterwards
    assert len(ShardedNetwork([FakeNet(0), FakeNet(1)]).evaluate(_leaves(5))) == 5
