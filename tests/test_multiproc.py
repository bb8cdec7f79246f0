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

    out[rank] = bench.reduce_max(float(10 * rank + 3), world)
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

    def evaluate_packed(self, boards, legal, priors, wdl):
        self.seen.append((threading.get_ident(), len(boards)))
        time.sleep(self.delay)
        if self.fail:
            raise RuntimeError(f"replica {self.tag} lost its device")
        priors[:] = np.where(legal >= 0, legal, 0).astype(priors.dtype)
        wdl[:] = 0.0
        wdl[:, 0] = boards[:, 0]
        return priors, wdl

    evaluate_packed_f16 = evaluate_packed

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


@pytest.mark.parametrize("method,dtype", [("evaluate_packed", np.float32), ("evaluate_packed_f16", np.float16)])
def test_sharded_packed_batches_land_in_order(method, dtype):
    """Packed batches: every replica writes its contiguous shard into its own rows of one output
    array (f32 or f16 priors), concurrently; a replica's failure fails the batch as NetworkError."""
    n = 11
    boards = np.zeros((n, 66), np.uint8)
    boards[:, 0] = np.arange(n)
    legal = np.full((n, 224), -1, np.int32)
    legal[:, :3] = np.arange(3 * n).reshape(n, 3)
    reps = [FakeNet(i, delay=0.2) for i in range(3)]
    net = ShardedNetwork(reps)
    t0 = time.perf_counter()
    priors, wdl = getattr(net, method)(boards, legal)
    assert time.perf_counter() - t0 < 0.5  # three 0.2 s shards overlap
    assert priors.dtype == dtype and priors.shape == (n, 224)
    assert np.array_equal(priors[:, :3], legal[:, :3].astype(dtype)) and not priors[:, 3:].any()
    assert np.array_equal(wdl[:, 0], np.arange(n, dtype=np.float32))
    assert [k for r in reps for _, k in r.seen] == [4, 4, 3]
    bad = ShardedNetwork([FakeNet(0), FakeNet(1, fail=True)])
    with pytest.raises(NetworkError, match="replica 1"):
        getattr(bad, method)(boards, legal)
