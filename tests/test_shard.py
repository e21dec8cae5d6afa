"""Host logic of neuron sharding, with two gloo ranks on the CPU: shard
ranges tile the neuron dimension on word boundaries, and summing the
per-shard oracle outputs with an all-reduce reproduces the unsharded layer."""
import os

import numpy as np
import pytest

from spbatch_b200.shard import shard_range


@pytest.mark.parametrize("f", [32, 1000, 11008, 28672])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shard_ranges_tile_f(f, world):
    edges = [shard_range(f, world, r) for r in range(world)]
    assert edges[0][0] == 0 and edges[-1][1] == f
    for (a0, a1), (b0, b1) in zip(edges, edges[1:]):
        assert a1 == b0 and a0 <= a1
    assert all(e[0] % 32 == 0 for e in edges)


def _worker(rank, world, port, q):
    import sys
    import torch
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "oracle"))
    import oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(5)
    B, d, f = 3, 64, 200
    W = [(rng.standard_normal((f, d)) * 0.1).astype(np.float16) for _ in range(3)]
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = (rng.random((B, f)) < 0.2).astype(np.float32)
    f0, f1 = shard_range(f, world, rank)
    part = oracle.ffn(*[w[f0:f1] for w in W], x, lab[:, f0:f1])
    t = torch.from_numpy(part)
    dist.all_reduce(t)
    full = oracle.ffn(*W, x, lab)
    q.put((rank, float(np.abs(t.numpy() - full).max())))
    dist.destroy_process_group()


def test_two_rank_allreduce_reproduces_layer():
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(err < 1e-4 for _, err in res), res
