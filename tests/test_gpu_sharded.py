"""Neuron sharding on real GPUs (config 5 path): two ranks, with the
library's one-shot all-reduce over NVLink peer memory (spb_allreduce_peer)
and with the NCCL all-reduce; outputs equal (within tolerance) to the
unsharded oracle layer, and with the peer all-reduce bit-identical on both
ranks and on calls in a row (its epochs advance on the device).  Skipped when
fewer than two GPUs are visible."""
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = r'''
import os, sys
import numpy as np, torch, torch.distributed as dist
sys.path.insert(0, {root!r}); sys.path.insert(0, os.path.join({root!r}, "oracle"))
import oracle, spbatch_b200 as spb
from spbatch_b200.shard import PeerAllReduce, ShardedFFN, shard_weights
from spbatch_b200.workload import zipf_active_labels
rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dev = torch.device("cuda", rank)
dist.init_process_group("nccl", device_id=dev)
rng = np.random.default_rng(7)
d, f = 1024, 4096
W = [(rng.standard_normal((f, d)) * 0.03).astype(np.float16) for _ in range(3)]
peer = PeerAllReduce(24 * d, dev)
f0, f1, part, _ = shard_weights(*[torch.from_numpy(w) for w in W], world, rank, device=dev)
for use_peer in (True, False):
    layer = ShardedFFN(*part, f=f, f0=f0, f1=f1, peer=peer if use_peer else None)
    for B in (2, 24, 24, 5):
        x = rng.standard_normal((B, d)).astype(np.float32)
        lab = zipf_active_labels(B, f, 410, seed=B)
        out = layer.forward(torch.from_numpy(x).to(dev), torch.from_numpy(lab).to(dev))
        torch.cuda.synchronize()
        ref = oracle.ffn(*W, x, lab)
        np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-2, atol=1e-3)
        if use_peer:
            both = [torch.empty_like(out) for _ in range(world)]
            dist.all_gather(both, out)
            assert all(torch.equal(both[0], o) for o in both), "ranks differ"
    assert peer.error() == 0, peer.error()
peer.close()
dist.destroy_process_group()
print("rank", rank, "ok")
'''


def test_two_gpu_sharded_layer(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    script = tmp_path / "worker.py"
    script.write_text(WORKER.format(root=ROOT))
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                        "--master-addr=127.0.0.1", f"--master-port={port}", str(script)],
                       capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("ok") == 2
