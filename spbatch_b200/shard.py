"""Neuron-dimension sharding of one sparse FFN layer across GPUs
(the reference is single-GPU).

Rank r of G owns neurons [f0, f1): the same rows of W_gate / W_up / W_down
(all stored [f][d]) and of the predictor's P2.  Each rank runs the
single-GPU kernels on its slice -- its union, gathers and partial down
projection only touch its own rows -- and one all-reduce (NCCL over NVLink
on GPUs) sums the [B][d] fp32 partial outputs.  There is no other exchange.
"""
from __future__ import annotations

from dataclasses import dataclass


def shard_range(f: int, world: int, rank: int, align: int = 32) -> tuple[int, int]:
    """Contiguous neuron range of `rank`; boundaries fall on multiples of
    `align` (a 32-neuron activity word) so no word is split between ranks."""
    if not (0 <= rank < world):
        raise ValueError("rank out of range")
    words = (f + align - 1) // align
    w0 = words * rank // world
    w1 = words * (rank + 1) // world
    return min(f, w0 * align), min(f, w1 * align)


@dataclass
class ShardedFFN:
    """One FFN layer's slice on this rank.

    w_gate / w_up / w_down: this rank's rows [f1 - f0][d] on its GPU (fp16, or
    Q8_0 / Q4_0 rows with wtype set).  forward() takes the full-width labels
    (or this shard's columns) and returns the all-reduced [B][d] output.
    """
    w_gate: object
    w_up: object
    w_down: object
    f: int
    f0: int
    f1: int
    wtype: int = 0
    group: object = None

    def forward(self, x, labels, *, per_token_mask: bool = True, path: int = 0, workspace=None, out=None):
        import torch
        import torch.distributed as dist
        import spbatch_b200 as spb
        if labels.shape[1] == self.f:
            labels = labels[:, self.f0:self.f1].contiguous()
        out = spb.ffn_forward(self.w_gate, self.w_up, self.w_down, x, labels, wtype=self.wtype,
                              per_token_mask=per_token_mask, path=path, workspace=workspace, out=out)
        if dist.is_available() and dist.is_initialized() and dist.get_world_size(self.group) > 1:
            dist.all_reduce(out, op=dist.ReduceOp.SUM, group=self.group)
        return out


def shard_weights(w_gate, w_up, w_down, world: int, rank: int, device=None, p2=None):
    """Slices full [f][d] weight rows (and optionally P2 [f][D]) for `rank`."""
    f = w_gate.shape[0]
    f0, f1 = shard_range(f, world, rank)
    part = [w[f0:f1].contiguous() for w in (w_gate, w_up, w_down)]
    if device is not None:
        part = [p.to(device) for p in part]
    extra = None
    if p2 is not None:
        extra = p2[f0:f1].contiguous()
        if device is not None:
            extra = extra.to(device)
    return f0, f1, part, extra
