"""Neuron-dimension sharding of one sparse FFN layer across GPUs
(the reference is single-GPU).

Rank r of G owns neurons [f0, f1): the same rows of W_gate / W_up / W_down
(all stored [f][d]) and of the predictor's P2.  Each rank runs the
single-GPU kernels on its slice -- its union, gathers and partial down
projection only touch its own rows -- and one all-reduce sums the [B][d] fp32
partial outputs.  There is no other exchange.  On GPUs the all-reduce is the
library's own one-shot kernel over NVLink peer memory (PeerAllReduce,
spb_allreduce_peer); without one, torch.distributed's all_reduce (NCCL on
GPUs, gloo on CPU).
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


class PeerAllReduce:
    """One-shot all-reduce of [B][d] fp32 partials over NVLink peer memory
    (spb_allreduce_peer: each rank pushes its partial into every peer's
    receive slots, then sums locally).  Collective set-up: every rank of
    `group` builds one with the same `max_elems`; it allocates this rank's
    partial buffer, sync words and receive slots, exchanges CUDA IPC handles
    over torch.distributed and maps the peers'.  Then `partial(n)` is the buffer a layer writes its partial
    output into, and `reduce(n, out)` sums the ranks' partials into `out`
    (rank order, bit-identical on every rank).  Every rank makes the same
    calls in the same order; between calls each rank's stream orders the
    layer's kernel before the reduction."""

    def __init__(self, max_elems: int, device, group=None):
        import ctypes as C
        import torch
        import torch.distributed as dist
        import spbatch_b200 as spb
        L = spb.lib()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise spb.SpbError("PeerAllReduce: at most 8 ranks")
        self.max_elems = (max_elems + 3) // 4 * 4
        # one IPC-shared allocation per rank: the sync words (zero-filled),
        # then the receive slots [2][world][max_elems] the peers push into
        head = max(64, int(L.spb_peer_sync_bytes()) // 4)
        self.mem = torch.zeros(head + 2 * self.world * self.max_elems, dtype=torch.float32, device=device)
        self.buf = torch.empty(self.max_elems, dtype=torch.float32, device=device)  # this rank's partial
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        nb = int(L.spb_peer_handle_bytes())
        h = C.create_string_buffer(nb)
        spb._check(L.spb_peer_export(self.mem.data_ptr(), h), "spb_peer_export")
        torch.cuda.synchronize(device)
        allh = [None] * self.world
        dist.all_gather_object(allh, h.raw, group=group)
        self._mapped = []
        recv, syncs = [], []
        for r in range(self.world):
            if r == self.rank:
                base = self.mem.data_ptr()
            else:
                p = C.c_void_p()
                spb._check(L.spb_peer_import(C.create_string_buffer(allh[r], nb), C.byref(p)), "spb_peer_import")
                base = p.value
                self._mapped.append(base)
            syncs.append(base)
            recv.append(base + 4 * head)
        self._recv = (C.c_void_p * self.world)(*recv)
        self._syncs = (C.c_void_p * self.world)(*syncs)
        dist.barrier(group=group)

    def partial(self, n: int):
        if n > self.max_elems:
            raise ValueError("PeerAllReduce: more elements than the buffer holds")
        return self.buf[:n]

    def reduce(self, n: int, out, stream=None) -> None:
        import spbatch_b200 as spb
        spb._check(spb.lib().spb_allreduce_peer(self.buf.data_ptr(), self._recv, self._syncs, self.world, self.rank,
                                                self.max_elems, out.data_ptr(), n, self.err.data_ptr(),
                                                spb._stream(stream)), "spb_allreduce_peer")

    def error(self) -> int:
        """Device error word (1 / 2: a peer never reached barrier in / out)."""
        return int(self.err.item())

    def close(self) -> None:
        import spbatch_b200 as spb
        for p in self._mapped:
            spb.lib().spb_peer_close(p)
        self._mapped = []


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
    peer: PeerAllReduce | None = None  # the all-reduce over peer memory; None: torch.distributed

    def forward(self, x, labels, *, per_token_mask: bool = True, path: int = 0, workspace=None, out=None):
        import torch
        import torch.distributed as dist
        import spbatch_b200 as spb
        if labels.shape[1] == self.f:
            labels = labels[:, self.f0:self.f1].contiguous()
        B, d = x.shape
        if self.peer is not None:
            part = self.peer.partial(B * d).view(B, d)
            spb.ffn_forward(self.w_gate, self.w_up, self.w_down, x, labels, wtype=self.wtype,
                            per_token_mask=per_token_mask, path=path, workspace=workspace, out=part)
            if out is None:
                out = torch.empty((B, d), dtype=torch.float32, device=x.device)
            self.peer.reduce(B * d, out)
            return out
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
