"""Decode loop over a stack of sparse FFN layers (the model-integration row
of the hot path: the end-to-end tok/s that the reference measures through
vLLM / transformers on a Bamboo model, vllm_test.py:8-83,
transformers_test.py:30-82).

Each layer of a decode step does, for the B tokens of the batch:

    a  = rmsnorm(x) @ W_o                 stand-in attention (one dense d x d
    x  = x + a                            projection through torch: the
                                          attention block's output GEMV cost;
                                          no KV cache)
    h  = rmsnorm(x)
    sets = predictor(h)                   DejaVu low-rank predictor, top-k,
                                          as bit words (spb_predict)
    x  = x + sparse_ffn(h, sets)          spb_ffn_forward_bits

The FFN and the predictor run in this library's kernels; the stand-in
attention and the norms are torch operations and are labelled as such.
Every buffer is allocated once, so a whole step can be captured in a CUDA
graph (`capture()`), which is how `tokens_per_second` times it.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import spbatch_b200 as spb


@dataclass
class DecoderShape:
    d: int = 4096
    f: int = 11008
    layers: int = 32
    rank: int = 1024       # predictor rank D
    activity: float = 0.10  # top-k fraction of f per token


class SparseDecoder:
    """A stack of `shape.layers` layers with seeded random weights on one GPU."""

    def __init__(self, shape: DecoderShape, batch: int, device, seed: int = 0, path: int = spb.PATH_AUTO):
        import torch
        self.shape, self.B, self.dev, self.path = shape, batch, device, path
        d, f, D = shape.d, shape.f, shape.rank
        self.k = max(1, int(round(shape.activity * f)))
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        self.layers = []
        for _ in range(shape.layers):
            self.layers.append(dict(
                wo=(torch.randn((d, d), generator=g, device=device) * 0.02).half(),
                wg=(torch.randn((f, d), generator=g, device=device) * 0.02).half(),
                wu=(torch.randn((f, d), generator=g, device=device) * 0.02).half(),
                wd=(torch.randn((f, d), generator=g, device=device) * 0.02).half(),
                p1=(torch.randn((D, d), generator=g, device=device) / math.sqrt(d)).half(),
                p2=(torch.randn((f, D), generator=g, device=device) / math.sqrt(D)).half()))
        self.x = torch.zeros((batch, d), device=device)
        self.h = torch.empty((batch, d), device=device)
        self.ffn_out = torch.empty((batch, d), device=device)
        self.bits = torch.empty((batch, (f + 31) // 32), dtype=torch.int32, device=device)
        self.ws = spb.new_workspace(batch, d, f, 0, device)
        self.pws = spb.predict_workspace(batch, D, f, device)
        self.graph = None

    @staticmethod
    def _rmsnorm(x, out):
        import torch
        torch.mul(x, torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6), out=out)
        return out

    def step(self, x_in=None):
        """One decode step over every layer; returns the [B][d] fp32 state."""
        import torch
        if x_in is not None:
            self.x.copy_(x_in)
        for ly in self.layers:
            a = (self._rmsnorm(self.x, self.h).half() @ ly["wo"]).float()  # stand-in attention
            self.x.add_(a)
            self._rmsnorm(self.x, self.h)
            spb.predict(ly["p1"], ly["p2"], self.h, k=self.k, bits_out=self.bits, labels=False, workspace=self.pws)
            spb.ffn_forward(ly["wg"], ly["wu"], ly["wd"], self.h, bits=self.bits, f=self.shape.f, out=self.ffn_out,
                            workspace=self.ws, path=self.path)
            self.x.add_(self.ffn_out)
        return self.x

    def capture(self):
        """Captures one step (all layers) in a CUDA graph; replay() runs it."""
        import torch
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                self.step()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=s):
            self.step()
        self._gstream = s
        return self.graph

    def tokens_per_second(self, steps: int = 20) -> dict:
        """Decode throughput of the captured step: B tokens per step."""
        import torch
        if self.graph is None:
            self.capture()
        torch.cuda.synchronize()
        self.graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self._gstream)
        with torch.cuda.stream(self._gstream):
            for _ in range(steps):
                self.graph.replay()
        e1.record(self._gstream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        return {"tokens_per_s": self.B / (ms / 1e3), "ms_per_step": ms, "layers": self.shape.layers,
                "batch": self.B, "device_error": spb.device_error(self.ws)}
