"""Decode loop over a layer stack (spbatch_b200.decode): one step through
this library's predictor and FFN matches the same step restated with the CPU
oracle for the FFN (and torch for the stand-in attention and norms), layer
by layer; the graph-captured step reproduces the eager one."""
import numpy as np
import pytest

from conftest import assert_close

pytestmark = pytest.mark.gpu


def test_decode_step_matches_oracle(spb, cuda, oracle_mod):
    import torch
    from spbatch_b200.decode import DecoderShape, SparseDecoder
    shape = DecoderShape(d=512, f=1024, layers=3, rank=256, activity=0.1)
    B = 4
    dec = SparseDecoder(shape, B, cuda, seed=3)
    x0 = torch.randn((B, shape.d), device=cuda)
    got = dec.step(x0).clone()
    torch.cuda.synchronize()
    assert spb.device_error(dec.ws) == 0
    # restate the step on the host: torch for the stand-in parts, the oracle
    # for predictor sets and the sparse FFN
    x = x0.cpu().double()
    for ly in dec.layers:
        def rms(v):
            return v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + 1e-6)
        a = (rms(x).float().half().double() @ ly["wo"].cpu().double()).float().double()
        x = x + a
        h = rms(x).float()
        p1, p2 = ly["p1"].cpu().numpy(), ly["p2"].cpu().numpy()
        _, lab, _, _ = oracle_mod.predict(p1, p2, h.numpy(), k=dec.k)
        ffn = oracle_mod.ffn(ly["wg"].cpu().numpy(), ly["wu"].cpu().numpy(), ly["wd"].cpu().numpy(), h.numpy(), lab)
        x = x + torch.from_numpy(ffn).double()
    assert_close(got.cpu().numpy(), x.float().numpy(), rtol=2e-2, atol=2e-2)


def test_decode_graph_replay_matches_eager(spb, cuda):
    import torch
    from spbatch_b200.decode import DecoderShape, SparseDecoder
    shape = DecoderShape(d=512, f=1024, layers=2, rank=256, activity=0.1)
    dec = SparseDecoder(shape, 8, cuda, seed=4)
    x0 = torch.randn((8, shape.d), device=cuda)
    want = dec.step(x0).clone()
    dec.capture()
    dec.x.copy_(x0)
    dec.graph.replay()
    torch.cuda.synchronize()
    # the FFN's output reductions may add in another order between runs
    assert_close(dec.x.cpu().numpy(), want.cpu().numpy(), rtol=1e-5, atol=1e-5)
    r = dec.tokens_per_second(steps=5)
    assert r["tokens_per_s"] > 0 and r["device_error"] == 0
