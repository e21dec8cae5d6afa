"""Whole-row-range streaming on the tensor-core path.

When the batch union covers most of the neurons the tensor-core kernel
stops gathering rows: every neuron becomes a position, W_gate / W_up /
W_down arrive as contiguous 2-D TMA boxes, and the neurons outside a token's
set get h = 0 from the mask.  The test-hook library forces that mode at any
union size (SPB_DEBUG_TC_DENSE_PERMILLE = 1) and forbids it (> 1000), so
both modes are checked against the oracle on the same inputs: labels and
bit words, both activations, union semantics, biases, ragged f, Np up to
256, and the 70B row length."""
import numpy as np
import pytest

from conftest import assert_close, assert_close_70b
from spbatch_b200.workload import zipf_active_labels

pytestmark = pytest.mark.gpu

DENSE_PERMILLE = 9


def _dev(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _bits(lab):
    b = np.packbits((lab > 0).astype(np.uint8), axis=1, bitorder="little")
    b = np.pad(b, ((0, 0), (0, (-b.shape[1]) % 4)))
    return np.ascontiguousarray(b.view(np.int32))


@pytest.fixture
def forced(spb, monkeypatch):
    """Runs spbatch_b200 calls through the test-hook library with the
    whole-row-range threshold set per call."""
    L = spb.debug_lib()
    monkeypatch.setattr(spb, "lib", spb.debug_lib)

    def run(permille, fn):
        assert L.spb_debug_config(DENSE_PERMILLE, permille) == 0
        try:
            return fn()
        finally:
            L.spb_debug_config(DENSE_PERMILLE, 0)
    return run


def _case(spb, cuda, rng, B, d, f, k, act=0, per_token=True, bits=False, bias=False, std=0.02):
    import torch
    W = [(rng.standard_normal((f, d)) * std).astype(np.float16) for _ in range(3)]
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = zipf_active_labels(B, f, k, seed=int(rng.integers(1 << 30)))
    bg = (rng.standard_normal(f) * 0.1).astype(np.float16) if bias else None
    bu = (rng.standard_normal(f) * 0.1).astype(np.float16) if bias else None
    Wd = [_dev(w, cuda) for w in W]
    args = dict(act=act, per_token_mask=per_token, path=spb.PATH_TENSOR)
    if bias:
        args.update(bias_gate=_dev(bg, cuda), bias_up=_dev(bu, cuda))

    def call():
        ws = spb.new_workspace(B, d, f, 0, cuda)
        if bits:
            out = spb.ffn_forward(*Wd, _dev(x, cuda), bits=_dev(_bits(lab), cuda), f=f, workspace=ws, **args)
        else:
            out = spb.ffn_forward(*Wd, _dev(x, cuda), _dev(lab, cuda), workspace=ws, **args)
        torch.cuda.synchronize()
        assert spb.device_error(ws) == 0
        return out.cpu().numpy()
    return W, x, lab, bg, bu, call


@pytest.mark.parametrize("B,d,f,k,act,per_token,bits,bias", [
    (8, 1024, 4096, 400, 0, True, False, False),
    (32, 4096, 11008, 1101, 0, True, False, False),   # 7B, B = 32
    (32, 4096, 11008, 1101, 1, True, True, False),    # bit words, dReLU
    (20, 512, 3000, 300, 0, False, False, False),     # union semantics, ragged f
    (16, 1024, 2016, 200, 0, True, False, True),      # sparse biases
    (256, 256, 1000, 100, 0, True, False, False),     # Np = 256
    (130, 512, 1500, 150, 1, True, True, False),      # Np = 144
])
def test_dense_and_gathered_match_oracle(spb, cuda, oracle_mod, forced, B, d, f, k, act, per_token, bits, bias):
    rng = np.random.default_rng(B * 1000 + f)
    W, x, lab, bg, bu, call = _case(spb, cuda, rng, B, d, f, k, act, per_token, bits, bias)
    if bias:
        want = oracle_mod.ffn_bias(*W, x, lab, bg, bu, act=act, per_token=per_token)
    else:
        want = oracle_mod.ffn(*W, x, lab, act=act, per_token=per_token)
    dense = forced(1, call)
    gathered = forced(1001, call)
    assert_close(dense, want)
    assert_close(gathered, want)


def test_dense_70b_rows(spb, cuda, oracle_mod, forced):
    """d = 8192 rows, f = 28672 / 8 neurons (one tp8 shard), B = 16."""
    rng = np.random.default_rng(70)
    B, d, f = 16, 8192, 3584
    W, x, lab, _, _, call = _case(spb, cuda, rng, B, d, f, 358)
    want = oracle_mod.ffn(*W, x, lab)
    assert_close_70b(forced(1, call), want)


def test_default_threshold_streams_dense_unions(spb, cuda, oracle_mod):
    """The product library at its default threshold: a B = 64 batch at 10%
    activity covers ~99% of the neurons, so whole row ranges stream."""
    import torch
    rng = np.random.default_rng(64)
    B, d, f = 64, 1024, 4096
    W = [(rng.standard_normal((f, d)) * 0.02).astype(np.float16) for _ in range(3)]
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = zipf_active_labels(B, f, 410, seed=64)
    assert (lab > 0).any(0).mean() > 0.9
    out = spb.ffn_forward(*[_dev(w, cuda) for w in W], _dev(x, cuda), _dev(lab, cuda))
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), oracle_mod.ffn(*W, x, lab))
