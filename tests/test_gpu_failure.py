"""Failure path of the tensor-core kernel, made on purpose without faulting
the GPU: the test-hook library (include/spb_debug.h) shortens the bounded
waits to 1 ms and stops one CTA of every pair from signalling its partner.
The partner's wait runs out, the kernel records error code 4 in the
workspace and returns; the context stays usable and the next call, with the
hooks off, gives the oracle's answer."""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_close
from spbatch_b200.workload import zipf_active_labels

pytestmark = pytest.mark.gpu

TIMEOUT_NS, INJECT = 1, 2
ERR_XCHG, ERR_H = 4, 5


def _call(L, W, x, lab, out, ws, stream):
    B, d = x.shape
    f = lab.shape[1]
    return L.spb_ffn_forward(W[0].data_ptr(), W[1].data_ptr(), W[2].data_ptr(), 0, x.data_ptr(), lab.data_ptr(),
                             B, d, f, 0, 1, 2, out.data_ptr(), None, None, ws.data_ptr(), ws.numel(), stream)


def test_exchange_wait_runs_out_and_recovers(spb, cuda, oracle_mod):
    import torch
    L = spb.debug_lib()
    rng = np.random.default_rng(5)
    B, d, f = 16, 1024, 4096
    Wh = [(rng.standard_normal((f, d)) * 0.03).astype(np.float16) for _ in range(3)]
    W = [torch.from_numpy(w).to(cuda) for w in Wh]
    x_h = rng.standard_normal((B, d)).astype(np.float32)
    lab_h = zipf_active_labels(B, f, 400, seed=5)
    x, lab = torch.from_numpy(x_h).to(cuda), torch.from_numpy(lab_h).to(cuda)
    out = torch.empty((B, d), device=cuda)
    ws = spb.new_workspace(B, d, f, 0, cuda)
    stream = torch.cuda.current_stream().cuda_stream
    try:
        assert L.spb_debug_config(TIMEOUT_NS, 1_000_000) == 0
        assert L.spb_debug_config(INJECT, 1) == 0
        assert _call(L, W, x, lab, out, ws, stream) == 0
        torch.cuda.synchronize()  # returns: every wait is bounded
        # the partner-exchange wait runs out (4), or first the MMA issuer's wait
        # for the h that exchange would have produced (5)
        assert spb.device_error(ws) in (ERR_XCHG, ERR_H)
    finally:
        L.spb_debug_config(INJECT, 0)
        L.spb_debug_config(TIMEOUT_NS, 0)
    spb.clear_device_error(ws)
    assert _call(L, W, x, lab, out, ws, stream) == 0
    torch.cuda.synchronize()
    assert spb.device_error(ws) == 0
    assert_close(out.cpu().numpy(), oracle_mod.ffn(*Wh, x_h, lab_h))


def test_check_option_raises_on_error_word(spb, cuda):
    """ffn_forward(check=True) reads the error word after the call."""
    import torch
    B, d, f = 8, 512, 1024
    W = [torch.zeros((f, d), dtype=torch.float16, device=cuda) for _ in range(3)]
    x = torch.zeros((B, d), device=cuda)
    lab = torch.zeros((B, f), device=cuda)
    ws = spb.new_workspace(B, d, f, 0, cuda)
    spb.ffn_forward(*W, x, lab, workspace=ws, path=spb.PATH_TENSOR, check=True)
    ws[:4].copy_(torch.tensor([7, 0, 0, 0], dtype=torch.uint8, device=cuda))  # a recorded code
    with pytest.raises(spb.SpbError, match="code 7"):
        spb.ffn_forward(*W, x, lab, workspace=ws, path=spb.PATH_TENSOR, check=True)
    assert spb.device_error(ws) == 0
