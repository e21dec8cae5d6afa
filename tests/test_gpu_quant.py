"""Q8_0 / Q4_0 weights on the GPU (config 4): in-kernel dequantisation gives
the oracle's values exactly, and the sparse FFN over quantised weights agrees
with the oracle FFN over the dequantised weights."""
import numpy as np
import pytest

from conftest import assert_close
from spbatch_b200.workload import zipf_active_labels

pytestmark = pytest.mark.gpu


def _dev(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.mark.parametrize("qt", [8, 4])
def test_dequantized_values_identical(spb, cuda, oracle_mod, qt):
    import torch
    rng = np.random.default_rng(qt)
    w = (rng.standard_normal((96, 512)) * 0.02).astype(np.float32)
    w[3, :32] = 0.0
    q = oracle_mod.quantize(w, qt)
    out = torch.empty((96, 512), device=cuda)
    code = spb.W_Q8_0 if qt == 8 else spb.W_Q4_0
    qd = _dev(q, cuda)
    rc = spb.lib().spb_dequantize_rows(qd.data_ptr(), code, 96, 512, out.data_ptr(),
                                       torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), oracle_mod.dequantize(q, qt, 512))


@pytest.mark.parametrize("qt", [8, 4])
@pytest.mark.parametrize("B", [1, 4, 16, 32])
def test_quantized_ffn_7b(spb, cuda, oracle_mod, qt, B):
    import torch
    rng = np.random.default_rng(100 * qt + B)
    d, f = 4096, 11008
    Wf = [(rng.standard_normal((f, d)) * 0.02).astype(np.float32) for _ in range(3)]
    Q = [oracle_mod.quantize(w, qt) for w in Wf]
    Wdq = [oracle_mod.dequantize(q, qt, d) for q in Q]
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = zipf_active_labels(B, f, 1101, seed=B)
    code = spb.W_Q8_0 if qt == 8 else spb.W_Q4_0
    out = spb.ffn_forward(*[_dev(q, cuda) for q in Q], _dev(x, cuda), _dev(lab, cuda), wtype=code)
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), oracle_mod.ffn_f32w(*Wdq, x, lab))
