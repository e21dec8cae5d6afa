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
@pytest.mark.parametrize("B,path", [(1, "auto"), (4, "auto"), (8, "auto"), (16, "auto"), (32, "auto"),
                                    (16, "gemv")])
def test_quantized_ffn_7b(spb, cuda, oracle_mod, qt, B, path):
    """B <= 4 streams on the CUDA cores; larger batches take the tensor-core
    path (blocks expanded to fp16 in shared memory); PATH_GEMV at B = 16 runs
    the per-token-group streaming launches."""
    import torch
    rng = np.random.default_rng(100 * qt + B)
    d, f = 4096, 11008
    Wf = [(rng.standard_normal((f, d)) * 0.02).astype(np.float32) for _ in range(3)]
    Q = [oracle_mod.quantize(w, qt) for w in Wf]
    Wdq = [oracle_mod.dequantize(q, qt, d) for q in Q]
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = zipf_active_labels(B, f, 1101, seed=B)
    code = spb.W_Q8_0 if qt == 8 else spb.W_Q4_0
    if B > 4 and path == "auto":
        # the tensor-core path multiplies the dequantised weights rounded to
        # its fp16 operand type (q * scale is exact in fp32, rounded once)
        Wdq = [oracle_mod.round_f16(w) for w in Wdq]
    ws = spb.new_workspace(B, d, f, 0, cuda)
    p = {"auto": spb.PATH_AUTO, "gemv": spb.PATH_GEMV}[path]
    out = spb.ffn_forward(*[_dev(q, cuda) for q in Q], _dev(x, cuda), _dev(lab, cuda), wtype=code, path=p,
                          workspace=ws)
    torch.cuda.synchronize()
    assert spb.device_error(ws) == 0
    assert_close(out.cpu().numpy(), oracle_mod.ffn_f32w(*Wdq, x, lab))


@pytest.mark.parametrize("qt", [8, 4])
@pytest.mark.parametrize("B,d,f,act,per_token", [(20, 1024, 2000, 0, 1), (64, 512, 3000, 1, 1), (9, 2048, 1500, 0, 0),
                                                 (130, 256, 700, 0, 1)])
def test_quantized_tensor_path_shapes(spb, cuda, oracle_mod, qt, B, d, f, act, per_token):
    """Tensor-core path over quantised rows at ragged f, both activations,
    union semantics, and batches over 128 (Np up to 144)."""
    import torch
    rng = np.random.default_rng(qt * 1000 + B)
    Wf = [(rng.standard_normal((f, d)) * 0.02).astype(np.float32) for _ in range(3)]
    Q = [oracle_mod.quantize(w, qt) for w in Wf]
    # the tensor-core path's operand: the dequantised weight rounded to fp16
    Wdq = [oracle_mod.round_f16(oracle_mod.dequantize(q, qt, d)) for q in Q]
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = zipf_active_labels(B, f, max(1, f // 10), seed=B + qt)
    code = spb.W_Q8_0 if qt == 8 else spb.W_Q4_0
    ws = spb.new_workspace(B, d, f, 0, cuda)
    out = spb.ffn_forward(*[_dev(q, cuda) for q in Q], _dev(x, cuda), _dev(lab, cuda), wtype=code,
                          path=spb.PATH_TENSOR, act=act, per_token_mask=per_token, workspace=ws)
    torch.cuda.synchronize()
    assert spb.device_error(ws) == 0
    want = oracle_mod.ffn_f32w(*Wdq, x, lab, act=act, per_token=bool(per_token))
    assert_close(out.cpu().numpy(), want)
