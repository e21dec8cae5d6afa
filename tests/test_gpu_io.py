"""The reference's on-disk artifacts through the GPU path.

* A predictor checkpoint in the layout DejaVu_predictor/main_mlp.py writes
  (an nn.Sequential(Linear(d, D, bias=False), ReLU, Linear(D, f,
  bias=False)) state dict, main_mlp.py:137-141, 148-156), loaded with
  io.load_predictor and run with spb_predict: logits against the module
  itself, index sets bit-exact against the oracle.
* A ProSparse-format activation dump (fp16 rows, the first 8 skipped as
  read_idx does, cuda/utility.cu:7-26), read with io.read_labels /
  io.read_queries and run through spb_ffn_forward against the oracle.
"""
import numpy as np
import pytest

from conftest import assert_close
from spbatch_b200 import io
from spbatch_b200.workload import zipf_active_labels

pytestmark = pytest.mark.gpu


def test_checkpoint_predictor_matches_module(spb, cuda, oracle_mod, tmp_path):
    import torch
    d, D, f, B, k = 1024, 256, 2048, 4, 205
    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Linear(d, D, bias=False), torch.nn.ReLU(),
                                torch.nn.Linear(D, f, bias=False))
    with torch.no_grad():  # fp16-representable weights, as the fp16 library stores them
        for m in (model[0], model[2]):
            m.weight.copy_(m.weight.half().float())
    path = tmp_path / "model_0.pt"
    torch.save(model.state_dict(), path)  # keys "0.weight", "2.weight"
    p1, p2 = io.load_predictor(str(path), device=cuda)
    x = torch.randn(B, d).half().float()  # fp16-representable inputs
    logits = torch.empty((B, f), device=cuda)
    labels = torch.empty((B, f), device=cuda)
    ws = spb.predict_workspace(B, D, f, cuda)
    L = spb.lib()
    assert L.spb_predict(p1.data_ptr(), p2.data_ptr(), x.to(cuda).data_ptr(), B, d, D, f, k, 0.0,
                         labels.data_ptr(), None, None, None, logits.data_ptr(), ws.data_ptr(), ws.numel(),
                         torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    with torch.no_grad():
        want = model(x).numpy()  # fp32 throughout; the library rounds the hidden layer to fp16
    got = logits.cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=2e-2, atol=2e-2 * np.abs(want).max())
    # the sets: bit-exact against the oracle restating the library's order
    _, lab_ref, _, _ = oracle_mod.predict(p1.cpu().numpy(), p2.cpu().numpy(), x.numpy(), k=k)
    np.testing.assert_array_equal(labels.cpu().numpy(), lab_ref)
    # and the module's own top-k agrees except at the boundary (near-equal logits)
    top = np.argsort(-want, axis=1, kind="stable")[:, :k]
    mod_lab = np.zeros_like(want)
    np.put_along_axis(mod_lab, top, 1.0, axis=1)
    assert (mod_lab != lab_ref).sum(axis=1).max() <= 4


def test_activation_dump_through_ffn(spb, cuda, oracle_mod, tmp_path):
    import torch
    d, f, B = 1024, 2048, 6
    rows = B + 8 + 3
    lab_rows = zipf_active_labels(rows, f, 205, seed=11)
    x_rows = np.random.default_rng(11).standard_normal((rows, d)).astype(np.float16)
    lab_path, x_path = tmp_path / "mlp_label_0.mmap", tmp_path / "mlp_sp_x_0.mmap"
    lab_rows.astype(np.float16).tofile(lab_path)
    x_rows.tofile(x_path)
    lab = io.read_labels(str(lab_path), f, B)      # rows 8 .. 8 + B
    x = io.read_queries(str(x_path), d, B)
    np.testing.assert_array_equal(lab, lab_rows[8:8 + B])
    rng = np.random.default_rng(12)
    W = [(rng.standard_normal((f, d)) * 0.04).astype(np.float16) for _ in range(3)]
    out = spb.ffn_forward(*[torch.from_numpy(w).to(cuda) for w in W], torch.from_numpy(x).to(cuda),
                          torch.from_numpy(lab).to(cuda))
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), oracle_mod.ffn(*W, x, lab))
