"""Readers for the reference's predictor checkpoints and activation dumps
(DejaVu_predictor/main_mlp.py:148-156, cuda/utility.cu:7-26)."""
import numpy as np
import pytest

from spbatch_b200 import io


def test_load_predictor_both_key_sets(tmp_path):
    import torch
    g = torch.Generator().manual_seed(0)
    fc1, fc2 = torch.randn(64, 256, generator=g), torch.randn(512, 64, generator=g)
    for keys in io.PRED_KEYS:
        p = tmp_path / f"{keys[0]}.pt"
        torch.save({keys[0]: fc1, keys[1]: fc2}, p)
        p1, p2 = io.load_predictor(str(p))
        assert p1.dtype == torch.float16 and p2.dtype == torch.float16
        assert tuple(p1.shape) == (64, 256) and tuple(p2.shape) == (512, 64)
        assert torch.equal(p1, fc1.half()) and torch.equal(p2, fc2.half())


def test_load_predictor_rejects_bad_shapes(tmp_path):
    import torch
    p = tmp_path / "bad.pt"
    torch.save({"fc1.weight": torch.zeros(64, 256), "fc2.weight": torch.zeros(512, 32)}, p)
    with pytest.raises(ValueError):
        io.load_predictor(str(p))
    torch.save({"w": torch.zeros(2, 2)}, p)
    with pytest.raises(KeyError):
        io.load_predictor(str(p))


def test_read_dump_skips_like_read_idx(tmp_path):
    rows, f = 20, 96
    data = (np.arange(rows * f) % 7 - 3).astype(np.float16).reshape(rows, f)
    p = tmp_path / "mlp_label_0.mmap"
    data.tofile(p)
    assert io.dump_rows(str(p), f) == rows
    lab = io.read_labels(str(p), f, 4)  # rows 8..11, as cuda/utility.cu read_idx
    np.testing.assert_array_equal(lab, data[8:12].astype(np.float32))
    np.testing.assert_array_equal(io.read_queries(str(p), f, 3, skip=0), data[:3].astype(np.float32))
    with pytest.raises(ValueError):
        io.read_labels(str(p), f, 13)
    with pytest.raises(ValueError):
        io.dump_rows(str(p), 97)
