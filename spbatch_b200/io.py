"""Readers for the reference's on-disk artifacts (host side, no GPU needed).

* Predictor checkpoints written by DejaVu_predictor/main_mlp.py:148-156:
  torch.save({"fc1.weight": [D][d], "fc2.weight": [f][D]}) -- the two bias-free
  Linear layers of the low-rank predictor (main_mlp.py:137-141).  The raw
  nn.Sequential keys ("0.weight", "2.weight") are accepted as well.
* ProSparse activation dumps (mlp_label_{l}.mmap, mlp_sp_x_{l}.mmap): raw
  fp16 row-major [rows][f] (labels) or [rows][d] (queries).  The reference's
  CUDA drivers skip the first 8 rows (cuda/utility.cu:7-26, read_idx);
  main_mlp.py:54-62 reads from row 0.  Labels are active where > 0, the
  format spb_ffn_forward and get_idx_cuda take (as fp32).
"""
from __future__ import annotations

import os

import numpy as np

PRED_KEYS = (("fc1.weight", "fc2.weight"), ("0.weight", "2.weight"))


def load_predictor(path: str, device=None):
    """(P1 [D][d], P2 [f][D]) as fp16 tensors for spbatch_b200.predict."""
    import torch
    sd = torch.load(path, map_location="cpu", weights_only=True)
    if hasattr(sd, "state_dict"):
        sd = sd.state_dict()
    for k1, k2 in PRED_KEYS:
        if k1 in sd and k2 in sd:
            p1, p2 = sd[k1], sd[k2]
            break
    else:
        raise KeyError(f"{path}: no predictor weights (expected one of {PRED_KEYS}), found {sorted(sd)[:8]}")
    if p1.dim() != 2 or p2.dim() != 2 or p2.shape[1] != p1.shape[0]:
        raise ValueError(f"{path}: fc1 {tuple(p1.shape)} and fc2 {tuple(p2.shape)} do not chain")
    p1 = p1.to(torch.float16).contiguous()
    p2 = p2.to(torch.float16).contiguous()
    if device is not None:
        p1, p2 = p1.to(device), p2.to(device)
    return p1, p2


def dump_rows(path: str, cols: int) -> int:
    """Number of fp16 rows of `cols` values in a dump file."""
    n = os.path.getsize(path)
    if n % (2 * cols):
        raise ValueError(f"{path}: {n} bytes is not a whole number of {cols}-value fp16 rows")
    return n // (2 * cols)


def read_dump(path: str, cols: int, rows: int, skip: int = 8) -> np.ndarray:
    """Rows [skip, skip + rows) of an fp16 [*][cols] dump (skip=8 as read_idx)."""
    total = dump_rows(path, cols)
    if skip + rows > total:
        raise ValueError(f"{path}: asked for rows {skip}..{skip + rows} of {total}")
    mm = np.memmap(path, dtype=np.float16, mode="r", shape=(total, cols))
    return np.array(mm[skip:skip + rows])


def read_labels(path: str, f: int, tokens: int, skip: int = 8) -> np.ndarray:
    """Activation labels of `tokens` tokens as fp32 [tokens][f] (active > 0)."""
    return read_dump(path, f, tokens, skip).astype(np.float32)


def read_queries(path: str, d: int, tokens: int, skip: int = 8) -> np.ndarray:
    """FFN inputs x of `tokens` tokens as fp32 [tokens][d]."""
    return read_dump(path, d, tokens, skip).astype(np.float32)
