"""Seeded synthetic inputs for the sparse-FFN benchmarks and tests.

The reference measures on ProSparse activation dumps
(``DejaVu_predictor/predictor_data/<model>/mlp_label_{l}.mmap``, read by
``read_idx`` in cuda/utility.cu:7-26).  Those files are not available, so the
benchmark configurations stand in seeded synthetic activity with the same
shapes:

* per-token active sets of exactly ``k`` neurons drawn without replacement
  from a Zipf-like popularity ``p_i ~ rank_i ** -alpha`` (alpha = 0.8), with
  ranks a seeded random permutation of the ``f`` neurons.  Sampling uses the
  Efraimidis-Spirakis keys ``log(u_i) / p_i`` (the k largest keys form a
  weighted sample without replacement);
* activity is written in the reference's label format: ``idx[t][j] > 0``
  means neuron j is active for token t (cuda/kernel.cu:553, 1289).
"""
from __future__ import annotations

import numpy as np

SHAPES = {
    "7b": dict(d=4096, f=11008),
    "13b": dict(d=5120, f=13824),
    "70b": dict(d=8192, f=28672),
}


def zipf_active_labels(B: int, f: int, k: int, alpha: float = 0.8, seed: int = 0,
                       layer: int = 0) -> np.ndarray:
    """[B][f] float32 labels (1.0 active, 0.0 inactive), exactly k per token."""
    rng = np.random.Generator(np.random.PCG64([seed, layer, 0x5b]))
    rank = rng.permutation(f).astype(np.float64) + 1.0
    inv_w = rank ** alpha  # 1 / p_i up to a constant
    u = rng.random((B, f))
    u = np.where(u <= 0.0, np.finfo(np.float64).tiny, u)
    keys = np.log(u) * inv_w[None, :]
    top = np.argpartition(-keys, k - 1, axis=1)[:, :k]
    lab = np.zeros((B, f), np.float32)
    np.put_along_axis(lab, top, 1.0, axis=1)
    return lab


def union_size(labels: np.ndarray) -> int:
    return int((labels > 0).any(axis=0).sum())


def active_bytes(d: int, U: int, B: int, w_bytes: float = 2.0, predictor: int = 0) -> float:
    """Algorithmic HBM bytes of one layer: 3*d*U weight bytes + x (fp16) + out (fp32)."""
    return 3.0 * d * U * w_bytes + B * d * 2 + B * d * 4 + predictor
