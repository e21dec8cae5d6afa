"""Generates tests/golden/union_ref.npz from the reference's own code.

The union/compaction fixtures are outputs of the reference's host routine
naive_sparsity_div (cuda/kernel.cu:1280-1297), compiled from the reference
sources into oracle/_ref/libspbatch_ref.so by oracle/Makefile.  Run where the
reference sources exist:

    make -C oracle ref && python tests/golden/make_golden.py

Each case stores the labels (raw fp32 for small cases, packed activity bits
for large ones), the per-group counts and the concatenated valid prefixes of
merge_idx.
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle  # noqa: E402
from spbatch_b200.workload import zipf_active_labels  # noqa: E402


def cases():
    rng = np.random.default_rng(20240611)
    # small raw-label cases, including edge values
    a = rng.standard_normal((16, 256)).astype(np.float32)
    yield "randn_16x256", a, True
    b = np.zeros((8, 96), np.float32)
    b[3, 5] = 1e-30  # tiny positive counts as active
    b[0, 95] = np.inf
    b[1, :] = -0.0
    b[2, 40] = np.nan  # NaN is not > 0
    b[7, 0] = -1.0
    yield "edge_8x96", b, True
    c = np.ones((24, 128), np.float32)
    c[8:16] = 0.0  # one fully inactive group
    yield "allone_gap_24x128", c, True
    # benchmark-shaped Zipf cases (7B neurons), stored as packed bits
    yield "zipf7b_64", zipf_active_labels(64, 11008, 1101, seed=1), False
    yield "zipf13b_32", zipf_active_labels(32, 13824, 1106, seed=2, layer=3), False


def main():
    if oracle.ref_lib() is None:
        raise SystemExit("oracle/_ref/libspbatch_ref.so missing: run `make -C oracle ref` with the reference present")
    out = {}
    for name, lab, raw in cases():
        merge, counts = oracle.ref_naive_sparsity_div(lab)
        flat = np.concatenate([merge[g, :counts[g]] for g in range(len(counts))]).astype(np.int32)
        if raw:
            out[f"{name}/labels"] = lab
        else:
            out[f"{name}/bits"] = np.packbits(lab > 0, axis=1)
            out[f"{name}/shape"] = np.array(lab.shape, np.int64)
        out[f"{name}/counts"] = counts.astype(np.int32)
        out[f"{name}/merge"] = flat
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "union_ref.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
