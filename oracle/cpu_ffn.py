"""PyTorch CPU masked-dense FFN -- the reported CPU baseline (TEST/BENCH
INFRASTRUCTURE ONLY; bench.py's cpu_baseline leg and --impl reference use it).

The reference has no CPU FFN; its correctness oracle is the masked GPU
composition MLP_naive (cuda/ffn_test.cu:144-163).  This restates the same
semantics on the host: dense gate/up products, mask, ReLU(gate)*up, dense
down, with fp16 weights upcast to fp32 once outside any timer.
"""
from __future__ import annotations

import os
import time

import numpy as np
import torch


class MaskedDenseFFN:
    def __init__(self, wg: np.ndarray, wu: np.ndarray, wd: np.ndarray, threads: int | None = None):
        self.threads = threads or len(os.sched_getaffinity(0))
        torch.set_num_threads(self.threads)
        self.wg = torch.from_numpy(np.asarray(wg, np.float32))
        self.wu = torch.from_numpy(np.asarray(wu, np.float32))
        self.wd = torch.from_numpy(np.asarray(wd, np.float32))  # [f][d]

    def __call__(self, x: np.ndarray, labels: np.ndarray) -> np.ndarray:
        xt = torch.from_numpy(x).half().float()
        mask = torch.from_numpy(labels) > 0
        g = xt @ self.wg.T
        u = xt @ self.wu.T
        h = (torch.relu(g) * u * mask).half().float()
        return (h @ self.wd).numpy()


def time_steps(ffn: MaskedDenseFFN, x, labels, budget_s: float = 15.0, max_steps: int = 10 ** 9,
               min_steps: int = 3):
    """Runs whole steps until the time budget is used; returns (steps, seconds)."""
    ffn(x, labels)  # warm-up
    n = 0
    t0 = time.perf_counter()
    while n < max_steps and (n < min_steps or time.perf_counter() - t0 < budget_s):
        ffn(x, labels)
        n += 1
    return n, time.perf_counter() - t0
