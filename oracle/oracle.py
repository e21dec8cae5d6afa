"""ctypes front end of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg import this module; it is the checker for the CUDA library, never part of
it.  Two libraries sit behind it:

* ``oracle/_build/libspb_oracle.so`` -- the C restatement in ``spb_oracle.c``
  (union/compaction after ``naive_sparsity_div``, cuda/kernel.cu:1280-1297;
  gather GEMMs after ``naive_mm_up_kernel``/``naive_mm_down_kernel``,
  cuda/kernel.cu:1079-1113; the full FFN after ``MLP_naive``,
  cuda/ffn_test.cu:144-163; ggml Q4_0/Q8_0).
* ``oracle/_ref/libspbatch_ref.so`` -- the reference's own ``cuda/kernel.cu``
  and ``cuda/utility.cu`` compiled by ``oracle/Makefile`` (present only where
  the reference sources were available at build time).  Its host function
  ``naive_sparsity_div`` pins ``spbo_union``; its naive GPU kernels pin the
  FFN restatement on a GPU box.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libspb_oracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libspbatch_ref.so")

_lib = None
_ref = None


def ref_dir() -> str | None:
    """The reference checkout: $SPB_REF_DIR, else a `reference` directory next
    to this repository; None when neither holds the reference's cuda/ sources."""
    cand = os.environ.get("SPB_REF_DIR") or os.path.join(os.path.dirname(HERE), os.pardir, "reference")
    cand = os.path.abspath(cand)
    return cand if os.path.isdir(os.path.join(cand, "cuda")) else None


def build(ref: bool = False) -> None:
    """Compile the oracle (and the reference library when asked and possible)."""
    subprocess.check_call(["make", "-s", "-C", HERE, "all"])
    rd = ref_dir() if ref else None
    if rd:
        subprocess.check_call(["make", "-s", "-C", HERE, "ref", f"REF_DIR={rd}"])
        # the reference's spmm_test / ffn_test drivers against this library and its own
        subprocess.check_call(["make", "-s", "-C", HERE, "drivers", f"REF_DIR={rd}"])


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        P = C.c_void_p
        i = C.c_int
        _lib.spbo_union.argtypes = [P, i, i, i, P, P]
        _lib.spbo_token_bits.argtypes = [P, i, i, P]
        _lib.spbo_up_compact.argtypes = [P, P, P, P, i, i, i, i, i, P]
        _lib.spbo_down_compact.argtypes = [P, P, P, P, i, i, i, i, i, P]
        _lib.spbo_ffn.argtypes = [P, P, P, P, P, i, i, i, i, i, i, P]
        _lib.spbo_ffn_bias.argtypes = [P, P, P, P, P, P, P, i, i, i, i, i, i, P]
        _lib.spbo_ffn_f32w.argtypes = [P, P, P, P, P, i, i, i, i, i, i, P]
        _lib.spbo_round_f16.argtypes = [P, P, C.c_int64]
        _lib.spbo_f32_to_f16_array.argtypes = [P, P, C.c_int64]
        _lib.spbo_quantize_q8_0.argtypes = [P, i, i, P]
        _lib.spbo_quantize_q4_0.argtypes = [P, i, i, P]
        _lib.spbo_dequantize.argtypes = [P, i, i, i, P]
        _lib.spbo_predict.argtypes = [P, P, P, i, i, i, i, i, C.c_float, P, P, P, P]
    return _lib


def ref_lib():
    """The reference's own library, or None where it was not built."""
    global _ref
    if _ref is None and os.path.exists(REF_PATH):
        _ref = C.CDLL(REF_PATH)
    return _ref


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _u16(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        a = a.view(np.uint16)
    assert a.dtype == np.uint16
    return a


def union(idx: np.ndarray, G: int):
    """Segment union (ascending indices) and per-segment counts."""
    idx = _f32(idx)
    B, f = idx.shape
    S = (B + G - 1) // G
    merge = np.zeros((S, f), np.int32)
    counts = np.zeros(S, np.int32)
    lib().spbo_union(_p(idx), B, f, G, _p(merge), _p(counts))
    return merge, counts


def token_bits(idx: np.ndarray) -> np.ndarray:
    idx = _f32(idx)
    B, f = idx.shape
    bits = np.zeros((B, (f + 31) // 32), np.uint32)
    lib().spbo_token_bits(_p(idx), B, f, _p(bits))
    return bits


def up_compact(w, x, merge, counts, G, round_x=True):
    w = _u16(w)
    x = _f32(x)
    B, d = x.shape
    f = w.shape[0]
    dst = np.zeros((B, f), np.float32)
    lib().spbo_up_compact(_p(w), _p(x), _p(np.ascontiguousarray(merge, np.int32)),
                          _p(np.ascontiguousarray(counts, np.int32)), B, d, f, G, int(round_x), _p(dst))
    return dst


def down_compact(wd, h, merge, counts, G, round_h=True):
    wd = _u16(wd)
    h = _f32(h)
    B, f = h.shape
    d = wd.shape[1]
    dst = np.zeros((B, d), np.float32)
    lib().spbo_down_compact(_p(wd), _p(h), _p(np.ascontiguousarray(merge, np.int32)),
                            _p(np.ascontiguousarray(counts, np.int32)), B, d, f, G, int(round_h), _p(dst))
    return dst


def ffn(wg, wu, wd, x, idx, G=None, per_token=True, act=0):
    """Sparse FFN forward (fp16 weights as float16/uint16 arrays)."""
    wg, wu, wd = _u16(wg), _u16(wu), _u16(wd)
    x, idx = _f32(x), _f32(idx)
    B, d = x.shape
    f = wg.shape[0]
    G = B if G is None else G
    out = np.zeros((B, d), np.float32)
    lib().spbo_ffn(_p(wg), _p(wu), _p(wd), _p(x), _p(idx), B, d, f, G, int(per_token), act, _p(out))
    return out


def ffn_bias(wg, wu, wd, x, idx, bias_gate=None, bias_up=None, per_token=True, act=0):
    """ffn with fp16 neuron biases (either None) added to gate / up before the activation."""
    wg, wu, wd = _u16(wg), _u16(wu), _u16(wd)
    x, idx = _f32(x), _f32(idx)
    B, d = x.shape
    f = wg.shape[0]
    bg = None if bias_gate is None else _u16(bias_gate)
    bu = None if bias_up is None else _u16(bias_up)
    out = np.zeros((B, d), np.float32)
    lib().spbo_ffn_bias(_p(wg), _p(wu), _p(wd), _p(x), _p(idx), None if bg is None else _p(bg),
                        None if bu is None else _p(bu), B, d, f, B, int(per_token), act, _p(out))
    return out


def ffn_f32w(wg, wu, wd, x, idx, G=None, per_token=True, act=0):
    wg, wu, wd, x, idx = map(_f32, (wg, wu, wd, x, idx))
    B, d = x.shape
    f = wg.shape[0]
    G = B if G is None else G
    out = np.zeros((B, d), np.float32)
    lib().spbo_ffn_f32w(_p(wg), _p(wu), _p(wd), _p(x), _p(idx), B, d, f, G, int(per_token), act, _p(out))
    return out


def round_f16(a):
    a = _f32(a)
    out = np.empty_like(a)
    lib().spbo_round_f16(_p(a), _p(out), a.size)
    return out


def to_f16_bits(a):
    a = _f32(a)
    out = np.empty(a.shape, np.uint16)
    lib().spbo_f32_to_f16_array(_p(a), _p(out), a.size)
    return out


def quantize(w, qtype: int) -> np.ndarray:
    """ggml Q8_0 (qtype 8) / Q4_0 (qtype 4) in the split row layout."""
    w = _f32(w)
    rows, n = w.shape
    qb = n if qtype == 8 else n // 2
    out = np.zeros((rows, qb + 2 * (n // 32)), np.uint8)
    fn = lib().spbo_quantize_q8_0 if qtype == 8 else lib().spbo_quantize_q4_0
    fn(_p(w), rows, n, _p(out))
    return out


def dequantize(q, qtype: int, n: int) -> np.ndarray:
    q = np.ascontiguousarray(q, np.uint8)
    rows = q.shape[0]
    out = np.zeros((rows, n), np.float32)
    lib().spbo_dequantize(_p(q), qtype, rows, n, _p(out))
    return out


def ref_naive_sparsity_div(idx: np.ndarray):
    """Run the reference's own host union (cuda/kernel.cu:1280-1297).

    Returns (merge_idx [groups][f], per-group counts) or None when the
    reference library is absent.  B must be a multiple of 8.
    """
    r = ref_lib()
    if r is None:
        return None
    fn = r._Z18naive_sparsity_divPKfPiS1_ii
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int]
    idx = _f32(idx)
    B, f = idx.shape
    groups = B // 8
    merge = np.zeros((groups, f), np.int32)
    act = np.zeros(groups, np.int32)
    fn(_p(idx), _p(merge), _p(act), B, f)
    return merge, act


def predict(p1, p2, x, k=0, threshold=0.0):
    """Predictor oracle: (logits [B][f], labels [B][f], idx [B][cap], counts [B])."""
    p1, p2 = _u16(p1), _u16(p2)
    x = _f32(x)
    B, d = x.shape
    D, f = p1.shape[0], p2.shape[0]
    cap = k if k > 0 else f
    logits = np.zeros((B, f), np.float32)
    labels = np.zeros((B, f), np.float32)
    idx = np.full((B, cap), -1, np.int32)
    counts = np.zeros(B, np.int32)
    lib().spbo_predict(_p(p1), _p(p2), _p(x), B, d, D, f, k, threshold, _p(logits), _p(labels), _p(idx), _p(counts))
    return logits, labels, idx, counts
