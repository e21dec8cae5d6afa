"""spbatch_b200 -- B200-native activation-sparse FFN (SpBatch hot path).

Python host bindings over ``libspbatch_b200.so`` (C ABI in ``include/spb.h``;
the reference's C++ API in ``include/spbatch/kernel.cuh``).  PyTorch supplies
device memory and streams only; every computation runs in the library's CUDA
kernels.  There is no CPU fallback: importing the bindings without the built
library raises, and calling them without a GPU raises.
"""
from __future__ import annotations

import ctypes as C
import os

from . import workload  # noqa: F401

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("SPB_LIB") or os.path.join(PKG, "libspbatch_b200.so")

SPB_OK = 0
W_F16, W_Q8_0, W_Q4_0 = 0, 1, 2
ACT_RELU_MUL, ACT_RELU_RELU_MUL = 0, 1
PATH_AUTO, PATH_GEMV, PATH_TENSOR = 0, 1, 2

DEBUG_LIB_PATH = os.path.join(PKG, "libspbatch_b200_debug.so")

_lib = None
_debug_lib = None


class SpbError(RuntimeError):
    pass


def _load(path: str) -> C.CDLL:
    if not os.path.exists(path):
        raise SpbError(f"{path} is missing: run `python -m spbatch_b200.build`")
    # The library uses cuBLASLt (the predictor's GEMMs for large batches).
    # PyTorch ships its own cuBLAS / cuBLASLt pair; loading torch first makes
    # the library bind to that already-loaded cuBLASLt (same soname) instead
    # of loading the toolkit's copy, which torch's cuBLAS would then pick up.
    import torch  # noqa: F401
    L = C.CDLL(path)
    _bind(L)
    return L


def lib() -> C.CDLL:
    """Loads libspbatch_b200.so (build it with ``python -m spbatch_b200.build``)."""
    global _lib
    if _lib is None:
        _lib = _load(LIB_PATH)
    return _lib


def debug_lib() -> C.CDLL:
    """The test-hook build of the library (include/spb_debug.h); tests only."""
    global _debug_lib
    if _debug_lib is None:
        _debug_lib = _load(DEBUG_LIB_PATH)
        _debug_lib.spb_debug_config.argtypes = [C.c_int, C.c_longlong]
    return _debug_lib


def _bind(L: C.CDLL) -> None:
    P, I, Z = C.c_void_p, C.c_int, C.c_size_t
    L.spb_last_error.restype = C.c_char_p
    L.spb_version.restype = I
    L.spb_ffn_workspace_bytes.argtypes = [I, I, I, I]
    L.spb_ffn_workspace_bytes.restype = Z
    L.spb_union.argtypes = [P, I, I, I, P, P, P, P, Z, P]
    L.spb_union_static.argtypes = [P, I, I, I, P, P, P, P]
    L.spb_weight_row_bytes.argtypes = [I, I]
    L.spb_weight_row_bytes.restype = C.c_int64
    L.spb_quantize.argtypes = [P, I, I, I, P]
    L.spb_dequantize_rows.argtypes = [P, I, I, I, P, P]
    L.spb_predict_workspace_bytes.argtypes = [I, I, I]
    L.spb_predict_workspace_bytes.restype = Z
    L.spb_predict.argtypes = [P, P, P, I, I, I, I, I, C.c_float, P, P, P, P, P, P, Z, P]
    L.spb_ffn_forward_bits.argtypes = [P, P, P, I, P, P, I, I, I, I, I, I, P, P, P, P, Z, P]
    L.spb_ffn_forward_bias.argtypes = [P, P, P, I, P, P, P, P, P, I, I, I, I, I, I, P, P, P, P, Z, P]
    L.spb_ffn_forward.argtypes = [P, P, P, I, P, P, I, I, I, I, I, I, P, P, P, P, Z, P]
    L.spb_ffn_launches.argtypes = [I, I, I, I]
    L.spb_trace_enable.argtypes = [P, Z]
    L.spb_peer_handle_bytes.restype = Z
    L.spb_peer_sync_bytes.restype = Z
    L.spb_peer_export.argtypes = [P, P]
    L.spb_peer_import.argtypes = [P, C.POINTER(C.c_void_p)]
    L.spb_peer_close.argtypes = [P]
    L.spb_allreduce_peer.argtypes = [P, P, P, I, I, C.c_int64, P, C.c_int64, P, P]


def _check(rc: int, what: str) -> None:
    if rc != SPB_OK:
        raise SpbError(f"{what} failed ({rc}): {lib().spb_last_error().decode()}")


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise SpbError("spbatch_b200 operates on CUDA tensors only (no CPU fallback)")
        if t is not None and not t.is_contiguous():
            raise SpbError("spbatch_b200 needs contiguous tensors")


def device_error(workspace) -> int:
    """The workspace's sticky device error code (0: no bounded wait ran out).

    Reads 4 bytes back to the host, so it synchronises with the stream."""
    import numpy as np
    return int(np.frombuffer(workspace[:4].cpu().numpy().tobytes(), np.uint32)[0])


def clear_device_error(workspace) -> None:
    workspace[:4].zero_()


def workspace_bytes(B: int, d: int, f: int, group: int = 0) -> int:
    return int(lib().spb_ffn_workspace_bytes(B, d, f, group))


def new_workspace(B: int, d: int, f: int, group: int = 0, device=None):
    import torch
    return torch.zeros(workspace_bytes(B, d, f, group), dtype=torch.uint8, device=device or "cuda")


def union(idx, group: int = 0, workspace=None, stream=None):
    """Segment union of active neurons (replaces get_idx_cuda).

    Returns (merge_idx [S][f] int32, act_cum [S] int32 cumulative, tok_bits
    [B][ceil(f/32)] int32 bit words).  group=0: one segment for the batch.
    """
    import torch
    _require_cuda(idx)
    B, f = idx.shape
    G = B if group == 0 else group
    S = (B + G - 1) // G
    dev = idx.device
    merge = torch.zeros((S, f), dtype=torch.int32, device=dev)
    act = torch.zeros(S, dtype=torch.int32, device=dev)
    bits = torch.zeros((B, (f + 31) // 32), dtype=torch.int32, device=dev)
    ws = workspace if workspace is not None else new_workspace(B, 64, f, group, dev)
    _check(lib().spb_union(idx.data_ptr(), B, f, group, merge.data_ptr(), act.data_ptr(), bits.data_ptr(),
                           ws.data_ptr(), ws.numel(), _stream(stream)), "spb_union")
    return merge, act, bits


def ffn_forward(w_gate, w_up, w_down, x, idx=None, *, bits=None, f: int | None = None, wtype: int = W_F16,
                act: int = ACT_RELU_MUL, per_token_mask: bool = True, path: int = PATH_AUTO, out=None,
                workspace=None, merge_idx_out=None, count_out=None, stream=None, check: bool = False,
                bias_gate=None, bias_up=None):
    """One sparse FFN layer on the GPU (see spb_ffn_forward in include/spb.h).

    w_gate / w_up / w_down: [f][d] rows (W_down stored transposed, as the
    reference stores it); x [B][d] fp32; the active sets either as idx [B][f]
    fp32 labels (> 0 active) or as bits [B][ceil(f/32)] int32 words
    (spb_ffn_forward_bits; f is then w_gate's row count unless given).
    bias_gate / bias_up ([f] fp16) add the linear layers' biases to the gate
    / up products before the activation (spb_ffn_forward_bias).
    check=True waits for the layer and raises if a bounded device wait ran
    out (the workspace's error word, which it then clears).
    """
    import torch
    _require_cuda(w_gate, w_up, w_down, x, idx, bits, out, merge_idx_out, count_out, bias_gate, bias_up)
    if (idx is None) == (bits is None):
        raise SpbError("ffn_forward: give exactly one of idx (labels) and bits")
    B, d = x.shape
    if idx is not None:
        f = idx.shape[1]
    elif f is None:
        f = w_gate.shape[0]
    if out is None:
        out = torch.empty((B, d), dtype=torch.float32, device=x.device)
    ws = workspace if workspace is not None else new_workspace(B, d, f, 0, x.device)
    if bias_gate is not None or bias_up is not None:
        _check(lib().spb_ffn_forward_bias(w_gate.data_ptr(), w_up.data_ptr(), w_down.data_ptr(), wtype, x.data_ptr(),
                                          _ptr(idx), _ptr(bits), _ptr(bias_gate), _ptr(bias_up), B, d, f, act,
                                          int(per_token_mask), path, out.data_ptr(), _ptr(merge_idx_out),
                                          _ptr(count_out), ws.data_ptr(), ws.numel(), _stream(stream)),
               "spb_ffn_forward_bias")
    else:
        fn, sets = (lib().spb_ffn_forward, idx) if idx is not None else (lib().spb_ffn_forward_bits, bits)
        _check(fn(w_gate.data_ptr(), w_up.data_ptr(), w_down.data_ptr(), wtype, x.data_ptr(), sets.data_ptr(), B, d,
                  f, act, int(per_token_mask), path, out.data_ptr(), _ptr(merge_idx_out), _ptr(count_out),
                  ws.data_ptr(), ws.numel(), _stream(stream)), "spb_ffn_forward")
    if check:
        code = device_error(ws)
        if code:
            clear_device_error(ws)
            raise SpbError(f"spb_ffn_forward: device wait ran out (code {code}); the output is not valid")
    return out


def quantize(w, wtype: int):
    """Host-side ggml quantisation of fp32 rows ([rows][d] numpy) to the split
    row layout; returns a [rows][row_bytes] uint8 numpy array."""
    import numpy as np
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, d = w.shape
    rb = int(lib().spb_weight_row_bytes(wtype, d))
    if rb <= 0:
        raise SpbError("quantize: d must be a multiple of 32")
    out = np.zeros((rows, rb), np.uint8)
    _check(lib().spb_quantize(w.ctypes.data, rows, d, wtype, out.ctypes.data), "spb_quantize")
    return out


def predict_workspace(B: int, D: int, f: int, device=None):
    """Scratch for spb_predict (allocate once, reuse: predict() then allocates nothing)."""
    import torch
    return torch.empty(int(lib().spb_predict_workspace_bytes(B, D, f)), dtype=torch.uint8, device=device or "cuda")


def predict(p1, p2, x, k: int = 0, threshold: float = 0.0, *, return_idx: bool = False, out=None, bits_out=None,
            labels: bool = True, workspace=None, stream=None):
    """DejaVu predictor on the GPU (spb_predict): labels [B][f] (1 active).

    p1 [D][d] fp16, p2 [f][D] fp16, x [B][d] fp32.  k > 0 selects the top-k
    logits per token; k = 0 thresholds the logits.  With return_idx, also the
    ascending active ids [B][k or f] and the per-token counts.  `out` ([B][f]
    fp32) and `workspace` (predict_workspace) make the call allocation-free,
    so it can be captured in a CUDA graph.  bits_out ([B][ceil(f/32)] int32)
    also receives the sets as bit words (the input of ffn_forward(bits=...));
    labels=False skips the [B][f] label output and returns bits_out.
    """
    import torch
    _require_cuda(p1, p2, x, out, workspace)
    B, d = x.shape
    D, f = p1.shape[0], p2.shape[0]
    dev = x.device
    _require_cuda(bits_out)
    lab_t = (out if out is not None else torch.empty((B, f), dtype=torch.float32, device=dev)) if labels else None
    if lab_t is None and bits_out is None:
        raise SpbError("predict: labels=False needs bits_out")
    idx = torch.full((B, k if k > 0 else f), -1, dtype=torch.int32, device=dev) if return_idx else None
    counts = torch.zeros(B, dtype=torch.int32, device=dev) if return_idx else None
    ws = workspace if workspace is not None else predict_workspace(B, D, f, dev)
    _check(lib().spb_predict(p1.data_ptr(), p2.data_ptr(), x.data_ptr(), B, d, D, f, k, threshold,
                             _ptr(lab_t), _ptr(bits_out), _ptr(idx), _ptr(counts), None, ws.data_ptr(), ws.numel(),
                             _stream(stream)), "spb_predict")
    res = lab_t if lab_t is not None else bits_out
    return (res, idx, counts) if return_idx else res


class dropin:
    """The reference's C++ API (include/spbatch/kernel.cuh), bound by its
    mangled names, with the reference's argument order and M/N/K meanings."""

    _SYMS = {
        "get_idx_cuda": ("_Z12get_idx_cudaPKfPiS1_iiP11CUstream_st", "PPPiiP"),
        "up_mul_mat_cuda_sparse": ("_Z22up_mul_mat_cuda_sparsePK6__halfPKfPfPiiiiPKiP11CUstream_st", "PPPPiiiPP"),
        "gate_and_up_mul_mat_cuda_sparse": (
            "_Z31gate_and_up_mul_mat_cuda_sparsePK6__halfS1_PKfPfS4_PiiiiPKiP11CUstream_stS9_", "PPPPPPiiiPPP"),
        "relu_and_mul_cuda": ("_Z17relu_and_mul_cudaPKfS0_PfiiP11CUstream_st", "PPPiiP"),
        "relu_relu_mul_cuda": ("_Z18relu_relu_mul_cudaPKfS0_PfiiP11CUstream_st", "PPPiiP"),
        "down_mul_mat_cuda_sparse": ("_Z24down_mul_mat_cuda_sparsePK6__halfPKfPfPiiiiPKiP11CUstream_st",
                                     "PPPPiiiPP"),
        "naive_mm_up_cuda": ("_Z16naive_mm_up_cudaPK6__halfPKfPfiiiPKiPiP11CUstream_st", "PPPiiiPPP"),
        "naive_mm_down_cuda": ("_Z18naive_mm_down_cudaPK6__halfPKfPfiiiPKiPiP11CUstream_st", "PPPiiiPPP"),
        "naive_sparsity_div": ("_Z18naive_sparsity_divPKfPiS1_ii", "PPPii"),
        "convert_fp32_to_fp16_cuda": ("_Z25convert_fp32_to_fp16_cudaPKvP6__halfiP11CUstream_st", "PPiP"),
        "convert_fp16_to_fp32_cuda": ("_Z25convert_fp16_to_fp32_cudaPKvPfiP11CUstream_st", "PPiP"),
        "convert_mul_mat_batch_f16_cuda_sparse": (
            "_Z37convert_mul_mat_batch_f16_cuda_sparsePKvPKfPfiiiiP11CUstream_stPiS3_", "PPPiiiiPPP"),
        "convert_axpy_sparse_batch_f16_cuda": (
            "_Z34convert_axpy_sparse_batch_f16_cudaPKvPKfPfiiiiP11CUstream_stPiS3_", "PPPiiiiPPP"),
        "relu_f32_cuda": ("_Z13relu_f32_cudaPKfPfiP11CUstream_st", "PPiP"),
        "mul_f32_cuda": ("_Z12mul_f32_cudaPKfS0_PfiiP11CUstream_st", "PPPiiP"),
        "add_sparse_cuda": ("_Z15add_sparse_cudaPKfPK6__halfPfiiPKiS6_P11CUstream_st", "PPPiiPPP"),
        "gemm_cuda": ("_Z9gemm_cudaPK6__halfPKfPfiiiP11CUstream_st", "PPPiiiP"),
    }

    @classmethod
    def fn(cls, name: str, library=None):
        sym, sig = cls._SYMS[name]
        f = getattr(library or lib(), sym)
        f.argtypes = [C.c_void_p if c == "P" else C.c_int for c in sig]
        f.restype = None
        return f
