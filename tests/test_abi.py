"""CPU tests of the C-ABI library: it loads, exports every symbol the public
headers declare, and rejects bad arguments before touching a device."""
import ctypes as C
import os
import re

import pytest

from conftest import ROOT


def _declared(header, pattern):
    src = open(os.path.join(ROOT, "include", header)).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = re.sub(r"//[^\n]*", "", src)
    return sorted(set(re.findall(pattern, src, flags=re.M)))


def test_c_abi_exports_everything_declared(spb):
    names = _declared("spb.h", r"\b(spb_[a-z0-9_]+)\s*\(")
    assert "spb_ffn_forward" in names and "spb_union" in names
    for n in names:
        assert hasattr(spb.lib(), n), f"{n} declared in include/spb.h but not exported"


def test_dropin_api_exports_everything_declared(spb):
    names = _declared("spbatch/kernel.cuh", r"^\s*void\s+([a-z0-9_]+)\s*\(")
    names = [n for n in names if n != "die"]
    assert len(names) == 17, names
    for n in names:
        assert n in spb.dropin._SYMS, f"{n} missing from the Python binding table"
        sym = spb.dropin._SYMS[n][0]
        assert hasattr(spb.lib(), sym), f"{n} ({sym}) not exported"


def test_version_and_workspace(spb):
    L = spb.lib()
    assert L.spb_version() >= 1
    assert L.spb_ffn_workspace_bytes(0, 4096, 11008, 0) == 0
    a = L.spb_ffn_workspace_bytes(1, 4096, 11008, 0)
    b = L.spb_ffn_workspace_bytes(32, 4096, 11008, 0)
    c = L.spb_ffn_workspace_bytes(32, 4096, 11008, 8)
    assert 0 < a < b < c
    assert a % 256 == 0


def test_invalid_arguments_fail_without_device(spb):
    L = spb.lib()
    rc = L.spb_ffn_forward(None, None, None, 0, None, None, 1, 4096, 11008, 0, 1, 0, None, None, None, None, 0,
                           None)
    assert rc == 1
    assert b"null" in L.spb_last_error()
    fake = C.c_void_p(256)  # never dereferenced: shape checks fail first
    rc = L.spb_ffn_forward(fake, fake, fake, 0, fake, fake, 1, 100, 11008, 0, 1, 0, fake, None, None, fake, 1 << 30,
                           None)
    assert rc == 1 and b"multiple of 64" in L.spb_last_error()
    rc = L.spb_ffn_forward(fake, fake, fake, 7, fake, fake, 1, 4096, 11008, 0, 1, 0, fake, None, None, fake,
                           1 << 30, None)
    assert rc == 1 and b"weight type" in L.spb_last_error()
    rc = L.spb_ffn_forward(fake, fake, fake, 0, fake, fake, 1, 4096, 11008, 0, 1, 0, fake, None, None, fake, 16,
                           None)
    assert rc == 2 and b"workspace" in L.spb_last_error()
    rc = L.spb_union(None, 8, 64, 8, None, None, None, None, 0, None)
    assert rc == 1
    rc = L.spb_union(fake, 8, 64, -1, fake, fake, None, fake, 1 << 20, None)
    assert rc == 1


def test_peer_allreduce_rejects_bad_arguments_without_device(spb):
    """spb_allreduce_peer validates everything before it launches."""
    L = spb.lib()
    assert L.spb_peer_handle_bytes() >= 64  # a CUDA IPC handle plus the pointer's offset
    assert L.spb_peer_sync_bytes() >= 4 * (16 + 8)
    fake = C.c_void_p(256)
    ptrs = (C.c_void_p * 2)(256, 512)
    err = C.c_void_p(1024)
    rc = L.spb_allreduce_peer(None, ptrs, ptrs, 2, 0, 1024, fake, 1024, err, None)
    assert rc == 1 and b"null" in L.spb_last_error()
    rc = L.spb_allreduce_peer(fake, ptrs, ptrs, 9, 0, 1024, fake, 1024, err, None)
    assert rc == 1 and b"world" in L.spb_last_error()
    rc = L.spb_allreduce_peer(fake, ptrs, ptrs, 2, 2, 1024, fake, 1024, err, None)
    assert rc == 1 and b"rank" in L.spb_last_error()
    rc = L.spb_allreduce_peer(fake, ptrs, ptrs, 2, 0, 1024, fake, 1022, err, None)
    assert rc == 1 and b"multiples of 4" in L.spb_last_error()
    rc = L.spb_allreduce_peer(fake, ptrs, ptrs, 2, 0, 512, fake, 1024, err, None)
    assert rc == 1 and b"n <= stride" in L.spb_last_error()
    unaligned = (C.c_void_p * 2)(256, 520)
    rc = L.spb_allreduce_peer(fake, unaligned, ptrs, 2, 0, 1024, fake, 1024, err, None)
    assert rc == 1 and b"aligned" in L.spb_last_error()
    rc = L.spb_peer_export(None, None)
    assert rc == 1


def test_python_wrappers_refuse_cpu_tensors(spb):
    import torch
    x = torch.zeros(2, 64)
    with pytest.raises(spb.SpbError):
        spb.ffn_forward(x, x, x, x, x)


def test_library_quantizer_matches_oracle(spb, oracle_mod):
    """Host-side spb_quantize produces the oracle's ggml bytes exactly."""
    import numpy as np
    rng = np.random.default_rng(31)
    w = (rng.standard_normal((40, 256)) * 0.02).astype(np.float32)
    w[0, :32] = 0.0                  # all-zero block (scale 0)
    w[1, :32] = 0.5                  # constant block
    w[2, 5] = -3.0                   # negative extreme sets the Q4_0 scale sign
    for qt, code in ((8, spb.W_Q8_0), (4, spb.W_Q4_0)):
        np.testing.assert_array_equal(spb.quantize(w, code), oracle_mod.quantize(w, qt))
        assert spb.lib().spb_weight_row_bytes(code, 4096) == (4096 if qt == 8 else 2048) + 256


def test_product_library_has_no_debug_hooks(spb):
    """The failure-injection hooks exist only in the test-hook build."""
    assert not hasattr(spb.lib(), "spb_debug_config")
    names = _declared("spb_debug.h", r"\b(spb_[a-z0-9_]+)\s*\(")
    assert names == ["spb_debug_config"]
    for n in names:
        assert hasattr(spb.debug_lib(), n)


def test_tensor_path_rejects_before_launch(spb):
    """Requests the tensor path cannot serve fail on the host, before any launch."""
    L = spb.lib()
    fake = C.c_void_p(256)
    # f above 32768 neurons (1024 bit words of union)
    rc = L.spb_ffn_forward(fake, fake, fake, 0, fake, fake, 8, 4096, 32769, 0, 1, 2, fake, None, None, fake,
                           1 << 40, None)
    assert rc == 4 and b"f > 32768" in L.spb_last_error()
    # d not a multiple of 256
    rc = L.spb_ffn_forward(fake, fake, fake, 0, fake, fake, 8, 384, 1024, 0, 1, 2, fake, None, None, fake,
                           1 << 40, None)
    assert rc == 1 and b"d % 256" in L.spb_last_error()
    # more than 256 tokens
    rc = L.spb_ffn_forward(fake, fake, fake, 1, fake, fake, 257, 4096, 1024, 0, 1, 2, fake, None, None, fake,
                           1 << 40, None)
    assert rc == 4 and b"B > 256" in L.spb_last_error()
