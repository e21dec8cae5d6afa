"""GPU test of spb_union_static, the entry point for callers that cannot
allocate device memory (a framework allocator owns the device, a plug-in is
handed only its input and output buffers, or a latency-critical path must
not call cudaMalloc).  It must produce exactly what spb_union produces with a
caller workspace.  Two calls in a row, the second smaller than the first, also
check that scratch contents left by one call do not leak into the next.

This file is named so that pytest collects it last."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _labels(rng, B, f, p):
    return np.where(rng.random((B, f)) < p, rng.random((B, f)), -rng.random((B, f))).astype(np.float32)


def test_union_static_matches_workspace_union(spb, cuda):
    import torch
    L = spb.lib()
    rng = np.random.default_rng(2024)
    stream = torch.cuda.current_stream().cuda_stream
    # a ragged last segment (20 % 8 != 0) with no token-bits output, then a
    # smaller call on the same scratch
    for B, f, group, want_tok in [(64, 11008, 8, True), (20, 1000, 8, False), (17, 1000, 0, True)]:
        lab = torch.from_numpy(_labels(rng, B, f, 0.1)).to(cuda)
        G = B if group == 0 else group
        S = (B + G - 1) // G
        W = (f + 31) // 32
        want_merge, want_act, want_bits = spb.union(lab, group=group)
        merge = torch.full((S, f), -5, dtype=torch.int32, device=cuda)
        act = torch.full((S,), -5, dtype=torch.int32, device=cuda)
        bits = torch.zeros((B, W), dtype=torch.int32, device=cuda)
        rc = L.spb_union_static(lab.data_ptr(), B, f, group, merge.data_ptr(), act.data_ptr(),
                                bits.data_ptr() if want_tok else None, stream)
        assert rc == 0, L.spb_last_error()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(act.cpu().numpy(), want_act.cpu().numpy())
        counts = np.diff(np.concatenate([[0], act.cpu().numpy()]))
        m, wm = merge.cpu().numpy(), want_merge.cpu().numpy()
        for s in range(S):
            np.testing.assert_array_equal(m[s, :counts[s]], wm[s, :counts[s]])
        if want_tok:
            np.testing.assert_array_equal(bits.cpu().numpy(), want_bits.cpu().numpy())


def test_union_static_rejects_oversized_requests(spb, cuda):
    import torch
    L = spb.lib()
    B, f = 256, 32768  # 256 segments x 1024 words > the fixed scratch array
    lab = torch.zeros((B, f), device=cuda)
    merge = torch.zeros((B, f), dtype=torch.int32, device=cuda)
    act = torch.zeros(B, dtype=torch.int32, device=cuda)
    rc = L.spb_union_static(lab.data_ptr(), B, f, 1, merge.data_ptr(), act.data_ptr(), None,
                            torch.cuda.current_stream().cuda_stream)
    assert rc == 4 and b"scratch" in L.spb_last_error()
