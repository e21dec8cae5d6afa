"""GPU parity of the low-rank predictor.  Up to 16 tokens: logits, label
sets and ascending index lists bit-exact against the CPU oracle (both use one
fixed fp32 reduction order).  Larger batches take the tensor-core route
(fp16 GEMMs, fp32 accumulation): logits agree with the oracle's to fp32
rounding, the sets are exactly the top-k of those logits, and they differ
from the oracle's only at near-ties of the k-th logit."""
import numpy as np
import pytest

from conftest import assert_close

pytestmark = pytest.mark.gpu


def _dev(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _weights(rng, d, D, f):
    p1 = (rng.standard_normal((D, d)) / np.sqrt(d)).astype(np.float16)
    p2 = (rng.standard_normal((f, D)) / np.sqrt(D)).astype(np.float16)
    return p1, p2


def _run(spb, cuda, p1, p2, x, k, thr=0.0):
    import torch
    B, f = x.shape[0], p2.shape[0]
    D = p1.shape[0]
    P1, P2, X = _dev(p1, cuda), _dev(p2, cuda), _dev(x, cuda)
    labels = torch.empty((B, f), device=cuda)
    cap = k if k > 0 else f
    idx = torch.full((B, cap), -1, dtype=torch.int32, device=cuda)
    counts = torch.zeros(B, dtype=torch.int32, device=cuda)
    logits = torch.empty((B, f), device=cuda)
    bits = torch.full((B, (f + 31) // 32), -1, dtype=torch.int32, device=cuda)
    ws = torch.zeros(int(spb.lib().spb_predict_workspace_bytes(B, D, f)), dtype=torch.uint8, device=cuda)
    rc = spb.lib().spb_predict(P1.data_ptr(), P2.data_ptr(), X.data_ptr(), B, x.shape[1], D, f, k, thr,
                               labels.data_ptr(), bits.data_ptr(), idx.data_ptr(), counts.data_ptr(), logits.data_ptr(),
                               ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, spb.lib().spb_last_error()
    torch.cuda.synchronize()
    lab = labels.cpu().numpy()
    # the bit words hold exactly the label sets
    want_bits = np.packbits((lab > 0).astype(np.uint8), axis=1, bitorder="little")
    want_bits = np.pad(want_bits, ((0, 0), (0, (-want_bits.shape[1]) % 4))).view(np.uint32)
    np.testing.assert_array_equal(bits.cpu().numpy().view(np.uint32), want_bits)
    return logits.cpu().numpy(), lab, idx.cpu().numpy(), counts.cpu().numpy()


@pytest.mark.parametrize("B,d,D,f,k", [(1, 4096, 1024, 11008, 1101), (4, 512, 256, 1000, 100), (16, 1024, 512, 2048, 300),
                                       (2, 8192, 1024, 28672, 2867)])
def test_predict_bit_exact(spb, cuda, oracle_mod, B, d, D, f, k):
    rng = np.random.default_rng(B * 7 + f)
    p1, p2 = _weights(rng, d, D, f)
    x = rng.standard_normal((B, d)).astype(np.float32)
    g = _run(spb, cuda, p1, p2, x, k)
    want = oracle_mod.predict(p1, p2, x, k=k)
    for got, ref, name in zip(g, want, ("logits", "labels", "idx", "counts")):
        np.testing.assert_array_equal(got, ref, err_msg=name)


def _topk_of(logits, k):
    """Exact top-k per row, ties to the lower id, as 0/1 labels."""
    lab = np.zeros_like(logits, dtype=np.float32)
    ids = np.arange(logits.shape[1])
    for t in range(logits.shape[0]):
        order = np.lexsort((ids, -logits[t]))
        lab[t, order[:k]] = 1.0
    return lab


@pytest.mark.parametrize("B,d,D,f,k", [(19, 1024, 512, 2048, 300), (64, 5120, 1024, 13824, 1106),
                                       (130, 4096, 1024, 11008, 1101)])
def test_predict_tensor_route(spb, cuda, oracle_mod, B, d, D, f, k):
    rng = np.random.default_rng(B * 7 + f)
    p1, p2 = _weights(rng, d, D, f)
    x = rng.standard_normal((B, d)).astype(np.float32)
    logits, lab, idx, counts = _run(spb, cuda, p1, p2, x, k)
    lg_ref, lab_ref, _, _ = oracle_mod.predict(p1, p2, x, k=k)
    scale = np.abs(lg_ref).max()
    np.testing.assert_allclose(logits, lg_ref, rtol=2e-3, atol=2e-3 * scale)
    # the selection itself is exact on the kernel's own logits
    np.testing.assert_array_equal(lab, _topk_of(logits, k))
    assert (counts == k).all()
    for t in range(B):
        np.testing.assert_array_equal(idx[t], np.flatnonzero(lab[t] > 0))
    # and matches the oracle's sets except where logits straddle the k-th by
    # less than their rounding difference
    kth = np.sort(lg_ref, axis=1)[:, ::-1][:, k - 1:k]
    near = np.abs(lg_ref - kth) <= 4e-3 * scale
    assert ((lab != lab_ref) & ~near).sum() == 0


def test_predict_ties_go_to_lower_ids(spb, cuda, oracle_mod):
    rng = np.random.default_rng(3)
    B, d, D, f, k = 2, 512, 256, 512, 37
    p1, p2 = _weights(rng, d, D, f)
    p2[100:200] = p2[5]  # 100 neurons share one logit per token
    x = rng.standard_normal((B, d)).astype(np.float32)
    g = _run(spb, cuda, p1, p2, x, k)
    want = oracle_mod.predict(p1, p2, x, k=k)
    for got, ref in zip(g, want):
        np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("k", [0, 512])
def test_predict_threshold_and_all(spb, cuda, oracle_mod, k):
    rng = np.random.default_rng(4)
    B, d, D, f = 3, 256, 256, 512
    p1, p2 = _weights(rng, d, D, f)
    x = rng.standard_normal((B, d)).astype(np.float32)
    g = _run(spb, cuda, p1, p2, x, k, 0.0)
    want = oracle_mod.predict(p1, p2, x, k=k, threshold=0.0)
    for got, ref in zip(g, want):
        np.testing.assert_array_equal(got, ref)


def test_predict_then_ffn_config1(spb, cuda, oracle_mod):
    """Config 1: predictor picks exactly 1101 of 11008 neurons, then the sparse FFN."""
    import torch
    rng = np.random.default_rng(0)
    B, d, D, f, k = 1, 4096, 1024, 11008, 1101
    p1, p2 = _weights(rng, d, D, f)
    W = [(rng.standard_normal((f, d)) * 0.02).astype(np.float16) for _ in range(3)]
    x = rng.standard_normal((B, d)).astype(np.float32)
    labels = spb.predict(_dev(p1, cuda), _dev(p2, cuda), _dev(x, cuda), k=k)
    out = spb.ffn_forward(*[_dev(w, cuda) for w in W], _dev(x, cuda), labels)
    torch.cuda.synchronize()
    _, lab_ref, _, _ = oracle_mod.predict(p1, p2, x, k=k)
    np.testing.assert_array_equal(labels.cpu().numpy(), lab_ref)
    assert_close(out.cpu().numpy(), oracle_mod.ffn(*W, x, lab_ref))


def _to_words(lab):
    b = np.packbits((lab > 0).astype(np.uint8), axis=1, bitorder="little")
    return np.pad(b, ((0, 0), (0, (-b.shape[1]) % 4))).view(np.uint32)


@pytest.mark.parametrize("B,d,D,f,k,ties", [(1, 4096, 1024, 11008, 1101, False), (5, 512, 256, 1000, 100, False),
                                            (2, 512, 256, 512, 37, True), (16, 5120, 1024, 13824, 1106, False),
                                            (2, 8192, 1024, 28672, 2867, False)])
def test_grid_select_sets_bit_exact(spb, cuda, oracle_mod, B, d, D, f, k, ties):
    """Set outputs without an index list take the grid-wide select (threshold
    bin from the logit histogram, exact selection among its candidates):
    labels and bit words bit-exact against the oracle, ties included, on two
    calls in a row (the candidate counters reset themselves)."""
    import torch
    rng = np.random.default_rng(B * 11 + f)
    p1, p2 = _weights(rng, d, D, f)
    if ties:
        p2[100:200] = p2[5]  # 100 neurons share one logit per token
    P1, P2 = _dev(p1, cuda), _dev(p2, cuda)
    ws = spb.predict_workspace(B, D, f, cuda)
    for call in range(2):
        x = rng.standard_normal((B, d)).astype(np.float32)
        X = _dev(x, cuda)
        _, lab_ref, _, cnt_ref = oracle_mod.predict(p1, p2, x, k=k)
        bits = torch.zeros((B, (f + 31) // 32), dtype=torch.int32, device=cuda)
        labels = spb.predict(P1, P2, X, k=k, bits_out=bits, workspace=ws)
        bits_only = torch.zeros_like(bits)
        spb.predict(P1, P2, X, k=k, bits_out=bits_only, labels=False, workspace=ws)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(labels.cpu().numpy(), lab_ref, err_msg=f"labels, call {call}")
        np.testing.assert_array_equal(bits.cpu().numpy().view(np.uint32), _to_words(lab_ref), err_msg="bits")
        np.testing.assert_array_equal(bits_only.cpu().numpy().view(np.uint32), _to_words(lab_ref), err_msg="bits")


@pytest.mark.parametrize("B,d,D,f,k,ties", [(1, 4096, 1024, 11008, 1101, "none"), (3, 1024, 512, 4096, 400, "none"),
                                            (1, 512, 256, 512, 37, "some"), (1, 512, 256, 2048, 100, "all"),
                                            (1, 5120, 1024, 13824, 1106, "none"), (1, 1024, 256, 1000, 97, "none")])
def test_set_outputs_without_index_list(spb, cuda, oracle_mod, B, d, D, f, k, ties):
    """Set outputs with no index list: at one token the one-launch predictor
    (P2 slices resident in shared memory, exact top-k in the same launch),
    otherwise the launch chain.  Logits, labels, bit words and counts
    bit-exact against the oracle, on two calls in a row, including a row
    where every logit ties (the k lowest ids win) and slices that f does
    not divide evenly."""
    import torch
    rng = np.random.default_rng(B * 13 + f)
    p1, p2 = _weights(rng, d, D, f)
    if ties == "some":
        p2[100:200] = p2[5]
    elif ties == "all":
        p2[:] = p2[0]
    P1, P2 = _dev(p1, cuda), _dev(p2, cuda)
    ws = spb.predict_workspace(B, D, f, cuda)
    for call in range(2):
        x = rng.standard_normal((B, d)).astype(np.float32)
        lg_ref, lab_ref, _, cnt_ref = oracle_mod.predict(p1, p2, x, k=k)
        X = _dev(x, cuda)
        labels = torch.full((B, f), -1.0, device=cuda)
        bits = torch.full((B, (f + 31) // 32), -1, dtype=torch.int32, device=cuda)
        counts = torch.zeros(B, dtype=torch.int32, device=cuda)
        logits = torch.empty((B, f), device=cuda)
        rc = spb.lib().spb_predict(P1.data_ptr(), P2.data_ptr(), X.data_ptr(), B, d, D, f, k, 0.0,
                                   labels.data_ptr(), bits.data_ptr(), None, counts.data_ptr(), logits.data_ptr(),
                                   ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
        assert rc == 0, spb.lib().spb_last_error()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(logits.cpu().numpy(), lg_ref, err_msg=f"logits, call {call}")
        np.testing.assert_array_equal(labels.cpu().numpy(), lab_ref, err_msg=f"labels, call {call}")
        np.testing.assert_array_equal(bits.cpu().numpy().view(np.uint32), _to_words(lab_ref), err_msg="bits")
        np.testing.assert_array_equal(counts.cpu().numpy(), cnt_ref, err_msg="counts")
