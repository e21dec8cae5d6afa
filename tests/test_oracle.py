"""CPU tests of the oracle itself: pinned against the reference's own code
(golden fixtures from naive_sparsity_div, and the compiled reference library
when present) and against independent numpy restatements."""
import numpy as np
import pytest

from conftest import golden_union_cases, assert_close


def _flatten(merge, counts):
    return np.concatenate([merge[g, :counts[g]] for g in range(len(counts))])


@pytest.mark.parametrize("case", list(golden_union_cases()), ids=lambda c: c[0])
def test_union_matches_reference_golden(oracle_mod, case):
    name, lab, counts, flat = case
    merge, cnt = oracle_mod.union(lab, 8)
    groups = lab.shape[0] // 8
    np.testing.assert_array_equal(cnt[:groups], counts)
    np.testing.assert_array_equal(_flatten(merge, cnt[:groups]), flat)


def test_union_matches_compiled_reference(oracle_mod):
    if oracle_mod.ref_lib() is None:
        pytest.skip("reference library not built here")
    rng = np.random.default_rng(7)
    for B, f in [(8, 32), (16, 1000 // 32 * 32), (64, 11008)]:
        lab = (rng.random((B, f)) < 0.07).astype(np.float32) - (rng.random((B, f)) < 0.3)
        m_ref, c_ref = oracle_mod.ref_naive_sparsity_div(lab)
        m, c = oracle_mod.union(lab, 8)
        np.testing.assert_array_equal(c, c_ref)
        for g in range(B // 8):
            np.testing.assert_array_equal(m[g, :c[g]], m_ref[g, :c[g]])


def test_union_whole_batch_and_ragged(oracle_mod):
    rng = np.random.default_rng(3)
    lab = (rng.random((5, 77)) < 0.2).astype(np.float32)
    m, c = oracle_mod.union(lab, 5)
    want = np.nonzero((lab > 0).any(0))[0]
    assert c[0] == len(want)
    np.testing.assert_array_equal(m[0, :c[0]], want)
    m, c = oracle_mod.union(lab, 2)  # segments of 2, last one short
    assert len(c) == 3
    np.testing.assert_array_equal(m[2, :c[2]], np.nonzero(lab[4] > 0)[0])


def test_token_bits(oracle_mod):
    rng = np.random.default_rng(4)
    lab = rng.standard_normal((3, 70)).astype(np.float32)
    bits = oracle_mod.token_bits(lab)
    for t in range(3):
        for j in range(70):
            assert bool((bits[t, j // 32] >> (j % 32)) & 1) == bool(lab[t, j] > 0)


def test_f16_conversion_matches_ieee(oracle_mod):
    rng = np.random.default_rng(5)
    a = (rng.standard_normal(200000) * 10.0 ** rng.integers(-9, 6, 200000)).astype(np.float32)
    a[:6] = [0.0, -0.0, np.inf, -np.inf, 65504.0, 65520.0]
    np.testing.assert_array_equal(oracle_mod.to_f16_bits(a), a.astype(np.float16).view(np.uint16))


def _numpy_ffn(wg, wu, wd, x, lab, G, per_token, act):
    B, d = x.shape
    xr = x.astype(np.float16).astype(np.float64)
    g = xr @ wg.astype(np.float64).T
    u = xr @ wu.astype(np.float64).T
    g32, u32 = g.astype(np.float32), u.astype(np.float32)
    h = np.maximum(g32, 0) * (np.maximum(u32, 0) if act == 1 else u32)
    act_mask = lab > 0
    if not per_token:
        for s in range(0, B, G):
            act_mask[s:s + G] = act_mask[s:s + G].any(0)
    h = np.where(act_mask, h, 0).astype(np.float16).astype(np.float64)
    return (h @ wd.astype(np.float64)).astype(np.float32)


@pytest.mark.parametrize("per_token,act,G", [(True, 0, 4), (False, 0, 4), (False, 1, 2), (True, 1, 4)])
def test_ffn_oracle_vs_numpy(oracle_mod, per_token, act, G):
    rng = np.random.default_rng(11)
    B, d, f = 4, 128, 256
    wg, wu, wd = ((rng.standard_normal((f, d)) * 0.05).astype(np.float16) for _ in range(3))
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = (rng.random((B, f)) < 0.2).astype(np.float32)
    got = oracle_mod.ffn(wg, wu, wd, x, lab, G=G, per_token=per_token, act=act)
    assert_close(got, _numpy_ffn(wg, wu, wd, x, lab, G, per_token, act), rtol=1e-4, atol=1e-5)


def test_compact_gemms_compose_to_ffn(oracle_mod):
    """MLP_naive composition (cuda/ffn_test.cu:144-163) equals the union FFN."""
    rng = np.random.default_rng(12)
    B, d, f = 16, 64, 128
    wg, wu, wd = ((rng.standard_normal((f, d)) * 0.1).astype(np.float16) for _ in range(3))
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = (rng.random((B, f)) < 0.1).astype(np.float32)
    merge, counts = oracle_mod.union(lab, 8)
    g = oracle_mod.up_compact(wg, x, merge, counts, 8)
    u = oracle_mod.up_compact(wu, x, merge, counts, 8)
    h = np.maximum(g, 0) * u
    out = oracle_mod.down_compact(wd, h, merge, counts, 8)
    assert_close(out, oracle_mod.ffn(wg, wu, wd, x, lab, G=8, per_token=False), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("qtype", [8, 4])
def test_quant_roundtrip_bounds(oracle_mod, qtype):
    rng = np.random.default_rng(13)
    w = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    q = oracle_mod.quantize(w, qtype)
    assert q.shape == (64, (256 if qtype == 8 else 128) + 16)
    deq = oracle_mod.dequantize(q, qtype, 256)
    blocks = np.abs(w.reshape(64, 8, 32)).max(-1, keepdims=True)
    step = blocks / (127.0 if qtype == 8 else 8.0)
    err = np.abs(deq.reshape(64, 8, 32) - w.reshape(64, 8, 32))
    # half a step of rounding (Q4_0: a full step at the clamped +8 end) plus
    # the fp16 rounding of the scale times the largest quant
    bound = step * (0.5 if qtype == 8 else 1.0) + step * (127 if qtype == 8 else 8) * 2.0 ** -11
    assert (err <= bound * 1.001 + 1e-9).all()


def test_q4_0_nibble_placement(oracle_mod):
    """Element j sits in the low nibble of byte j, element j+16 in the high
    nibble (cuda/kernel.cu:348,354-355)."""
    w = np.zeros((1, 32), np.float32)
    w[0, 3] = -8.0
    w[0, 19] = 4.0
    q = oracle_mod.quantize(w, 4)
    assert q[0, 3] & 0xF == 0 and q[0, 3] >> 4 == 12
    deq = oracle_mod.dequantize(q, 4, 32)
    assert deq[0, 3] == -8.0 and deq[0, 19] == 4.0


def test_predictor_oracle_vs_numpy(oracle_mod):
    rng = np.random.default_rng(21)
    B, d, D, f = 3, 512, 256, 1024
    p1 = (rng.standard_normal((D, d)) / np.sqrt(d)).astype(np.float16)
    p2 = (rng.standard_normal((f, D)) / np.sqrt(D)).astype(np.float16)
    x = rng.standard_normal((B, d)).astype(np.float32)
    lg, lab, idx, counts = oracle_mod.predict(p1, p2, x, k=100)
    h = np.maximum(x.astype(np.float16).astype(np.float64) @ p1.astype(np.float64).T, 0)
    ref = h.astype(np.float16).astype(np.float64) @ p2.astype(np.float64).T
    assert np.abs(ref - lg).max() < 1e-4
    assert (counts == 100).all() and (lab.sum(1) == 100).all()
    for t in range(B):
        order = np.lexsort((np.arange(f), -lg[t]))  # logit desc, id asc
        np.testing.assert_array_equal(idx[t], np.sort(order[:100]))
    _, lab0, _, c0 = oracle_mod.predict(p1, p2, x, k=0, threshold=0.0)
    np.testing.assert_array_equal(lab0, (lg >= 0).astype(np.float32))
    assert (c0 == lab0.sum(1)).all()


def test_oracle_bias_reduces_to_plain_ffn(oracle_mod):
    """With zero biases the biased oracle is the plain one; with a gate bias it
    matches a numpy restatement of add-then-activate."""
    rng = np.random.default_rng(5)
    B, d, f = 3, 64, 96
    W = [(rng.standard_normal((f, d)) * 0.1).astype(np.float16) for _ in range(3)]
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = (rng.random((B, f)) < 0.3).astype(np.float32)
    z = np.zeros(f, np.float16)
    np.testing.assert_array_equal(oracle_mod.ffn_bias(*W, x, lab, z, z), oracle_mod.ffn(*W, x, lab))
    bg = (rng.standard_normal(f) * 0.5).astype(np.float16)
    xr = x.astype(np.float16).astype(np.float64)
    g = (xr @ W[0].astype(np.float64).T).astype(np.float32) + bg.astype(np.float32)
    u = (xr @ W[1].astype(np.float64).T).astype(np.float32)
    h = (np.maximum(g, 0) * u * (lab > 0)).astype(np.float16).astype(np.float64)
    want = h @ W[2].astype(np.float64)
    np.testing.assert_allclose(oracle_mod.ffn_bias(*W, x, lab, bg, None), want, rtol=1e-5, atol=1e-5)
