"""GPU parity of the fused sparse-FFN path against the CPU oracle
(rel 1e-2 / abs 1e-3 for fp16 weights with fp32 accumulation; union
indices bit-exact)."""
import numpy as np
import pytest

from conftest import assert_close, assert_close_70b
from spbatch_b200.workload import zipf_active_labels

pytestmark = pytest.mark.gpu


def _dev(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _layer(rng, d, f, std=0.02):
    return [(rng.standard_normal((f, d)) * std).astype(np.float16) for _ in range(3)]


def _run(spb, cuda, wg, wu, wd, x, lab, **kw):
    import torch
    f = lab.shape[1]
    merge = torch.full((f,), -1, dtype=torch.int32, device=cuda)
    count = torch.zeros(1, dtype=torch.int32, device=cuda)
    ws = spb.new_workspace(x.shape[0], x.shape[1], f, 0, cuda)
    out = spb.ffn_forward(_dev(wg, cuda), _dev(wu, cuda), _dev(wd, cuda), _dev(x, cuda), _dev(lab, cuda),
                          merge_idx_out=merge, count_out=count, workspace=ws, **kw)
    torch.cuda.synchronize()
    assert _ws_error(ws) == 0, "device wait timed out"
    return out.cpu().numpy(), merge.cpu().numpy(), int(count.cpu()[0])


@pytest.mark.parametrize("B", [1, 2, 3, 4])
@pytest.mark.parametrize("per_token", [True, False])
def test_gemv_path_small(spb, cuda, oracle_mod, B, per_token):
    rng = np.random.default_rng(100 + B)
    d, f = 256, 640
    wg, wu, wd = _layer(rng, d, f, 0.05)
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = (rng.random((B, f)) < 0.15).astype(np.float32)
    out, merge, U = _run(spb, cuda, wg, wu, wd, x, lab, per_token_mask=per_token, path=spb.PATH_GEMV)
    want = oracle_mod.ffn(wg, wu, wd, x, lab, per_token=per_token)
    assert_close(out, want)
    m_ref, c_ref = oracle_mod.union(lab, B)
    assert U == c_ref[0]
    np.testing.assert_array_equal(merge[:U], m_ref[0, :U])


@pytest.mark.parametrize("act", [0, 1])
def test_gemv_path_7b_b1(spb, cuda, oracle_mod, act):
    """Config 1 shape: 7B layer, one token, exactly 1101 active neurons."""
    rng = np.random.default_rng(0)
    d, f = 4096, 11008
    wg, wu, wd = _layer(rng, d, f)
    x = rng.standard_normal((1, d)).astype(np.float32)
    lab = zipf_active_labels(1, f, 1101, seed=0)
    out, merge, U = _run(spb, cuda, wg, wu, wd, x, lab, act=act, path=spb.PATH_GEMV)
    assert U == 1101
    np.testing.assert_array_equal(merge[:U], np.nonzero(lab[0])[0])
    assert_close(out, oracle_mod.ffn(wg, wu, wd, x, lab, act=act))


@pytest.mark.parametrize("B", [2, 4])
def test_gemv_path_13b_zipf(spb, cuda, oracle_mod, B):
    rng = np.random.default_rng(1)
    d, f = 5120, 13824
    wg, wu, wd = _layer(rng, d, f)
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = zipf_active_labels(B, f, 1106, seed=1)
    out, merge, U = _run(spb, cuda, wg, wu, wd, x, lab, path=spb.PATH_GEMV)
    assert_close(out, oracle_mod.ffn(wg, wu, wd, x, lab))


def test_empty_union_gives_zero(spb, cuda):
    rng = np.random.default_rng(2)
    d, f = 512, 1024
    wg, wu, wd = _layer(rng, d, f)
    x = rng.standard_normal((2, d)).astype(np.float32)
    lab = np.zeros((2, f), np.float32)
    out, _, U = _run(spb, cuda, wg, wu, wd, x, lab, path=spb.PATH_GEMV)
    assert U == 0 and not out.any()


def test_repeated_calls_reuse_workspace(spb, cuda, oracle_mod):
    """Workspace contents from one call must not leak into the next."""
    import torch
    rng = np.random.default_rng(3)
    d, f = 1024, 2048
    wg, wu, wd = _layer(rng, d, f)
    ws = spb.new_workspace(4, d, f, 0, cuda)
    W = [_dev(w, cuda) for w in (wg, wu, wd)]
    for it in range(3):
        B = [4, 1, 3][it]
        x = rng.standard_normal((B, d)).astype(np.float32)
        lab = (rng.random((B, f)) < [0.3, 0.01, 0.1][it]).astype(np.float32)
        out = spb.ffn_forward(*W, _dev(x, cuda), _dev(lab, cuda), workspace=ws, path=spb.PATH_GEMV)
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), oracle_mod.ffn(wg, wu, wd, x, lab))


def _ws_error(ws):
    """The workspace's sticky device error code (first 4 bytes)."""
    return int(np.frombuffer(ws[:4].cpu().numpy().tobytes(), np.uint32)[0])


def _run_ws(spb, cuda, W, x, lab, **kw):
    """Like _run but with an explicit workspace, also returning its error word."""
    import torch
    B, d = x.shape
    f = lab.shape[1]
    ws = spb.new_workspace(B, d, f, 0, cuda)
    ws.zero_()
    merge = torch.full((f,), -1, dtype=torch.int32, device=cuda)
    count = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = spb.ffn_forward(*[_dev(w, cuda) for w in W], _dev(x, cuda), _dev(lab, cuda), merge_idx_out=merge,
                          count_out=count, workspace=ws, **kw)
    torch.cuda.synchronize()
    return out.cpu().numpy(), merge.cpu().numpy(), int(count.cpu()[0]), _ws_error(ws)


@pytest.mark.parametrize("B", [1, 5, 16, 33])
def test_tensor_path_small_shapes(spb, cuda, oracle_mod, B):
    rng = np.random.default_rng(200 + B)
    d, f = 256, 1024
    W = _layer(rng, d, f, 0.05)
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = (rng.random((B, f)) < 0.08).astype(np.float32)
    out, merge, U, err = _run_ws(spb, cuda, W, x, lab, path=spb.PATH_TENSOR)
    assert err == 0
    m_ref, c_ref = oracle_mod.union(lab, B)
    assert U == c_ref[0]
    np.testing.assert_array_equal(merge[:U], m_ref[0, :U])
    assert_close(out, oracle_mod.ffn(*W, x, lab))


@pytest.mark.parametrize("B", [8, 16, 32])
def test_tensor_path_7b_zipf(spb, cuda, oracle_mod, B):
    """Config 2: 7B layer, Zipf(0.8) activity, 10% per token."""
    rng = np.random.default_rng(B)
    d, f = 4096, 11008
    W = _layer(rng, d, f)
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = zipf_active_labels(B, f, 1101, seed=B)
    out, merge, U, err = _run_ws(spb, cuda, W, x, lab, path=spb.PATH_TENSOR)
    assert err == 0
    ref_idx = np.nonzero((lab > 0).any(0))[0]
    assert U == len(ref_idx)
    np.testing.assert_array_equal(merge[:U], ref_idx)
    assert_close(out, oracle_mod.ffn(*W, x, lab))


@pytest.mark.parametrize("act", [0, 1])
def test_tensor_path_union_semantics(spb, cuda, oracle_mod, act):
    rng = np.random.default_rng(7)
    B, d, f = 24, 1024, 2048
    W = _layer(rng, d, f, 0.03)
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = zipf_active_labels(B, f, 205, seed=3)
    out, _, _, err = _run_ws(spb, cuda, W, x, lab, path=spb.PATH_TENSOR, per_token_mask=False, act=act)
    assert err == 0
    assert_close(out, oracle_mod.ffn(*W, x, lab, per_token=False, act=act))


def test_tensor_path_dense_and_large_batch(spb, cuda, oracle_mod):
    """Every neuron active (a dense control) at B=128: split-K is off (T >= grid
    would need f >= 19k), many tiles per chunk."""
    rng = np.random.default_rng(9)
    B, d, f = 128, 512, 1024
    W = _layer(rng, d, f, 0.03)
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = np.ones((B, f), np.float32)
    out, merge, U, err = _run_ws(spb, cuda, W, x, lab, path=spb.PATH_TENSOR)
    assert err == 0 and U == f
    assert_close(out, oracle_mod.ffn(*W, x, lab))


def test_tensor_path_13b_b64(spb, cuda, oracle_mod):
    """Config 3 layer shape: 13B, B=64, 8% activity."""
    rng = np.random.default_rng(13)
    B, d, f = 64, 5120, 13824
    W = _layer(rng, d, f)
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = zipf_active_labels(B, f, 1106, seed=13)
    out, merge, U, err = _run_ws(spb, cuda, W, x, lab, path=spb.PATH_TENSOR)
    assert err == 0
    assert U == int((lab > 0).any(0).sum())
    assert_close(out, oracle_mod.ffn(*W, x, lab))


@pytest.mark.parametrize("d,f,B,p", [(8192, 1000, 1, 0.1), (8192, 2048, 2, 0.2), (64, 33, 3, 0.5),
                                     (4096, 4096, 4, 1.0), (2048, 96, 4, 0.0)])
def test_stream_path_shapes(spb, cuda, oracle_mod, d, f, B, p):
    """Single-launch streaming path: ragged f, d = 8192 (two chunks per
    thread), tiny d, a fully dense union (the stage ring wraps many times),
    and an empty one; no index outputs requested."""
    import torch
    rng = np.random.default_rng(d + f + B)
    wg, wu, wd = _layer(rng, d, f, 0.05)
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = (rng.random((B, f)) < p).astype(np.float32)
    ws = spb.new_workspace(B, d, f, 0, cuda)
    out = spb.ffn_forward(_dev(wg, cuda), _dev(wu, cuda), _dev(wd, cuda), _dev(x, cuda), _dev(lab, cuda),
                          workspace=ws, path=spb.PATH_GEMV)
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), oracle_mod.ffn(wg, wu, wd, x, lab))
    assert _ws_error(ws) == 0


def test_stream_path_many_calls(spb, cuda, oracle_mod):
    """The streaming kernel's launch counters are reset by its last CTA, so
    back-to-back calls on one workspace (no host sync between them) all give
    the oracle's answer."""
    import torch
    rng = np.random.default_rng(11)
    d, f, B = 1024, 3000, 2
    wg, wu, wd = _layer(rng, d, f, 0.05)
    W = [_dev(w, cuda) for w in (wg, wu, wd)]
    ws = spb.new_workspace(B, d, f, 0, cuda)
    xs = [rng.standard_normal((B, d)).astype(np.float32) for _ in range(6)]
    labs = [(rng.random((B, f)) < 0.05 * (i + 1)).astype(np.float32) for i in range(6)]
    outs = [spb.ffn_forward(*W, _dev(x, cuda), _dev(l, cuda), workspace=ws, path=spb.PATH_GEMV)
            for x, l in zip(xs, labs)]
    torch.cuda.synchronize()
    for x, l, o in zip(xs, labs, outs):
        assert_close(o.cpu().numpy(), oracle_mod.ffn(wg, wu, wd, x, l))
    assert _ws_error(ws) == 0


def _gpu_layer(cuda, d, f, seed, std=0.02):
    """fp16 N(0, std^2) weights drawn on the GPU (fast at 70B size), with host copies for the oracle."""
    import torch
    g = torch.Generator(device=cuda)
    g.manual_seed(seed)
    Wd = [(torch.randn((f, d), generator=g, device=cuda) * std).half() for _ in range(3)]
    return Wd, [w.cpu().numpy() for w in Wd]


def _tensor_case(spb, cuda, oracle_mod, d, f, B, k, seed, check_tokens, lab=None):
    """Tensor path on (d, f, B) with Zipf activity: union bit-exact, the output
    rows of `check_tokens` against the oracle (with the per-token mask a token's
    output depends only on its own active set, so the oracle runs on those
    tokens alone)."""
    import torch
    Wd, Wh = _gpu_layer(cuda, d, f, seed)
    x = np.random.default_rng(seed).standard_normal((B, d)).astype(np.float32)
    if lab is None:
        lab = zipf_active_labels(B, f, k, seed=seed)
    ws = spb.new_workspace(B, d, f, 0, cuda)
    merge = torch.full((f,), -1, dtype=torch.int32, device=cuda)
    count = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = spb.ffn_forward(*Wd, _dev(x, cuda), _dev(lab, cuda), merge_idx_out=merge, count_out=count,
                          workspace=ws, path=spb.PATH_TENSOR)
    torch.cuda.synchronize()
    assert _ws_error(ws) == 0
    ref_idx = np.nonzero((lab > 0).any(0))[0]
    U = int(count.cpu()[0])
    assert U == len(ref_idx)
    np.testing.assert_array_equal(merge.cpu().numpy()[:U], ref_idx)
    tok = np.asarray(check_tokens)
    (assert_close_70b if d >= 8192 else assert_close)(out.cpu().numpy()[tok], oracle_mod.ffn(*Wh, x[tok], lab[tok]))
    return U


@pytest.mark.parametrize("B", [16, 32])
def test_tensor_path_70b_zipf(spb, cuda, oracle_mod, B):
    """Config 5 layer (d=8192, f=28672), 10% Zipf activity: the union spans
    ~150-190 tiles, so every cluster walks two or three tiles."""
    U = _tensor_case(spb, cuda, oracle_mod, 8192, 28672, B, 2867, 70 + B, [0, B // 2 + 1, B - 1])
    assert U > 74 * 128  # more than one tile per cluster of two SMs


def test_tensor_path_70b_b256(spb, cuda, oracle_mod):
    """Largest config-5 batch: N = 256 (the MMA's widest tile), union dense."""
    U = _tensor_case(spb, cuda, oracle_mod, 8192, 28672, 256, 2867, 256, [0, 129, 255])
    assert U == 28672


@pytest.mark.parametrize("B", [128, 200, 256])
def test_tensor_path_wide_batches(spb, cuda, oracle_mod, B):
    """N = 128 / 208 / 256 at a small layer with a fully dense union."""
    lab = np.ones((B, 4096), np.float32)
    _tensor_case(spb, cuda, oracle_mod, 1024, 4096, B, 0, 500 + B, [0, B // 3, B - 1], lab=lab)


def test_tensor_path_7b_b64_b128(spb, cuda, oracle_mod):
    for B in (64, 128):
        _tensor_case(spb, cuda, oracle_mod, 4096, 11008, B, 1101, 640 + B, [0, B - 1])


def test_tensor_path_tiny_union(spb, cuda, oracle_mod):
    """Fewer active neurons than clusters: most clusters own nothing."""
    B, f = 8, 4096
    lab = np.zeros((B, f), np.float32)
    lab[:, [3, 700, 701, 4000, 4095]] = 1.0
    lab[5, 9] = 1.0
    _tensor_case(spb, cuda, oracle_mod, 512, f, B, 0, 77, list(range(B)), lab=lab)


@pytest.mark.parametrize("B", [5, 6, 7])
@pytest.mark.parametrize("wtype", [1, 2])
def test_quantised_token_groups_ragged(spb, cuda, oracle_mod, B, wtype):
    """Quantised batches above the streaming kernel's 4 tokens run as one
    launch per token group; ragged last group (B % 4 != 0, B = 5 leaves a
    one-token group) and ragged f, all launches sharing one workspace."""
    import torch
    rng = np.random.default_rng(900 + B + wtype)
    d, f = 1024, 2050
    Wf = [(rng.standard_normal((f, d)) * 0.02).astype(np.float32) for _ in range(3)]
    qt = 8 if wtype == 1 else 4
    Q = [spb.quantize(w, wtype) for w in Wf]
    Wdq = [oracle_mod.dequantize(q, qt, d) for q in Q]
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = zipf_active_labels(B, f, 205, seed=B)
    ws = spb.new_workspace(B, d, f, 0, cuda)
    out = spb.ffn_forward(*[_dev(q, cuda) for q in Q], _dev(x, cuda), _dev(lab, cuda), wtype=wtype, workspace=ws,
                          path=spb.PATH_GEMV)
    torch.cuda.synchronize()
    assert _ws_error(ws) == 0
    assert_close(out.cpu().numpy(), oracle_mod.ffn_f32w(*Wdq, x, lab))


@pytest.mark.parametrize("B", [3, 4])
def test_gemv_70b_token_groups(spb, cuda, oracle_mod, B):
    """fp16 d=8192 with B > 2 runs as two-token streaming launches (a ragged
    one-token tail at B = 3); ragged f."""
    import torch
    rng = np.random.default_rng(950 + B)
    d, f = 8192, 3001
    W = _layer(rng, d, f)
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = zipf_active_labels(B, f, 300, seed=B)
    ws = spb.new_workspace(B, d, f, 0, cuda)
    out = spb.ffn_forward(*[_dev(w, cuda) for w in W], _dev(x, cuda), _dev(lab, cuda), workspace=ws,
                          path=spb.PATH_GEMV)
    torch.cuda.synchronize()
    assert _ws_error(ws) == 0
    assert_close(out.cpu().numpy(), oracle_mod.ffn(*W, x, lab))


def _to_bits(lab):
    """[B][f] labels -> [B][ceil(f/32)] int32 bit words (bit j % 32 of word j / 32)."""
    b = np.packbits((lab > 0).astype(np.uint8), axis=1, bitorder="little")
    b = np.pad(b, ((0, 0), (0, (-b.shape[1]) % 4)))
    return np.ascontiguousarray(b.view(np.int32))


@pytest.mark.parametrize("B,d,f,path", [(1, 4096, 11008, 1), (3, 1024, 2050, 1), (4, 8192, 3001, 1),
                                        (6, 1024, 2050, 1), (8, 4096, 11008, 2), (32, 4096, 11008, 2),
                                        (33, 1024, 1000, 2), (64, 1024, 4096, 2)])
def test_bits_input_matches_labels(spb, cuda, oracle_mod, B, d, f, path):
    """spb_ffn_forward_bits gives spb_ffn_forward's results (union exact,
    outputs within tolerance of the oracle) on every path: streaming
    (B <= 4), token groups (d = 8192 with B > 2, B > 4), tensor cores."""
    import torch
    rng = np.random.default_rng(1000 + B + f)
    W = _layer(rng, d, f, 0.02 if d >= 4096 else 0.04)
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = zipf_active_labels(B, f, max(1, f // 10), seed=B + f)
    Wd = [_dev(w, cuda) for w in W]
    outs = []
    for sets in ("labels", "bits"):
        ws = spb.new_workspace(B, d, f, 0, cuda)
        merge = torch.full((f,), -1, dtype=torch.int32, device=cuda)
        count = torch.zeros(1, dtype=torch.int32, device=cuda)
        kw = dict(idx=_dev(lab, cuda)) if sets == "labels" else dict(bits=_dev(_to_bits(lab), cuda))
        want_idx = path == 2  # index outputs: tensor path (the streaming path writes them too for B <= 4)
        out = spb.ffn_forward(*Wd, _dev(x, cuda), **kw, path=path, workspace=ws,
                              merge_idx_out=merge if want_idx else None, count_out=count if want_idx else None)
        torch.cuda.synchronize()
        assert _ws_error(ws) == 0
        if want_idx:
            ref_idx = np.nonzero((lab > 0).any(0))[0]
            U = int(count.cpu()[0])
            assert U == len(ref_idx)
            np.testing.assert_array_equal(merge.cpu().numpy()[:U], ref_idx)
        outs.append(out.cpu().numpy())
    want = oracle_mod.ffn(*W, x, lab)
    (assert_close_70b if d >= 8192 else assert_close)(outs[0], want)
    (assert_close_70b if d >= 8192 else assert_close)(outs[1], want)


@pytest.mark.parametrize("B,d,f,path,which", [(1, 4096, 11008, 1, "both"), (3, 1024, 2050, 1, "gate"),
                                              (6, 1024, 2050, 1, "up"), (8, 1024, 4096, 2, "both"),
                                              (32, 4096, 11008, 2, "both"), (64, 1024, 4096, 2, "gate")])
def test_bias_in_fused_epilogues(spb, cuda, oracle_mod, B, d, f, path, which):
    """Sparse bias add (add_sparse_cuda, cuda/kernel.cu:818-830) fused into
    every path: streaming (B <= 4), token groups / fallback GEMV (B = 6 with
    the index outputs requested), tensor cores; labels and bit-word input."""
    import torch
    rng = np.random.default_rng(3000 + B + f)
    W = _layer(rng, d, f, 0.02 if d >= 4096 else 0.04)
    x = rng.standard_normal((B, d)).astype(np.float32)
    lab = zipf_active_labels(B, f, max(1, f // 10), seed=7 * B)
    bg = (rng.standard_normal(f) * 0.5).astype(np.float16) if which in ("both", "gate") else None
    bu = (rng.standard_normal(f) * 0.5).astype(np.float16) if which in ("both", "up") else None
    want = oracle_mod.ffn_bias(*W, x, lab, bg, bu)
    Wd = [_dev(w, cuda) for w in W]
    for sets in ("labels", "bits"):
        ws = spb.new_workspace(B, d, f, 0, cuda)
        kw = dict(idx=_dev(lab, cuda)) if sets == "labels" else dict(bits=_dev(_to_bits(lab), cuda))
        merge = torch.empty(f, dtype=torch.int32, device=cuda) if B == 6 else None  # B = 6: the fallback GEMV
        out = spb.ffn_forward(*Wd, _dev(x, cuda), **kw, path=path, workspace=ws, merge_idx_out=merge,
                              bias_gate=None if bg is None else _dev(bg, cuda),
                              bias_up=None if bu is None else _dev(bu, cuda))
        torch.cuda.synchronize()
        assert _ws_error(ws) == 0
        assert_close(out.cpu().numpy(), want)
